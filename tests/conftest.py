"""Shared helpers of the parity tests.

The parity bar is bit-exactness: every observation, reward and done flag of every step, and every
environment's GRF state bytes, equal the reference's (its published digests in
tests/golden/digests.json, and its CPU backend built from source into oracle/_ref, run live).
"""

import hashlib
import json
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, 'tests', 'golden', 'digests.json')
DATA = os.path.join(ROOT, 'cuju_b200', 'data')
ANIMATIONS = os.path.join(DATA, 'animations.bin')


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (a B200) and the built library')


def golden():
    with open(GOLDEN, encoding='utf-8') as handle:
        return json.load(handle)


def actions_at(step, environments, agents, action_count):
    """The actions of a step from integer arithmetic alone (cuju tests/conftest.py:60-66)."""
    return [[(step * 7 + e * 3 + a * 5) % action_count for a in range(agents)] for e in range(environments)]


def resolve(assets):
    """Bundle paths and per-bundle agent counts of an asset name or list of names."""
    from cuju_b200.environment import resolve_asset

    names = [assets] if isinstance(assets, str) else list(assets)
    resolved = [resolve_asset(n) for n in names]
    return [p for p, _ in resolved], [c for _, c in resolved]


def tensor_bytes(tensor):
    """The bytes of an observation; a dict of arrays (the raw representation) in name order, as
    the reference's digest reads it."""
    if isinstance(tensor, dict):
        return b''.join(tensor_bytes(tensor[name]) for name in sorted(tensor))
    tensor = tensor.detach().to('cpu').contiguous()
    return tensor.numpy().tobytes()


def device_digest(assets, steps, seed=7, environments=4, **options):
    """The golden digest of a run of the B200 batch (cuju tests/conftest.py:69-99)."""
    from cuju_b200 import BatchEnvironment

    batch = BatchEnvironment(assets, environment_count=environments, seed=seed, **options)
    digest = hashlib.sha256()
    digest.update(tensor_bytes(batch.reset()))
    for step in range(steps):
        actions = torch.tensor(actions_at(step, environments, batch.agents, batch.action_count), dtype=torch.int32)
        observation, reward, done, _ = batch.step(actions.cuda())
        digest.update(tensor_bytes(observation))
        digest.update(tensor_bytes(reward))
        digest.update(tensor_bytes(done))
    if not batch.stacked:
        for index in range(environments):
            digest.update(batch.get_state(index))
    batch.close()
    return digest.hexdigest()


def oracle_digest(assets, steps, seed=7, environments=4, library=None, **options):
    """The same digest from the reference CPU backend (oracle/_ref/libcuju_cpu.so), or from another
    library with its C-ABI that runs on the host (`library`)."""
    import struct

    from cuju_b200.environment import pickle_episode
    from oracle.driver import OracleBatch

    paths, counts = resolve(assets)
    checkpoints = 'checkpoints' in options.get('rewards', '')
    stack = 4 if options.get('stacked') else 1
    representation = {'simple115': 1, 'simple115v2': 2, 'extracted': 4, 'raw': 8}[options.get('representation', 'simple115v2')]
    batch = OracleBatch(paths, counts, environments, seed, ANIMATIONS, checkpoints=checkpoints, stack=stack,
                        assignment=options.get('assignment'), representation=representation, library=library)
    digest = hashlib.sha256()
    digest.update(batch.reset()[0])
    for step in range(steps):
        flat = [x for row in actions_at(step, environments, batch.agents, 19) for x in row]
        obs, reward, done, _ = batch.step(flat)
        digest.update(obs)
        digest.update(reward)
        digest.update(done)
    if stack == 1:
        for index in range(environments):
            match, episode = batch.engine_state(index)
            collected = episode[3:3 + batch.agents] if checkpoints else None
            data = pickle_episode(episode[:3], collected)
            digest.update(struct.pack('<i', len(data)) + data + match)
    batch.close()
    return digest.hexdigest()


def simple115_cases():
    """The golden cases of the representations this backend writes."""
    cases = golden()['cases']
    return sorted(name for name, case in cases.items()
                  if case['options'].get('representation') in (None, 'simple115v2', 'simple115', 'extracted', 'raw'))


needs_data = pytest.mark.skipif(not os.path.isfile(ANIMATIONS), reason='run __graft_entry__.build() to stage the data')


@pytest.fixture(scope='session')
def host_library(tmp_path_factory):
    """The library built for the host from tests/host/hostsim.cu (test infrastructure: the C-ABI and
    the simulation source with host memory and a serial loop in place of each kernel)."""
    import shutil
    import subprocess

    nvcc = shutil.which('nvcc') or '/usr/local/cuda/bin/nvcc'
    if not os.path.isfile(nvcc):
        pytest.skip('nvcc is needed to build the host harness')
    out = str(tmp_path_factory.mktemp('hostsim') / 'libhostsim.so')
    subprocess.run([nvcc, '-std=c++17', '-O2', '--fmad=false', '-prec-div=true', '-prec-sqrt=true', '-ftz=false',
                    '-Xcompiler', '-ffp-contract=off,-fPIC,-fvisibility=hidden',
                    '-I', os.path.join(ROOT, 'cuju_b200', 'csrc'), '-shared',
                    os.path.join(ROOT, 'tests', 'host', 'hostsim.cu'), '-o', out], check=True, capture_output=True)
    return out


LIBM_NAMES = {0: 'sinf', 1: 'cosf', 2: 'powf', 3: 'acosf', 4: 'asinf', 5: 'atanf', 6: 'atan2f', 7: 'sin', 8: 'cos',
              9: 'acos', 10: 'pow', 11: 'sincosf sine', 12: 'sincosf cosine', 13: 'powf, positive base'}


def libm_inputs(which, count=20000):
    """Seeded arguments (x, y) for the math function `which` (numbering of tests/host/libm_eval.cuh):
    special values, the ranges the simulation uses, and wide magnitudes. Arguments of the float
    functions are exactly representable floats."""
    import math
    import random
    import struct

    rng = random.Random(1000 + which)
    single = which in (0, 1, 2, 3, 4, 5, 6, 11, 12, 13)

    def rnd(v):
        return struct.unpack('<f', struct.pack('<f', v))[0] if single and math.isfinite(v) and abs(v) < 3.4e38 else v

    def wide(lo, hi):
        return rng.choice((-1.0, 1.0)) * 10.0 ** rng.uniform(lo, hi)

    special = [0.0, -0.0, 1.0, -1.0, 0.5, -0.5, 2.0, -2.0, math.pi / 4, math.pi / 2, math.pi, 2 ** -12, 1e-30,
               -1e-30, 1e-42, 1e3, 1e6, 3e7, 1e20, 3e38, math.inf, -math.inf, math.nan]
    xs, ys = [], []
    if which in (2, 10):
        for a in special:
            for b in (0.0, -0.0, 1.0, -1.0, 2.0, 3.0, 0.5, -0.5, 2.5, 1e10, math.inf, -math.inf, math.nan):
                xs.append(a)
                ys.append(b)
        span = (-6, 4) if which == 2 else (-8, 8)
        for _ in range(count):
            xs.append(10.0 ** rng.uniform(*span) * (1.0 if rng.random() < 0.9 else -1.0))
            ys.append(rng.uniform(-8, 8) if which == 2 else rng.uniform(-20, 20))
            if rng.random() < 0.1:
                ys[-1] = float(round(ys[-1]))
    elif which == 13:
        for _ in range(count):
            xs.append(rng.uniform(0, 1) if rng.random() < 0.7 else rng.uniform(0, 100))
            ys.append(rng.uniform(0.05, 4))
        xs += [0.0, 1.0, 0.0, 1.0]
        ys += [0.7, 0.8, 1.5, 2.6]
    elif which == 6:
        for a in special:
            for b in special:
                xs.append(a)
                ys.append(b)
        for _ in range(count):
            xs.append(rng.uniform(-100, 100))
            ys.append(rng.uniform(-100, 100))
    else:
        xs = list(special)
        if which in (3, 4, 9):
            xs += [rng.uniform(-1.05, 1.05) for _ in range(count)] + [1 - 2 ** -24, -(1 - 2 ** -24)]
        else:
            xs += [rng.uniform(-10, 10) for _ in range(count)]
            xs += [rng.uniform(-1e4, 1e4) for _ in range(count // 4)]
            xs += [wide(-10, 38 if single else 300) for _ in range(count // 4)]
        ys = [0.0] * len(xs)
    return [rnd(v) for v in xs], [rnd(v) for v in ys]


def libm_compare(evaluate, which, xs, ys):
    """Evaluates the library's and the reference's function on the same arguments and returns the
    first argument pair whose results differ in any bit (any NaN equals any NaN), or None."""
    import ctypes
    import math
    import struct

    units_path = os.path.join(ROOT, 'oracle', '_ref', 'liboracle_units.so')
    if not os.path.isfile(units_path):
        pytest.skip('run make -C oracle for the unit shim')
    units = ctypes.CDLL(units_path)
    n = len(xs)
    arr = ctypes.c_double * n
    x, y, mine, ref = arr(*xs), arr(*ys), arr(), arr()
    assert evaluate(which, x, y, mine, n) == 0
    assert units.oracle_libm(which, x, y, ref, n) == 0
    for i in range(n):
        a, b = mine[i], ref[i]
        if math.isnan(a) and math.isnan(b):
            continue
        if struct.pack('<d', a) != struct.pack('<d', b):
            return xs[i], ys[i], a, b
    return None
