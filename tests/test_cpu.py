"""CPU checks: the oracle against the reference's golden digests, the C-ABI library's exports, and
the host-side logic of the Python mirror. No GPU is needed."""

import ctypes
import os
import re

import pytest

from conftest import ROOT, golden, needs_data, oracle_digest

HEADER = os.path.join(ROOT, 'include', 'cuju_b200.h')
LIBRARY = os.path.join(ROOT, 'cuju_b200', 'lib', 'libcuju_b200.so')
ORACLE = os.path.join(ROOT, 'oracle', '_ref', 'libcuju_cpu.so')


def declared_symbols():
    with open(HEADER, encoding='utf-8') as handle:
        text = handle.read()
    return sorted(set(re.findall(r'\b(cuju_[a-z0-9_]+)\s*\(', text)))


def test_header_declares_the_reference_entry_points():
    names = declared_symbols()
    for required in ('cuju_environment_create', 'cuju_environment_step', 'cuju_environment_reset',
                     'cuju_environment_reset_masked', 'cuju_environment_get_state', 'cuju_environment_buffer',
                     'cuju_last_error', 'cuju_backend'):
        assert required in names


@pytest.mark.skipif(not os.path.isfile(LIBRARY), reason='library not built')
def test_library_loads_and_exports_every_declared_symbol():
    library = ctypes.CDLL(LIBRARY)
    missing = [name for name in declared_symbols() if not hasattr(library, name)]
    assert missing == []
    library.cuju_backend.restype = ctypes.c_char_p
    assert library.cuju_backend() == b'cuda'


@pytest.mark.skipif(not os.path.isfile(LIBRARY), reason='library not built')
def test_library_rejects_a_wrong_configuration_version_without_a_device():
    from cuju_b200 import _native

    library = _native.declare(ctypes.CDLL(LIBRARY))
    config = _native.Configuration(version=1)
    assert not library.cuju_environment_create(ctypes.byref(config))
    assert b'configuration version 2' in library.cuju_last_error()


def test_pickle_of_the_episode_logic_is_grf_protocol_2():
    import pickle

    from cuju_b200.environment import pickle_episode

    class EnvState:
        pass

    class Unpickler(pickle.Unpickler):
        def find_class(self, module, name):
            assert (module, name) == ('gfootball.env.football_env_core', 'EnvState')
            return EnvState

    import io

    data = Unpickler(io.BytesIO(pickle_episode([1, 0, -1], [0, 3]))).load()
    assert data['FootballEnvCore'].__dict__ == {'previous_score_diff': 1, 'previous_game_mode': 0,
                                                'prev_ball_owned_team': -1}
    assert data['CheckpointRewardWrapper'] == {1: 3}


@needs_data
def test_asset_names_resolve_to_bundles_and_agent_counts():
    from cuju_b200.environment import resolve_asset

    path, counts = resolve_asset('5_vs_5_l4_r0')
    assert path.endswith('5_vs_5_l0_r0.cjb') and counts == (4, 0)
    path, counts = resolve_asset('academy_corner')
    assert path.endswith('academy_corner_l0_r0.cjb') and counts == (1, 0)
    with pytest.raises(FileNotFoundError):
        resolve_asset('no_such_scenario_l1_r0')


# The oracle (the reference CPU backend built from source) reproduces the reference's published
# digests: the pin of every parity test. A sample that runs in seconds; the rest run on the GPU box.
ORACLE_CASES = ['5_vs_5/simple115v2', 'academy_empty_goal_close/simple115v2', '1_vs_1_easy/simple115v2',
                'mixed', '11_vs_11_stochastic/checkpoints', '5_vs_5/stacked', '5_vs_5/extracted', '5_vs_5/raw']


@needs_data
@pytest.mark.skipif(not os.path.isfile(ORACLE), reason='oracle not built')
@pytest.mark.parametrize('case', ORACLE_CASES)
def test_oracle_matches_the_golden_digest(case):
    g = golden()
    entry = g['cases'][case]
    assert oracle_digest(entry['assets'], g['steps'], seed=g['seed'], environments=g['environments'],
                         **entry['options']) == entry['digest']


@needs_data
@pytest.mark.skipif(not os.path.isfile(ORACLE), reason='oracle not built')
def test_a_planted_difference_changes_the_oracle_digest():
    # The digest is sensitive: one more step, or another seed, gives another digest.
    g = golden()
    entry = g['cases']['1_vs_1_easy/simple115v2']
    assert oracle_digest(entry['assets'], g['steps'], seed=g['seed'] + 1, environments=g['environments']) != entry['digest']


def test_episode_pickle_reads_back():
    from cuju_b200.environment import pickle_episode, unpickle_episode

    assert unpickle_episode(pickle_episode([0, 0, -1], None), 2) == [0, 0, -1, 0, 0]
    assert unpickle_episode(pickle_episode([2, 3, 1], [0, 4, 1, 0]), 4) == [2, 3, 1, 0, 4, 1, 0]


@needs_data
@pytest.mark.skipif(not os.path.isfile(LIBRARY), reason='library not built')
def test_memory_estimate_without_a_device():
    """cuju_memory_estimate plans the batch's buffers without touching a GPU: linear in the
    environments, and the SMM and raw representations add exactly their buffers (up to the
    256-byte rounding of each allocation)."""
    from conftest import ANIMATIONS, resolve
    from cuju_b200 import _native

    library = _native.declare(ctypes.CDLL(LIBRARY))
    paths, counts = resolve('11_vs_11_stochastic_l1_r0')
    keep = []

    def estimate(envs, observation=2):
        p = (ctypes.c_char_p * 1)(paths[0].encode())
        c = (ctypes.c_int * 2)(*counts[0])
        keep.extend([p, c])
        config = _native.Configuration(version=2, assets=p, asset_count=1, animations=ANIMATIONS.encode(),
                                       environment_count=envs, seed=0, observation=observation, auto_reset=1,
                                       ticks_per_step=10, smm_width=96, smm_height=72, stack=1,
                                       agent_counts=ctypes.cast(c, ctypes.c_void_p))
        out = ctypes.c_ulonglong()
        assert library.cuju_memory_estimate(ctypes.byref(config), ctypes.byref(out)) == 0, library.cuju_last_error()
        return out.value

    slack = 64 * 256
    step = estimate(32) - estimate(16)
    assert step > 16 * 370_000
    assert abs((estimate(48) - estimate(32)) - step) <= slack
    # One agent: the SMM map and its final copy (72 x 96 x 4 bytes each), two mark rows of 25
    # int32, in place of the two simple115 buffers (115 float32 each).
    smm = 2 * 72 * 96 * 4 + 2 * 25 * 4 - 2 * 115 * 4
    assert abs((estimate(16, 4) - estimate(16)) - 16 * smm) <= slack


@needs_data
@pytest.mark.skipif(not (os.path.isfile(LIBRARY) and os.path.isfile(ORACLE)), reason='library or oracle not built')
@pytest.mark.parametrize('assets', ['11_vs_11_stochastic_l1_r0', '5_vs_5_l4_r0', 'academy_corner_l1_r0'])
def test_state_padding_equals_the_reference(assets):
    """cuju_state_padding marks the same padding bytes of a state as the reference's (state_api.h:21),
    without a device: the angles' three uninitialized bytes."""
    import random

    from conftest import ANIMATIONS, resolve
    from oracle.driver import OracleBatch

    paths, counts = resolve(assets)
    batch = OracleBatch(paths, counts, 2, 5, ANIMATIONS, threads=1)
    ours = ctypes.CDLL(LIBRARY)
    try:
        batch.reset()
        rng = random.Random(2)
        for _ in range(20):
            batch.step([rng.randrange(19) for _ in range(2 * batch.agents)])
        data, _ = batch.engine_state(1)
        masks = []
        for library in (ours, batch.lib):
            library.cuju_state_padding.argtypes = [ctypes.c_char_p, ctypes.c_ulonglong, ctypes.c_void_p]
            mask = (ctypes.c_ubyte * len(data))()
            assert library.cuju_state_padding(data, len(data), mask) == 0
            masks.append(bytes(mask))
        assert masks[0] == masks[1]
        assert sum(masks[0]) > 0
        bad = (ctypes.c_ubyte * 4)()
        assert ours.cuju_state_padding(b'\x00\x01', 2, bad) == -1
    finally:
        batch.close()


@pytest.mark.skipif(not os.path.isfile(LIBRARY), reason='library not built')
def test_a_c_program_binds_the_header_and_the_library(tmp_path):
    """The C-ABI from C: the header compiles as C11, and a C program linked against the library
    calls entry points that need no device (the backend name, the last error, the local memory a
    batch reserves per thread)."""
    import shutil
    import subprocess

    cc = shutil.which('gcc') or shutil.which('cc')
    if cc is None:
        pytest.skip('no C compiler')
    source = tmp_path / 'bind.c'
    source.write_text(
        '#include <stdio.h>\n'
        '#include "cuju_b200.h"\n'
        'int main(void) {\n'
        '    cuju_configuration c = {0};\n'
        '    c.version = CUJU_CONFIGURATION_VERSION;\n'
        '    if (cuju_environment_create(&c) != NULL) return 2;  /* no assets: refused */\n'
        '    printf("%s|%s\\n", cuju_backend(), cuju_last_error());\n'
        '    return 0;\n'
        '}\n')
    exe = tmp_path / 'bind'
    libdir = os.path.dirname(LIBRARY)
    subprocess.run([cc, '-std=c11', '-Wall', '-Werror', '-I', os.path.join(ROOT, 'include'), str(source), '-o',
                    str(exe), '-L', libdir, '-lcuju_b200', f'-Wl,-rpath,{libdir}'], check=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr
    backend, message = run.stdout.strip().split('|', 1)
    assert backend == 'cuda'
    assert message  # the refusal says why
