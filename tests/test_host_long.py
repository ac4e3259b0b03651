"""The simulation source compiled for the host against the reference's long golden digests.

tests/host/hostsim.cu builds the library's C-ABI and simulation headers for the host, each kernel
replaced by a serial loop over the environments (test infrastructure; the product has no host
path). Run through the same digest as the reference's tests, it must reproduce the long cases of
digests.json: two full 3,010-step 11v11 matches (simple115v2, and raw), a full 5v5 match with the
checkpoint reward, and 1,500-2,000 steps of academy drills over many episodes (extracted, and
checkpoints). The device kernels compile the same source; the GPU tests pin them on shorter runs.
"""

import pytest

from conftest import golden, needs_data, oracle_digest


@needs_data
@pytest.mark.parametrize('case', sorted(golden()['long_cases']))
def test_long_golden_digest_on_the_host(host_library, case):
    g = golden()
    entry = g['long_cases'][case]
    assert oracle_digest(entry['assets'], entry['steps'], seed=g['seed'], environments=g['environments'],
                         library=host_library, **entry['options']) == entry['digest']


@needs_data
@pytest.mark.parametrize('representation,width', [(4, 72 * 96 * 4 * 4), (2, 115 * 4 * 4)])
def test_set_stack_on_the_host_against_the_oracle(host_library, representation, width):
    """set_state then set_stack (SMM or simple115 frames) on a stacked batch, built for the host,
    against the reference CPU backend: the same outputs at once and over the following steps."""
    import ctypes
    import random

    from conftest import ANIMATIONS, resolve
    from oracle.driver import OracleBatch

    envs = 4
    paths, counts = resolve('5_vs_5_l4_r0')
    batches = [OracleBatch(paths, counts, envs, 2, ANIMATIONS, threads=1, stack=4, representation=representation,
                           library=library) for library in (None, host_library)]
    ref, mine = batches
    rng = random.Random(8)
    try:
        assert mine.reset() == ref.reset()

        def step_both(steps):
            for step in range(steps):
                acts = [rng.randrange(19) for _ in range(envs * mine.agents)]
                assert mine.step(acts) == ref.step(acts), f'step {step} differs'

        step_both(12)
        data, episode = ref.engine_state(2)
        per_env = mine.agents * width
        frames = ref.outputs()[0][2 * per_env:3 * per_env]
        name = b'smm' if representation == 4 else b'simple115'
        for batch in batches:
            batch.set_state(0, data, episode)
            batch.lib.cuju_environment_set_stack.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p,
                                                             ctypes.c_char_p, ctypes.c_ulonglong]
            assert batch.lib.cuju_environment_set_stack(batch.handle, 0, name, frames, len(frames)) == 0, \
                batch.lib.cuju_last_error()
        assert mine.outputs() == ref.outputs()
        step_both(12)
    finally:
        for batch in batches:
            batch.close()
