"""GPU parity of set_state (batch_environment.h:396, SetState): a state taken from the reference
CPU backend and loaded into both batches gives the same outputs at once and over the following
steps, and the loaded bytes read back unchanged. The full GRF byte format (episode pickle, then
engine bytes) round-trips through the Python mirror."""

import ctypes
import random

import pytest
import torch

from conftest import ANIMATIONS, needs_data, resolve

pytestmark = [pytest.mark.gpu, needs_data]


def _outputs(batch):
    obs, reward, done, _, score = batch._outputs()
    return tuple(t.cpu().numpy().tobytes() for t in (obs, reward, done, score))


@pytest.mark.parametrize('assets', ['11_vs_11_stochastic_l1_r0', '5_vs_5_l4_r0'])
def test_set_state_matches_the_reference_cpu_backend(assets):
    from cuju_b200 import BatchEnvironment
    from oracle.driver import OracleBatch

    envs = 8
    paths, counts = resolve(assets)
    mine = BatchEnvironment(assets, environment_count=envs, seed=3, difficulty=[(0.2, 0.2)])
    ref = OracleBatch(paths, counts, envs, 3, ANIMATIONS, threads=0, difficulty=[0.2, 0.2] * envs)
    rng = random.Random(4)

    def step_both(steps, tag):
        for step in range(steps):
            acts = [[rng.randrange(19) for _ in range(mine.agents)] for _ in range(envs)]
            mine.step(torch.tensor(acts, dtype=torch.int32).cuda())
            expected = ref.step([x for row in acts for x in row])
            assert _outputs(mine) == expected, f'outputs differ {tag} at step {step}'

    try:
        mine.reset()
        assert _outputs(mine) == ref.reset()
        step_both(25, 'before set_state')
        data, episode = ref.engine_state(5)
        expected = ref.set_state(1, data, episode)
        mine.set_engine_state(1, data, episode)
        assert _outputs(mine) == expected, 'outputs after set_state differ'
        assert mine.engine_state(1)[0] == data, 'the loaded state does not read back'
        # The full byte format through the mirror: environment 6 takes environment 2's state.
        mine.set_state(6, mine.get_state(2))
        assert mine.get_state(6) == mine.get_state(2)
        data2, episode2 = ref.engine_state(2)
        ref.set_state(6, data2, episode2)
        step_both(25, 'after set_state')
        for index in range(envs):
            assert mine.engine_state(index)[0] == ref.engine_state(index)[0], f'state {index} differs'
    finally:
        mine.close()
        ref.close()


def test_set_state_refuses_another_scenario():
    from cuju_b200 import BatchEnvironment
    from cuju_b200.errors import StateError
    from oracle.driver import OracleBatch

    paths, counts = resolve('5_vs_5_l4_r0')
    other = OracleBatch(paths, counts, 1, 1, ANIMATIONS, threads=1)
    mine = BatchEnvironment('11_vs_11_stochastic_l1_r0', environment_count=2, seed=1)
    try:
        other.reset()
        mine.reset()
        data, episode = other.engine_state(0)
        # A refused state is a StateError, as in the reference (environment.py:1611-1612).
        with pytest.raises(StateError, match='scenario of the environment'):
            mine.set_engine_state(0, data, episode)
    finally:
        mine.close()
        other.close()


def test_set_stack_restores_a_stacked_observation():
    from cuju_b200 import BatchEnvironment
    from oracle.driver import OracleBatch

    envs, assets = 4, '5_vs_5_l4_r0'
    paths, counts = resolve(assets)
    mine = BatchEnvironment(assets, environment_count=envs, seed=2, stacked=True)
    ref = OracleBatch(paths, counts, envs, 2, ANIMATIONS, threads=0, stack=4)
    rng = random.Random(6)
    try:
        mine.reset()
        assert _outputs(mine) == ref.reset()

        def step_both(steps):
            for step in range(steps):
                acts = [[rng.randrange(19) for _ in range(mine.agents)] for _ in range(envs)]
                mine.step(torch.tensor(acts, dtype=torch.int32).cuda())
                assert _outputs(mine) == ref.step([x for row in acts for x in row]), f'step {step} differs'

        step_both(12)
        data, episode = ref.engine_state(2)
        width = mine.agents * 115 * 4 * 4
        frames = ref.outputs()[0][2 * width:3 * width]
        ref.set_state(0, data, episode)
        ref.lib.cuju_environment_set_stack.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p,
                                                       ctypes.c_char_p, ctypes.c_ulonglong]
        assert ref.lib.cuju_environment_set_stack(ref.handle, 0, b'simple115', frames, len(frames)) == 0
        mine.set_engine_state(0, data, episode)
        mine.set_stack(0, frames)
        assert _outputs(mine) == ref.outputs(), 'outputs after set_state and set_stack differ'
        step_both(12)
    finally:
        mine.close()
        ref.close()
