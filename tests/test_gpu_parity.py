"""GPU parity: the B200 batch against the reference, bit for bit.

1. Every golden digest of the simple115 representations (tests/golden/digests.json, the
   reference's published known answers): observations, rewards and done flags of 100 steps of 4
   environments, then every environment's GRF state bytes.
2. Step-by-step against the reference CPU backend run live (oracle/_ref/libcuju_cpu.so) on larger
   batches, seeds, masked resets and per-environment difficulty, comparing full output buffers
   each step and the engine state bytes at the end.
"""

import random

import pytest
import torch

from conftest import ANIMATIONS, actions_at, device_digest, golden, needs_data, resolve, simple115_cases

pytestmark = [pytest.mark.gpu, needs_data]


@pytest.mark.parametrize('case', simple115_cases())
def test_golden_digest(case):
    g = golden()
    entry = g['cases'][case]
    assert device_digest(entry['assets'], g['steps'], seed=g['seed'], environments=g['environments'],
                         **entry['options']) == entry['digest']


@pytest.mark.parametrize('case', ['5_vs_5/simple115v2', '11_vs_11_stochastic/simple115v2', 'mixed'])
def test_golden_digest_one_lane_per_environment(case):
    """Golden cases with each environment on a lane of its own (the layout of large batches),
    where the four lanes of a partial warp run every branch themselves."""
    g = golden()
    entry = g['cases'][case]
    assert device_digest(entry['assets'], g['steps'], seed=g['seed'], environments=g['environments'],
                         lanes_per_environment=1, **entry['options']) == entry['digest']


def _outputs(batch):
    obs, reward, done, _, score = batch._outputs()
    return (obs.cpu().numpy().tobytes(), reward.cpu().numpy().tobytes(), done.cpu().numpy().tobytes(),
            score.cpu().numpy().tobytes())


def _compare(assets, environments, steps, seed, actions_fn, mask_fn=None, difficulty=None, rewards='scoring',
             lanes=None):
    from cuju_b200 import BatchEnvironment
    from oracle.driver import OracleBatch

    paths, counts = resolve(assets)
    mine = BatchEnvironment(assets, environment_count=environments, seed=seed, rewards=rewards,
                            difficulty=None if difficulty is None else [difficulty], lanes_per_environment=lanes)
    flat_difficulty = None
    if difficulty is not None:
        flat_difficulty = [(-1.0 if v is None else v) for _ in range(environments) for v in difficulty]
    ref = OracleBatch(paths, counts, environments, seed, ANIMATIONS, threads=0, checkpoints='checkpoints' in rewards,
                      difficulty=flat_difficulty)
    try:
        mine.reset()
        expected = ref.reset()
        assert _outputs(mine) == expected, 'reset outputs differ'
        for step in range(steps):
            acts = actions_fn(step, environments, mine.agents)
            mine.step(torch.tensor(acts, dtype=torch.int32).cuda())
            expected = ref.step([x for row in acts for x in row])
            got = _outputs(mine)
            for name, a, b in zip(('simple115', 'reward', 'done', 'score_reward'), got, expected):
                assert a == b, f'{name} differs at step {step}'
            if mask_fn is not None:
                mask, seeds = mask_fn(step, environments)
                if any(mask):
                    mine.reset(mask=torch.tensor(mask, dtype=torch.bool), seeds=seeds)
                    expected = ref.reset_masked(mask, seeds)
                    assert _outputs(mine) == expected, f'masked reset differs at step {step}'
        for index in range(environments):
            assert mine.engine_state(index)[0] == ref.engine_state(index)[0], f'state {index} differs'
    finally:
        mine.close()
        ref.close()


@pytest.mark.parametrize('lanes', [None, 1, 8])
def test_5v5_four_agents_64_environments_against_the_oracle(lanes):
    """The same batch with the library's layout for its size (a warp per environment), a lane per
    environment (the assisted branches dealt to crews of the warp) and crews of eight lanes."""
    rng = random.Random(0)
    _compare('5_vs_5_l4_r0', 64, 200, 0,
             lambda s, e, a: [[rng.randrange(19) for _ in range(a)] for _ in range(e)], lanes=lanes)


def test_11v11_difficulty_and_masked_resets_against_the_oracle():
    rng = random.Random(1)
    mrng = random.Random(2)

    def mask_fn(step, e):
        mask = [1 if mrng.random() < 0.05 else 0 for _ in range(e)]
        seeds = [mrng.randrange(0, 2**32) if m and mrng.random() < 0.5 else -1 for m in mask]
        return mask, seeds

    _compare('11_vs_11_stochastic_l1_r0', 16, 120, 3,
             lambda s, e, a: [[rng.randrange(19) for _ in range(a)] for _ in range(e)],
             mask_fn=mask_fn, difficulty=(0.2, 0.2))


def test_academy_drill_many_episodes_against_the_oracle():
    _compare('academy_empty_goal_close_l1_r0', 32, 300, 5,
             lambda s, e, a: actions_at(s, e, a, 19), rewards='scoring,checkpoints')
