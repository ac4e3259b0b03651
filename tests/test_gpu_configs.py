"""GPU parity on the benchmark's configurations, each as it is specified, against the reference CPU
backend (the oracle).

* Configuration 1: 64 environments of 5-a-side with four controlled agents, the right team at
  difficulty 0.6, seed 0, 1,000 steps of actions drawn by torch's seeded CPU generator; every
  output buffer every step, then every environment's GRF state bytes.
* Configuration 2: the single-attacker drill (tests/golden/academy_attacker_vs_keeper.py, built by
  make_drill.py) at 4,096 environments with reset seeds 0..4095, over enough steps that episodes end
  and restart inside the step; a sample of environments against one-environment oracle batches.
* Configuration 4: 11-a-side with all eleven left players controlled, the right team at 0.95, with a
  Bernoulli(0.001) masked reset with fresh seeds after every step; the batch is one GPU's slice of
  the 65,536 (first_index past the first slice) and a sample of environments, some of them forced
  into the masks, is checked.
* Configuration 5: one GPU's slice of the mixed batch (11-a-side, 5-a-side and the drill interleaved
  by index as 0, 1, 0, 1, 2), four-frame stacked observations; a sample of each bundle is checked.

The seed rule makes environment i of a batch identical to the single environment of a batch with
`first_index` = i (same bundles, same assignment), which is how a sample is checked without
stepping the whole batch on the CPU.
"""

import os

import pytest
import torch

from conftest import ANIMATIONS, ROOT, needs_data, resolve

pytestmark = [pytest.mark.gpu, needs_data]

DRILL = os.path.join(ROOT, 'tests', 'golden', 'academy_attacker_vs_keeper_l0_r0.cjb')


def _row(tensor, index):
    return tensor[index].detach().cpu().contiguous().numpy().tobytes()


def test_configuration_1_five_a_side_64_environments_1000_steps():
    from cuju_b200 import BatchEnvironment
    from oracle.driver import OracleBatch

    envs, steps = 64, 1000
    paths, counts = resolve('5_vs_5_l4_r0')
    mine = BatchEnvironment('5_vs_5_l4_r0', environment_count=envs, seed=0, difficulty=[(None, 0.6)])
    ref = OracleBatch(paths, counts, envs, 0, ANIMATIONS, threads=0, difficulty=[-1.0, 0.6] * envs)
    try:
        assert mine.agents == 4
        generator = torch.Generator().manual_seed(0)
        mine.reset()
        assert _row(mine._outputs()[0], slice(None)) == ref.reset()[0], 'reset observations differ'
        for step in range(steps):
            actions = torch.randint(0, 19, (envs, 4), generator=generator, dtype=torch.int32)
            mine.step(actions.cuda())
            expected = ref.step(actions.flatten().tolist())
            obs, reward, done, _, score = mine._outputs()
            got = (_row(obs, slice(None)), _row(reward, slice(None)), _row(done, slice(None)), _row(score, slice(None)))
            for name, a, b in zip(('simple115', 'reward', 'done', 'score_reward'), got, expected):
                assert a == b, f'{name} differs at step {step}'
        for index in range(envs):
            assert mine.engine_state(index)[0] == ref.engine_state(index)[0], f'state {index} differs'
    finally:
        mine.close()
        ref.close()


def _sampled(assets, agent_counts, envs, steps, sample, seed=0, difficulty=None, first_index=0, mask_fn=None,
             assignment=None, stacked=False, reset_seeds=None, lanes=None):
    """Steps a batch on the GPU and one-environment oracle batches for `sample`, comparing each
    sampled environment's outputs every step and its state bytes at the end."""
    from cuju_b200 import BatchEnvironment
    from oracle.driver import OracleBatch

    names = [assets] if isinstance(assets, str) else list(assets)
    paths, counts = resolve(names)
    counts = [c if a is None else a for c, a in zip(counts, agent_counts or [None] * len(counts))]
    options = {'agent_counts': agent_counts} if agent_counts else {}
    if lanes is not None:
        options['lanes_per_environment'] = lanes
    mine = BatchEnvironment(names if len(names) > 1 else names[0], environment_count=envs, seed=seed,
                            difficulty=None if difficulty is None else [difficulty], first_index=first_index,
                            assignment=assignment, stacked=stacked, **options)
    flat = None if difficulty is None else [(-1.0 if v is None else v) for v in difficulty]
    refs = {e: OracleBatch(paths, counts, 1, seed, ANIMATIONS, threads=1, difficulty=flat, first_index=first_index + e,
                           assignment=None if assignment is None else [assignment[e]], stack=4 if stacked else 1)
            for e in sample}
    try:
        generator = torch.Generator().manual_seed(seed + 17)
        if reset_seeds is None:
            mine.reset()
        else:
            mine.reset(seeds=torch.tensor(reset_seeds, dtype=torch.int64))
        for e, ref in refs.items():
            expected = ref.reset(None if reset_seeds is None else [reset_seeds[e]])
            assert _row(mine._outputs()[0], e) == expected[0], f'reset of environment {e} differs'
        for step in range(steps):
            actions = torch.randint(0, 19, (envs, mine.agents), generator=generator, dtype=torch.int32)
            mine.step(actions.cuda())
            obs, reward, done, _, score = mine._outputs()
            for e, ref in refs.items():
                expected = ref.step(actions[e][:ref.agents].tolist())
                got = (_row(obs, e), _row(reward, e)[:4 * ref.agents], _row(done, e), _row(score, e))
                for name, a, b in zip(('observation', 'reward', 'done', 'score_reward'), got, expected):
                    assert a == b, f'{name} of environment {e} differs at step {step}'
            if mask_fn is not None:
                mask, seeds = mask_fn(step)
                if mask.any():
                    mine.reset(mask=mask, seeds=seeds)
                    for e, ref in refs.items():
                        if mask[e]:
                            expected = ref.reset_masked([1], [int(seeds[e])])
                            assert _row(mine._outputs()[0], e) == expected[0], \
                                f'masked reset of environment {e} differs at step {step}'
        for e, ref in refs.items():
            assert mine.engine_state(e)[0] == ref.engine_state(0)[0], f'state of environment {e} differs'
    finally:
        mine.close()
        for ref in refs.values():
            ref.close()


def test_configuration_2_drill_4096_environments_through_restarts():
    envs = 4096
    _sampled(DRILL, [(1, 0)], envs, 150, [0, 1, 31, 32, 777, 2048, 4000, 4095],
             reset_seeds=list(range(envs)))


def test_configuration_4_all_players_controlled_with_masked_resets():
    envs = 8192  # one GPU's slice when 65,536 environments are split over eight
    first = 3 * envs
    sample = [0, 5, 32, 1000, 4095, 4096, 8000, 8191]
    forced = {2: [5, 4096], 5: [1000], 7: [8191, 0]}
    generator = torch.Generator().manual_seed(4)

    def masks(step):
        mask = torch.rand(envs, generator=generator) < 0.001
        for e in forced.get(step, []):
            mask[e] = True
        seeds = torch.where(mask, torch.randint(0, 2**32 - 1, (envs,), generator=generator, dtype=torch.int64),
                            torch.full((envs,), -1, dtype=torch.int64))
        return mask, seeds

    _sampled('11_vs_11_hard_stochastic_l11_r0', None, envs, 10, sample, first_index=first, mask_fn=masks)


def test_configuration_5_mixed_stacked_slice():
    envs = 16384
    first = 2 * envs
    assignment = [[0, 1, 0, 1, 2][(first + i) % 5] for i in range(envs)]
    sample = [0, 1, 4, 9, 32, 5003, 12004, 16383]  # bundles 0, 1, 2 and both ends
    assert {assignment[e] for e in sample} == {0, 1, 2}
    _sampled(['11_vs_11_stochastic_l1_r0', '5_vs_5_l4_r0', DRILL], [(1, 0), (4, 0), (1, 0)], envs, 10, sample,
             first_index=first, assignment=assignment, stacked=True)
