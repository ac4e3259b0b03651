"""GPU parity at sizes where the lanes of every warp are all busy.

Large batches run one environment per lane and, when all 32 lanes of a warp reach a humanoid's
command request, animation selection or ball touch together, deal that branch to crews of the warp.
Batches smaller than a warp never take that path, so these tests use full warps: a 64-environment
11v11 batch on a lane per environment compared step by step with the reference CPU backend,
and the bench workload itself (16,384 environments) with a sample of its environments compared
against single-environment reference batches. The seed rule makes environment i identical in
any batch that holds it (`first_index` = i for a batch of one), so the sample checks the full-size
run without stepping 16,384 environments on the CPU. Where the reference's CUDA backend has been
built from its sources (`make -C oracle cuda`), the whole bench batch is also compared with it.
"""

import os

import pytest
import torch

from conftest import ANIMATIONS, ROOT, needs_data, resolve

pytestmark = [pytest.mark.gpu, needs_data]

ASSETS = '11_vs_11_stochastic_l1_r0'
DIFFICULTY = (0.2, 0.2)


def _row_bytes(tensor, index):
    return tensor[index].detach().cpu().contiguous().numpy().tobytes()


def test_11v11_full_warps_against_the_oracle():
    from cuju_b200 import BatchEnvironment
    from oracle.driver import OracleBatch

    envs, steps = 64, 40
    paths, counts = resolve(ASSETS)
    mine = BatchEnvironment(ASSETS, environment_count=envs, seed=11, difficulty=[DIFFICULTY], lanes_per_environment=1)
    ref = OracleBatch(paths, counts, envs, 11, ANIMATIONS, threads=0, difficulty=list(DIFFICULTY) * envs)
    try:
        generator = torch.Generator().manual_seed(3)
        mine.reset()
        expected = ref.reset()
        obs, reward, done, _, score = mine._outputs()
        assert obs.cpu().numpy().tobytes() == expected[0], 'reset observations differ'
        for step in range(steps):
            actions = torch.randint(0, 19, (envs, mine.agents), generator=generator, dtype=torch.int32)
            mine.step(actions.cuda())
            expected = ref.step(actions.flatten().tolist())
            got = tuple(t.cpu().numpy().tobytes() for t in (mine._outputs()[i] for i in (0, 1, 2, 4)))
            for name, a, b in zip(('simple115', 'reward', 'done', 'score_reward'), got, expected):
                assert a == b, f'{name} differs at step {step}'
        for index in range(envs):
            assert mine.engine_state(index)[0] == ref.engine_state(index)[0], f'state {index} differs'
    finally:
        mine.close()
        ref.close()


def test_bench_workload_sampled_environments_match_the_oracle():
    from cuju_b200 import BatchEnvironment
    from oracle.driver import OracleBatch

    envs, steps = 16384, 12
    sample = [0, 1, 31, 32, 4097, 8191, 12345, 16383]
    paths, counts = resolve(ASSETS)
    mine = BatchEnvironment(ASSETS, environment_count=envs, seed=0, difficulty=[DIFFICULTY])
    refs = {e: OracleBatch(paths, counts, 1, 0, ANIMATIONS, threads=1, difficulty=list(DIFFICULTY), first_index=e)
            for e in sample}
    try:
        generator = torch.Generator().manual_seed(9)
        mine.reset(seeds=torch.arange(envs))
        for e, ref in refs.items():
            expected = ref.reset([e])
            assert _row_bytes(mine._outputs()[0], e) == expected[0], f'reset of environment {e} differs'
        for step in range(steps):
            actions = torch.randint(0, 19, (envs, mine.agents), generator=generator, dtype=torch.int32)
            mine.step(actions.cuda())
            obs, reward, done, _, score = mine._outputs()
            for e, ref in refs.items():
                expected = ref.step(actions[e].tolist())
                got = (_row_bytes(obs, e), _row_bytes(reward, e), _row_bytes(done, e), _row_bytes(score, e))
                for name, a, b in zip(('simple115', 'reward', 'done', 'score_reward'), got, expected):
                    assert a == b, f'{name} of environment {e} differs at step {step}'
        for e, ref in refs.items():
            assert mine.engine_state(e)[0] == ref.engine_state(0)[0], f'state of environment {e} differs'
    finally:
        mine.close()
        for ref in refs.values():
            ref.close()


def test_batch_of_several_waves_matches_the_oracle():
    """A batch larger than four warps on every SM steps as equal waves of launches (20,000
    environments: two of 10,000). Environments on both sides of the wave boundary, through a masked
    reset inside the second wave, against single-environment reference batches."""
    from cuju_b200 import BatchEnvironment
    from oracle.driver import OracleBatch

    envs, steps = 20000, 10
    sample = [0, 31, 9999, 10000, 10001, 10031, 15000, 19999]
    paths, counts = resolve(ASSETS)
    mine = BatchEnvironment(ASSETS, environment_count=envs, seed=3, difficulty=[DIFFICULTY])
    refs = {e: OracleBatch(paths, counts, 1, 3, ANIMATIONS, threads=1, difficulty=list(DIFFICULTY), first_index=e)
            for e in sample}
    try:
        generator = torch.Generator().manual_seed(21)
        mine.reset()
        for e, ref in refs.items():
            assert _row_bytes(mine._outputs()[0], e) == ref.reset()[0], f'reset of environment {e} differs'
        for step in range(steps):
            actions = torch.randint(0, 19, (envs, mine.agents), generator=generator, dtype=torch.int32)
            mine.step(actions.cuda())
            obs, reward, done, _, score = mine._outputs()
            for e, ref in refs.items():
                expected = ref.step(actions[e].tolist())
                got = (_row_bytes(obs, e), _row_bytes(reward, e), _row_bytes(done, e), _row_bytes(score, e))
                for name, a, b in zip(('simple115', 'reward', 'done', 'score_reward'), got, expected):
                    assert a == b, f'{name} of environment {e} differs at step {step}'
            if step == 4:
                mask = torch.zeros(envs, dtype=torch.bool)
                mask[[10001, 15000]] = True
                seeds = torch.full((envs,), -1, dtype=torch.int64)
                seeds[10001], seeds[15000] = 987654321, 123456789
                mine.reset(mask=mask, seeds=seeds)
                for e in (10001, 15000):
                    expected = refs[e].reset_masked([1], [int(seeds[e])])
                    assert _row_bytes(mine._outputs()[0], e) == expected[0], f'masked reset of {e} differs'
        for e, ref in refs.items():
            assert mine.engine_state(e)[0] == ref.engine_state(0)[0], f'state of environment {e} differs'
    finally:
        mine.close()
        for ref in refs.values():
            ref.close()


REFERENCE_CUDA = os.path.join(ROOT, 'oracle', '_ref', 'libcuju_cuda.so')


@pytest.mark.skipif(not os.path.isfile(REFERENCE_CUDA), reason='run make -C oracle cuda to build the reference GPU backend')
def test_bench_workload_equals_the_reference_cuda_backend():
    """The whole 16,384-environment bench batch against the reference's own CUDA backend, compiled
    from its sources for sm_100a (oracle/Makefile, target `cuda`) and driven through the same C-ABI:
    every output buffer, every step."""
    import hashlib

    from cuju_b200 import BatchEnvironment

    envs, steps = 16384, 6
    digests = {}
    for name, library in (('b200', None), ('reference', REFERENCE_CUDA)):
        options = {'library': library} if library else {}
        batch = BatchEnvironment(ASSETS, environment_count=envs, seed=0, difficulty=[DIFFICULTY], **options)
        try:
            generator = torch.Generator(device='cuda').manual_seed(21)
            batch.reset(seeds=torch.arange(envs))
            trail = [hashlib.sha256(_row_bytes(batch._outputs()[0], slice(None))).hexdigest()]
            for step in range(steps):
                actions = torch.randint(0, 19, (envs, batch.agents), generator=generator, device='cuda',
                                        dtype=torch.int32)
                batch.step(actions)
                obs, reward, done, _, score = batch._outputs()
                h = hashlib.sha256()
                for t in (obs, reward, done, score):
                    h.update(_row_bytes(t, slice(None)))
                trail.append(h.hexdigest())
            digests[name] = trail
        finally:
            batch.close()
    for step, (a, b) in enumerate(zip(digests['b200'], digests['reference'])):
        assert a == b, f'outputs differ from the reference CUDA backend at step {step}'
