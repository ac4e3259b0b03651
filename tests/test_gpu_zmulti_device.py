"""The multi-device front end and the device-resident masked reset on a B200.

A `MultiDeviceBatch` whose parts share one GPU (a device may repeat, as in the reference's
tests/test_multi_device.py) must give, environment for environment, what one batch of all the
environments gives: the parts differ only in `first_index`, so this checks the seed rule across
parts with drawn seeds and automatic restarts. A masked reset with seeds and mask in device memory
(`cuju_b200_environment_reset_masked_device`) must give what the reference-shaped masked reset with
the same seeds from the host gives. `EpisodeTotals` must equal the same sums taken on the host.
"""

import pytest
import torch

from conftest import needs_data

pytestmark = [pytest.mark.gpu, needs_data]

DRILL = 'academy_empty_goal_close_l1_r0'


def _bytes(tensor):
    return tensor.detach().cpu().contiguous().numpy().tobytes()


def test_parts_on_one_gpu_equal_one_batch():
    from cuju_b200 import BatchEnvironment
    from cuju_b200.multi_device import EpisodeTotals, MultiDeviceBatch

    envs, steps = 48, 60
    single = BatchEnvironment(DRILL, environment_count=envs, seed=5)
    multi = MultiDeviceBatch(DRILL, devices=[0, 0, 0], environment_count=envs, split=[20, 12, 16], seed=5)
    try:
        assert multi.ranges == [(0, 20), (20, 32), (32, 48)]
        totals, expected = EpisodeTotals(device='cuda'), torch.zeros(4, dtype=torch.float64)
        assert _bytes(multi.reset()) == _bytes(single.reset())
        generator = torch.Generator().manual_seed(17)
        for step in range(steps):
            actions = torch.randint(0, 19, (envs, single.agents), generator=generator, dtype=torch.int32)
            got = multi.step(actions.cuda())
            want = single.step(actions.cuda())
            for name, a, b in (('observation', got[0], want[0]), ('reward', got[1], want[1]),
                               ('done', got[2], want[2]), ('score_reward', got[3]['score_reward'],
                                                           want[3]['score_reward']),
                               ('final_observation', got[3]['final_observation'], want[3]['final_observation'])):
                assert _bytes(a) == _bytes(b), f'{name} differs at step {step}'
            totals.update(got[1], got[2], got[3]['score_reward'])
            reward, done, score = (t.cpu() for t in (want[1], want[2], want[3]['score_reward']))
            expected += torch.tensor([float(done.sum()), float((score > 0).sum()), float((score < 0).sum()),
                                      float(reward.double().sum())], dtype=torch.float64)
        for index in (0, 19, 20, 31, 32, 47):
            assert multi.get_state(index) == single.get_state(index), f'state {index} differs'
        result = totals.all_reduce()
        assert result['episodes'] > 0
        assert list(result.values()) == pytest.approx(expected.tolist(), rel=1e-12, abs=1e-9)
    finally:
        multi.close()
        single.close()


def test_device_seed_masked_reset_equals_host_seeds():
    from cuju_b200 import BatchEnvironment

    envs = 64
    host = BatchEnvironment(DRILL, environment_count=envs, seed=8)
    device = BatchEnvironment(DRILL, environment_count=envs, seed=8)
    try:
        assert _bytes(host.reset()) == _bytes(device.reset())
        generator = torch.Generator().manual_seed(4)
        for step in range(30):
            actions = torch.randint(0, 19, (envs, 1), generator=generator, dtype=torch.int32).cuda()
            a, b = host.step(actions), device.step(actions)
            assert _bytes(a[0]) == _bytes(b[0]), f'observation differs at step {step}'
            if step % 5 == 2:
                mask = torch.rand(envs, generator=generator) < 0.3
                seeds = torch.randint(0, 2**32, (envs,), generator=generator, dtype=torch.int64)
                seeds[torch.rand(envs, generator=generator) < 0.5] = -1
                want = host.reset(mask=mask.cuda(), seeds=seeds)
                got = device.reset(mask=mask.cuda(), seeds=seeds.cuda())
                torch.cuda.synchronize()
                assert _bytes(got) == _bytes(want), f'masked reset after step {step} differs'
        for index in range(0, envs, 9):
            assert host.get_state(index) == device.get_state(index), f'state {index} differs'
    finally:
        host.close()
        device.close()
