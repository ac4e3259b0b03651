"""The multi-device front end's host logic on CPU (reference tests/test_multi_device.py): the split
of environments into contiguous parts with `first_index` set to each part's start, per-environment
options and arguments cut to each part, outputs gathered in environment order (dicts too), state
calls routed to the part that holds the environment, and the refusals. The parts here are stand-ins
whose outputs name the environment of the seed rule, so a wrong slice or offset shows; the device
parts are checked against one batch on a GPU in tests/test_gpu_zmulti_device.py. `EpisodeTotals`
is summed over two gloo ranks.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from cuju_b200.multi_device import EpisodeTotals, MultiDeviceBatch


class _Part:
    """A stand-in part: observation row e holds (first_index + e, resets, last action, seed)."""

    def __init__(self, count, first_index, options):
        self.count, self.first = count, first_index
        self.options = options
        self.agents, self.action_count, self.squeeze, self.stacked = 2, 19, False, False
        self.left_agents = torch.full((count,), 2, dtype=torch.int32)
        self.right_agents = torch.zeros(count, dtype=torch.int32)
        self.obs = torch.zeros((count, 2, 4), dtype=torch.float32)
        self.obs[:, :, 0] = torch.arange(first_index, first_index + count, dtype=torch.float32)[:, None]
        self.closed = False
        self.pending = None

    def reset(self, seeds=None, reverse=None):
        self.obs[:, :, 1] += 1
        if seeds is not None:
            self.obs[:, :, 3] = torch.as_tensor(seeds, dtype=torch.float32).reshape(-1, 1).expand(self.count, 1)
        return self.obs

    def reset_done(self):
        self.obs[:, :, 1] += 10

    def step_async(self, actions):
        assert actions.shape == (self.count, 2)
        self.pending = actions

    def step_wait(self):
        self.obs[:, :, 2] = self.pending.to(torch.float32)
        reward = self.obs[:, :, 0] * 0.5
        done = (self.obs[:, 0, 0] % 2) == 0
        score = self.obs[:, 0, 0].to(torch.int32)
        return self.obs, reward, done, {'final_observation': {'x': self.obs[:, :, :2]}, 'score_reward': score}

    def observation(self):
        return self.obs

    def get_state(self, index):
        return f'{self.first + index}'.encode()

    def set_state(self, index, state):
        self.obs[index, :, 3] = float(state.decode())

    def close(self):
        self.closed = True


class _Batch(MultiDeviceBatch):
    @staticmethod
    def _device(device):
        return torch.device('cpu')

    def _make_part(self, assets, device, count, first_index, options):
        return _Part(count, first_index, options)


def test_split_gather_and_routing():
    batch = _Batch('5_vs_5_l4_r0', devices=['a', 'b', 'c'], environment_count=11,
                   assignment=list(range(11)), game_engine_random_seed=7)
    assert batch.ranges == [(0, 4), (4, 8), (8, 11)]
    assert [p.first for p in batch.parts] == [0, 4, 8]
    assert batch.parts[1].options['assignment'] == [4, 5, 6, 7]
    assert batch.parts[2].options['game_engine_random_seed'] == 7
    assert batch.left_agents.shape == (11,)
    obs = batch.reset(seeds=torch.arange(100, 111))
    assert obs[:, 0, 0].tolist() == list(range(11))
    assert obs[:, 0, 3].tolist() == list(range(100, 111))
    actions = torch.arange(22, dtype=torch.int32).reshape(11, 2)
    obs, reward, done, info = batch.step(actions)
    assert torch.equal(obs[:, :, 2], actions.float())
    assert torch.equal(reward, obs[:, :, 0] * 0.5)
    assert done.tolist() == [e % 2 == 0 for e in range(11)]
    assert info['score_reward'].tolist() == list(range(11))
    assert torch.equal(info['final_observation']['x'], obs[:, :, :2])
    batch.reset_done()
    assert batch.observation()[:, 0, 1].tolist() == [11.0] * 11
    assert [batch.get_state(i) for i in (0, 3, 4, 10)] == [b'0', b'3', b'4', b'10']
    batch.set_state(9, b'42')
    assert batch.parts[2].obs[1, 0, 3].item() == 42.0
    with pytest.raises(IndexError):
        batch.get_state(11)
    parts = batch.parts
    batch.close()
    assert all(p.closed for p in parts)
    batch.close()
    with pytest.raises(RuntimeError):
        batch.step(actions)


def test_explicit_split_and_refusals():
    batch = _Batch('5_vs_5_l4_r0', devices=[0, 1], environment_count=5, split=[1, 4])
    assert batch.ranges == [(0, 1), (1, 5)]
    batch.close()
    for kwargs in ({'split': [2, 2]}, {'split': [0, 5]}, {'first_index': 3}, {'device': 'cuda'},
                   {'assignment': [0, 1]}):
        with pytest.raises(ValueError):
            _Batch('5_vs_5_l4_r0', devices=[0, 1], environment_count=5, **kwargs)
    with pytest.raises(ValueError):
        _Batch('5_vs_5_l4_r0', devices=[], environment_count=5)
    with pytest.raises(ValueError):
        MultiDeviceBatch('5_vs_5_l4_r0', devices=['cpu'], environment_count=5)


def test_episode_totals_on_one_rank():
    totals = EpisodeTotals(device='cpu')
    totals.update(torch.tensor([[1.0, -1.0], [0.5, 0.0]]), torch.tensor([True, False]), torch.tensor([1, -1]))
    totals.update(torch.tensor([[0.0, 0.0], [2.0, 0.0]]), torch.tensor([True, True]), torch.tensor([0, 1]))
    assert totals.all_reduce() == {'episodes': 3.0, 'left_goals': 2.0, 'right_goals': 1.0, 'reward': 2.5}


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _totals_rank(rank, port, out):
    import datetime

    import torch.distributed as dist

    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    try:
        totals = EpisodeTotals(device='cpu')
        for step in range(3):
            done = torch.tensor([step == rank, True])
            score = torch.tensor([1 if rank == 0 else -1, 0], dtype=torch.int32)
            totals.update(torch.full((2, 1), 0.25 * (rank + 1)), done, score)
        result = totals.all_reduce()
        if rank == 0:
            out.put(result)
    finally:
        dist.destroy_process_group()


def test_episode_totals_summed_over_two_gloo_ranks():
    ctx = mp.get_context('spawn')
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_totals_rank, args=(r, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    result = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # Per rank: 3 steps x (1 + 1 ended) = 4 episodes; rank 0 scores 3 left goals, rank 1 three right.
    assert result == {'episodes': 8.0, 'left_goals': 3.0, 'right_goals': 3.0, 'reward': 3 * 2 * 0.25 + 3 * 2 * 0.5}
