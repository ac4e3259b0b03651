"""The multi-GPU split on CPU: two gloo ranks, each stepping its own contiguous slice of
environments (`first_index = rank * slice`), must produce exactly what one batch of all the
environments produces, with no collective on the step path; the timed region's maximum over ranks
is the only reduction (as in bench.py). The ranks run the reference CPU backend (the oracle), so the
test checks the slicing and seeding logic that bench.py relies on, not the device kernels.
"""

import os
import socket

import pytest
import torch.multiprocessing as mp

from conftest import ANIMATIONS, needs_data, resolve

ASSETS = '5_vs_5_l4_r0'
SLICE = 3
STEPS = 12
WORLD = 2


def _actions(step, first, count, agents):
    return [((step * 7 + (first + e) * 3 + a * 5) % 19) for e in range(count) for a in range(agents)]


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank_main(rank, port, out):
    import datetime

    import torch
    import torch.distributed as dist

    from oracle.driver import OracleBatch

    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    try:
        paths, counts = resolve(ASSETS)
        batch = OracleBatch(paths, counts, SLICE, 0, ANIMATIONS, threads=1, first_index=rank * SLICE)
        outputs = [batch.reset()[0]]
        for step in range(STEPS):
            obs, reward, done, _ = batch.step(_actions(step, rank * SLICE, SLICE, batch.agents))
            outputs.append(obs + reward + done)
        batch.close()
        # The only collectives: gather for the check, and the max of a per-rank time.
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, outputs)
        elapsed = torch.tensor([1.0 + rank], dtype=torch.float64)
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        if rank == 0:
            out.put((gathered, float(elapsed)))
    finally:
        dist.destroy_process_group()


@needs_data
def test_two_rank_slices_equal_one_batch():
    from oracle.driver import OracleBatch

    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, queue)) for r in range(WORLD)]
    for p in procs:
        p.start()
    gathered, elapsed = queue.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert elapsed == float(WORLD)

    paths, counts = resolve(ASSETS)
    whole = OracleBatch(paths, counts, WORLD * SLICE, 0, ANIMATIONS, threads=1)
    agents = whole.agents
    expected = [whole.reset()[0]]
    for step in range(STEPS):
        obs, reward, done, _ = whole.step(_actions(step, 0, WORLD * SLICE, agents))
        expected.append(obs + reward + done)
    whole.close()

    # Reassemble the slices in rank order and compare every step byte for byte.
    obs_bytes = SLICE * agents * 115 * 4
    for step in range(STEPS + 1):
        if step == 0:
            merged = b''.join(gathered[r][0] for r in range(WORLD))
            assert merged == expected[0], 'reset observations differ'
            continue
        parts = [gathered[r][step] for r in range(WORLD)]
        obs = b''.join(p[:obs_bytes] for p in parts)
        rest_w = SLICE * agents * 4
        reward = b''.join(p[obs_bytes:obs_bytes + rest_w] for p in parts)
        done = b''.join(p[obs_bytes + rest_w:] for p in parts)
        whole_step = expected[step]
        w_obs = WORLD * obs_bytes
        w_rew = WORLD * rest_w
        assert obs == whole_step[:w_obs], f'observations differ at step {step}'
        assert reward == whole_step[w_obs:w_obs + w_rew], f'rewards differ at step {step}'
        assert done == whole_step[w_obs + w_rew:], f'done flags differ at step {step}'


if __name__ == '__main__':
    pytest.main([__file__, '-q'])
