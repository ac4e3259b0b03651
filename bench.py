"""Throughput of GRF's batched match step on B200: environment steps per second.

Default workload (the metric's 1-GPU configuration): `11_vs_11_stochastic`,
one controlled agent (the active player), every other player built-in AI at difficulty 0.2 on both
sides, 16,384 environments per GPU, automatic restart, seeded uniform int32 actions in [0, 19).
With N GPUs each rank steps its own contiguous slice of environments (the seed rule's
`first_index = rank * envs`), so per-GPU work is fixed (weak scaling) and no collective runs on the
step path; the only collectives are the barrier and the max of the timed region over ranks.

`--config` picks another of BASELINE.json's configurations: 1 (5-a-side, 64 environments), 2 (the
single-attacker drill, 4,096 environments per GPU), 4 (11-a-side with all eleven left players
controlled at 0.95, 65,536 environments split over the ranks, a Bernoulli(0.001) masked reset with
fresh seeds after every step) or 5 (131,072 mixed environments split over the ranks: 11-a-side,
5-a-side and the drill interleaved by index, four-frame stacked observations).

`value` times the device step with inputs resident (actions pre-generated on the device); `e2e`
times the same steps through the public API with pinned host actions copied in (and host masks and
seeds for configuration 4) and the step's observation, reward and done read back every step. The
roofline uses the algorithmic bytes of an env-step, B = 2*S + 4*A + 4*obs*A + 4*A + 5 (S the
scenario's GRF state size, measured with get_state; obs = 115 floats, 460 when stacked), plus
p*2*S for a masked reset of probability p, over the CUDA-event duration of the step kernel.
`--impl reference` times the reference CPU backend (built from source into oracle/_ref) on this
host's cores on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = 'env steps/sec, 11v11 at 1/2/4/8 B200 vs host-CPU path; % HBM roofline'
DRILL = os.path.join(ROOT, 'tests', 'golden', 'academy_attacker_vs_keeper_l0_r0.cjb')
# DRAM bytes (read + write) of one step_kernel launch of configuration 3 in GB: one ncu capture at
# 8,192 environments (dram__bytes_read.sum + dram__bytes_write.sum = 44.64 GB, the 4th step)
# scaled by the environments of a 16,384-environment launch, since the traffic is per-environment
# state and stack; None where no capture covers the configuration.
TRAFFIC_GB = {3: 89.3}

CONFIGS = {
    1: dict(assets=['5_vs_5_l4_r0'], agents=None, difficulty=(None, 0.6), envs=64, split=False, masked=0.0,
            stacked=False, interleave=None, seeds='rule',
            text='5_vs_5_l4_r0, 4 controlled agents, difficulty (scenario, 0.6), 64 envs, seed 0'),
    2: dict(assets=[DRILL], agents=[(1, 0)], difficulty=None, envs=4096, split=False, masked=0.0, stacked=False,
            interleave=None, seeds='index',
            text='single attacker vs goalkeeper drill (tests/golden/academy_attacker_vs_keeper.py), 1 controlled '
                 'agent, 4096 envs per GPU, reset seeds 0..4095'),
    3: dict(assets=['11_vs_11_stochastic_l1_r0'], agents=None, difficulty=(0.2, 0.2), envs=16384, split=False,
            masked=0.0, stacked=False, interleave=None, seeds='index',
            text='11_vs_11_stochastic_l1_r0, 1 controlled agent, difficulty (0.2, 0.2), 16384 envs per GPU'),
    4: dict(assets=['11_vs_11_hard_stochastic_l11_r0'], agents=None, difficulty=None, envs=65536, split=True,
            masked=0.001, stacked=False, interleave=None, seeds='index',
            text='11_vs_11_hard_stochastic_l11_r0, 11 controlled agents, right team 0.95, 65536 envs split over '
                 'the ranks, Bernoulli(0.001) masked reset with fresh seeds every step'),
    5: dict(assets=['11_vs_11_stochastic_l1_r0', '5_vs_5_l4_r0', DRILL], agents=[(1, 0), (4, 0), (1, 0)],
            difficulty=None, envs=131072, split=True, masked=0.0, stacked=True, interleave=[0, 1, 0, 1, 2],
            seeds='index',
            text='131072 mixed envs split over the ranks: 11_vs_11_stochastic_l1_r0 / 5_vs_5_l4_r0 / drill '
                 'interleaved by index as 0,1,0,1,2, four-frame stacked observations'),
}


def measured_peak() -> tuple[float, str]:
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    try:
        with open(path, encoding='utf-8') as handle:
            peaks = json.load(handle)
        for key in ('hbm_gbs', 'hbm_GBs', 'hbm'):
            if key in peaks:
                return float(peaks[key]), 'measured'
    except (OSError, ValueError):
        pass
    return 6650.0, 'fallback'


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join(ROOT, 'gpurun_out', f'clocks_{index}.csv')

    def __enter__(self):
        os.makedirs(os.path.dirname(self.path), exist_ok=True)
        try:
            self.handle = open(self.path, 'w')
            self.proc = subprocess.Popen(
                ['nvidia-smi', f'--id={self.index}',
                 '--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,'
                 'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
                 'clocks_event_reasons.sw_power_cap', '--format=csv,noheader,nounits', '-lms', '200'],
                stdout=self.handle, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.handle.close()

    def summary(self) -> dict:
        sms, maxes, reasons = [], [], set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        try:
            with open(self.path, encoding='utf-8') as handle:
                for line in handle:
                    parts = [p.strip() for p in line.split(',')]
                    if len(parts) < 6:
                        continue
                    try:
                        sms.append(float(parts[0]))
                        maxes.append(float(parts[1]))
                    except ValueError:
                        continue
                    for name, flag in zip(names, parts[2:6]):
                        if flag.lower() == 'active':
                            reasons.add(name)
        except OSError:
            pass
        return {'sm_mhz': statistics.median(sms) if sms else None,
                'sm_max_mhz': max(maxes) if maxes else None, 'reasons': sorted(reasons), 'samples': len(sms)}


def slice_of(cfg: dict, world: int, rank: int) -> tuple[int, int]:
    """This rank's environment count and first index."""
    if cfg['split']:
        per = cfg['envs'] // world
        return per, rank * per
    return cfg['envs'], rank * cfg['envs']


def assignment_of(cfg: dict, envs: int, first: int):
    if cfg['interleave'] is None:
        return None
    pattern = cfg['interleave']
    return [pattern[(first + i) % len(pattern)] for i in range(envs)]


def workload_config(cfg_id: int, envs: int, world: int) -> dict:
    cfg = CONFIGS[cfg_id]
    return {'workload': f"configuration {cfg_id}: {cfg['text']}; auto-reset, seeded uniform int32 actions in [0,19)",
            'envs_per_gpu': envs, 'parallelism': f'env-slice x{world}',
            'l2': 'state larger than L2 (environments x ~370 KB matches), no flush needed'
                  if envs * 370_000 > 126e6 else 'state fits L2: timed steps run on resident state'}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_reference(cfg_id: int, envs: int, steps: int, warmup: int, threads: int) -> dict:
    """The reference CPU backend on this host: env-steps/s over a bounded sample of the workload."""
    import random

    from cuju_b200.environment import resolve_asset
    from oracle.driver import OracleBatch

    cfg = CONFIGS[cfg_id]
    paths, counts = [], []
    for i, a in enumerate(cfg['assets']):
        path, count = resolve_asset(a)
        paths.append(path)
        counts.append(cfg['agents'][i] if cfg['agents'] else count)
    difficulty = None
    if cfg['difficulty'] is not None:
        difficulty = [(-1.0 if v is None else v) for _ in range(envs) for v in cfg['difficulty']]
    animations = os.path.join(ROOT, 'cuju_b200', 'data', 'animations.bin')
    batch = OracleBatch(paths, counts, envs, 0, animations, threads=threads, difficulty=difficulty,
                        assignment=assignment_of(cfg, envs, 0), stack=4 if cfg['stacked'] else 1)
    rng = random.Random(0)
    batch.reset(list(range(envs)))

    def one_step():
        batch.step([rng.randrange(19) for _ in range(envs * batch.agents)])
        if cfg['masked']:
            mask = [1 if rng.random() < cfg['masked'] else 0 for _ in range(envs)]
            if any(mask):
                batch.reset_masked(mask, [rng.randrange(2**32) if m else -1 for m in mask])

    for _ in range(warmup):
        one_step()
    start = time.perf_counter()
    for _ in range(steps):
        one_step()
    elapsed = time.perf_counter() - start
    batch.close()
    return {'value': envs * steps / elapsed, 'elapsed_s': elapsed, 'envs': envs, 'steps': steps}


def reference_envs(cfg_id: int, threads: int) -> int:
    # 64 environments per host thread (the reference saturates near 16 per thread), at most the
    # configuration's own count.
    return min(CONFIGS[cfg_id]['envs'], 64 * threads)


def run_reference(args) -> None:
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    threads = host_threads()
    envs = reference_envs(args.config, threads)
    steps = max(1, args.steps)
    result = cpu_reference(args.config, envs, steps, max(1, args.warmup), threads)
    value = result['value']
    world = args.gpus
    gpu_envs, _ = slice_of(CONFIGS[args.config], world, 0)
    line = {
        'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': 'env steps/s', 'n_gpus': args.gpus,
        'steps': steps, 'warmup': args.warmup, 'ms_per_step': 1000 * result['elapsed_s'] / steps,
        'higher_is_better': True, 'scaling': 'strong' if CONFIGS[args.config]['split'] else 'weak',
        'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'config': workload_config(args.config, gpu_envs, world),
        'cpu_baseline': {'value': value, 'unit': 'env steps/s', 'cores': threads, 'kind': 'reference',
                         'sample': f'{envs} envs (64 per host thread, at most the configuration\'s count) x {steps} '
                                   f'steps after {args.warmup} warm-up steps of the same workload, reference CPU '
                                   'backend built from source'},
        'e2e': {'value': value, 'unit': 'env steps/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def make_batch(cfg: dict, envs: int, first: int, device, lanes: int = 0):
    from cuju_b200 import BatchEnvironment

    options = {}
    if cfg['agents']:
        options['agent_counts'] = cfg['agents']
    if lanes:
        options['lanes_per_environment'] = lanes
    return BatchEnvironment(cfg['assets'] if len(cfg['assets']) > 1 else cfg['assets'][0], environment_count=envs,
                            seed=0, device=device, difficulty=None if cfg['difficulty'] is None else [cfg['difficulty']],
                            first_index=first, assignment=assignment_of(cfg, envs, first), stacked=cfg['stacked'],
                            **options)


def waves_for(envs: int, lanes: int, sms: int) -> int:
    """Kernel launches of one step (or one masked reset) of `envs` environments on `sms` SMs: a
    batch above four warps per SM runs as equal waves of launches. Mirrors the library's choice
    (cuju_b200/csrc/kernels.cu: default_crew_log2, wave_size); `lanes` 0 is its default layout."""
    if lanes:
        log2 = max(0, lanes.bit_length() - 1)
    else:
        log2 = 0
        while log2 < 5 and (envs << (log2 + 1)) <= sms * 4 * 32:
            log2 += 1
    full = (sms * 4 * 32) >> log2
    return 1 if envs <= full else -(-envs // full)


def launches_per_step(envs: int, lanes: int, device) -> int:
    import torch

    return waves_for(envs, lanes, torch.cuda.get_device_properties(device).multi_processor_count)


def bytes_per_env_step(cfg: dict, batch, envs: int, first: int) -> float:
    """B = 2*S + 4*A + 4*obs*A + 4*A + 5 per environment (A its agents), plus p*2*S for a masked
    reset; S measured with get_state on one environment of each bundle; the batch mean."""
    assignment = assignment_of(cfg, envs, first) or [0] * envs
    obs = 460 if cfg['stacked'] else 115
    sizes = {}
    for b in sorted(set(assignment)):
        sizes[b] = len(batch.get_state(assignment.index(b)))
    agents = [(cfg['agents'][b][0] + cfg['agents'][b][1]) if cfg['agents'] else batch.agents for b in range(len(cfg['assets']))]
    total = 0.0
    for b in assignment:
        s = sizes[b]
        a = agents[b]
        total += 2 * s + 4 * a + 4 * obs * a + 4 * a + 5 + cfg['masked'] * 2 * s
    return total / envs


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    device = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=600), device_id=device)

    cfg = CONFIGS[args.config]
    envs, first = slice_of(cfg, world, rank)
    if args.envs:
        envs, first = args.envs, rank * args.envs
    batch = make_batch(cfg, envs, first, device, args.lanes)
    agents = batch.agents
    generator = torch.Generator(device=device).manual_seed(1000 + rank)
    total_steps = args.warmup + args.steps
    actions = torch.randint(0, 19, (total_steps, envs, agents), generator=generator, device=device, dtype=torch.int32)
    masks = seeds = None
    if cfg['masked']:
        masks = torch.rand((total_steps, envs), generator=generator, device=device) < cfg['masked']
        drawn = torch.randint(0, 2**32 - 1, (total_steps, envs), generator=generator, device=device, dtype=torch.int64)
        seeds = torch.where(masks, drawn, torch.full_like(drawn, -1))
    reset_seeds = torch.arange(first, first + envs) if cfg['seeds'] == 'index' else None

    def start(b):
        b.reset(seeds=reset_seeds) if reset_seeds is not None else b.reset()

    start(batch)
    per_step_bytes = bytes_per_env_step(cfg, batch, envs, first)
    stream = torch.cuda.current_stream(device)

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    def device_step(b, i):
        b.step(actions[i], synchronize=False)
        if masks is not None:
            b.reset(seeds=seeds[i], mask=masks[i])

    for step in range(args.warmup):
        device_step(batch, step)
    batch.synchronize()
    barrier()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        begin = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        begin.record(stream)
        for i in range(args.steps):
            events[i][0].record(stream)
            batch.step(actions[args.warmup + i], synchronize=False)
            events[i][1].record(stream)
            if masks is not None:
                batch.reset(seeds=seeds[args.warmup + i], mask=masks[args.warmup + i])
        end.record(stream)
        batch.synchronize()
    barrier()
    elapsed_ms = begin.elapsed_time(end)
    kernel_ms = [a.elapsed_time(b) for a, b in events]
    clock = clocks.summary()

    # End to end through the public API: pinned host actions in (and host masks and seeds), the
    # observation, reward and done out. A fresh batch of the same configuration replays the same
    # seeds, warm-up and actions, so the timed steps are the same simulated steps as above (a step's
    # cost depends on the match situation).
    host_actions = actions[args.warmup:].cpu().pin_memory()
    host_masks = masks[args.warmup:].cpu() if masks is not None else None
    host_seeds = seeds[args.warmup:].cpu() if seeds is not None else None
    obs_dev = batch.observation()
    obs_host = torch.empty(obs_dev.shape, dtype=obs_dev.dtype, pin_memory=True)
    reward_host = torch.empty((envs, agents), dtype=torch.float32, pin_memory=True)
    done_host = torch.empty((envs,), dtype=torch.bool, pin_memory=True)
    e2e_steps = max(1, min(args.steps, args.e2e_steps if args.e2e_steps else args.steps))
    batch.close()
    batch = make_batch(cfg, envs, first, device, args.lanes)
    start(batch)
    for step in range(args.warmup):
        device_step(batch, step)
    batch.synchronize()
    barrier()
    e_begin = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_begin.record(stream)
    for i in range(e2e_steps):
        obs, reward, done, _ = batch.step(host_actions[i], synchronize=False)
        obs_host.copy_(obs, non_blocking=True)
        reward_host.copy_(reward, non_blocking=True)
        done_host.copy_(done, non_blocking=True)
        if host_masks is not None and bool(host_masks[i].any()):
            batch.reset(seeds=host_seeds[i].tolist(), mask=host_masks[i])
    e_end.record(stream)
    batch.synchronize()
    barrier()
    e2e_ms = e_begin.elapsed_time(e_end)

    times = torch.tensor([elapsed_ms, e2e_ms], device=device, dtype=torch.float64)
    per_rank = [torch.zeros_like(times) for _ in range(world)]
    if world > 1:
        dist.all_gather(per_rank, times)
    else:
        per_rank = [times]
    rank_ms = [t[0].item() / args.steps for t in per_rank]
    elapsed_ms = max(t[0].item() for t in per_rank)
    e2e_ms = max(t[1].item() for t in per_rank)
    batch.close()

    if rank == 0:
        value = world * envs * args.steps / (elapsed_ms / 1000)
        e2e_value = world * envs * e2e_steps / (e2e_ms / 1000)
        mean_kernel_s = statistics.mean(kernel_ms) / 1000
        achieved = per_step_bytes * envs / mean_kernel_s / 1e9
        peak, peak_kind = measured_peak()
        traffic = TRAFFIC_GB.get(args.config) if envs == CONFIGS[args.config]['envs'] else None
        obs_floats = obs_dev[0].numel()
        line = {
            'metric': METRIC, 'value': value, 'unit': 'env steps/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': elapsed_ms / args.steps, 'higher_is_better': True,
            'scaling': 'strong' if cfg['split'] else 'weak', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic', 'config': workload_config(args.config, envs, world),
            'e2e': {'value': e2e_value, 'unit': 'env steps/s', 'h2d_bytes_per_step': 4 * envs * agents,
                    'd2h_bytes_per_step': envs * obs_floats * 4 + envs * agents * 4 + envs},
            'gpu_launches': args.steps * launches_per_step(envs, args.lanes, device) * (2 if masks is not None else 1),
            'per_rank_ms_per_step': [round(x, 3) for x in rank_ms],
            'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': peak, 'unit': 'GB/s',
                         'frac': achieved / peak, 'traffic': traffic,
                         'note': f'algorithmic {per_step_bytes:.0f} B per env-step (2 x the measured GRF state size '
                                 'plus actions and outputs) x the environments of a launch over the mean CUDA-event '
                                 f'time of a step launch; peak {peak_kind} (of measured); traffic in GB per launch, '
                                 'DRAM read+write of one ncu capture at 8,192 environments scaled to this launch\'s '
                                 'environments'},
            'clocks': clock,
        }
        if args.cpu_baseline and world == 1:
            threads = host_threads()
            # The same match phase as the timed device steps: the same warm-up, then as many steps
            # (a step's cost grows as the matches get going after kick-off).
            cpu_steps = args.cpu_steps or args.steps
            cpu_warmup = max(1, args.warmup)
            cpu = cpu_reference(args.config, reference_envs(args.config, threads), cpu_steps, cpu_warmup, threads)
            line['cpu_baseline'] = {'value': cpu['value'], 'unit': 'env steps/s', 'cores': threads,
                                    'kind': 'reference',
                                    'sample': f"{cpu['envs']} envs x {cpu['steps']} steps after {cpu_warmup} warm-up "
                                              'steps of the same workload (the device line\'s match phase), '
                                              'reference CPU backend built from source'}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument('--gpus', type=int, default=1)
    parser.add_argument('--steps', type=int, default=20)
    parser.add_argument('--warmup', type=int, default=3)
    parser.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    parser.add_argument('--config', type=int, default=3, choices=sorted(CONFIGS))
    parser.add_argument('--envs', type=int, default=0, help='environments per GPU (default: the configuration\'s)')
    parser.add_argument('--lanes', type=int, default=0,
                        help='lanes per environment, 1-32 (default: the library\'s choice for the batch size)')
    parser.add_argument('--e2e-steps', type=int, default=0, help='end-to-end steps (default: --steps)')
    parser.add_argument('--cpu-steps', type=int, default=0, help='CPU baseline steps (default: --steps)')
    parser.add_argument('--no-cpu-baseline', dest='cpu_baseline', action='store_false')
    args = parser.parse_args()
    if args.impl == 'reference':
        run_reference(args)
    else:
        run_b200(args)


if __name__ == '__main__':
    main()
