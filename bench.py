"""Throughput of GRF's batched 11-a-side step on B200: environment steps per second.

Workload (the metric's 1-GPU configuration): `11_vs_11_stochastic`, one
controlled agent (the active player), every other player built-in AI at difficulty 0.2 on both
sides, 16,384 environments per GPU, automatic restart, seeded uniform int32 actions in [0, 19).
With N GPUs each rank steps its own contiguous slice of environments (the seed rule's
`first_index = rank * 16384`), so per-GPU work is fixed (weak scaling) and no collective runs on
the step path; the only collectives are the barrier and the max of the timed region over ranks.

`value` times the device step with inputs resident (actions pre-generated on the device); `e2e`
times the same steps through the public API with pinned host actions copied in and the step's
observation, reward and done read back every step. The roofline uses the algorithmic bytes of an
env-step, B = 2*S + 4*A + 460*A*stack + 4*A + 5 (S the scenario's GRF state size), over the CUDA
event duration of the step kernel. `--impl reference` times the reference CPU backend (built from
source into oracle/_ref) on this host's cores on a bounded sample of the same workload.
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

ASSETS = '11_vs_11_stochastic_l1_r0'
DIFFICULTY = (0.2, 0.2)
ENVS_PER_GPU = 16384
METRIC = 'env steps/sec, 11v11 at 1/2/4/8 B200 vs host-CPU path; % HBM roofline'
STATE_BYTES = 106914  # serialized GRF state of 11_vs_11 with one left agent (measured by get_state)
# DRAM bytes (read + write) per env-step of step_kernel: 13.660 GB over one 4,096-environment launch
# (ncu --set full, dram__bytes_read.sum + dram__bytes_write.sum).
TRAFFIC_PER_ENV_STEP = 13.660e9 / 4096


def bytes_per_env_step(agents: int = 1, stack: int = 1, state: int = STATE_BYTES) -> int:
    return 2 * state + 4 * agents + 460 * agents * stack + 4 * agents + 5


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


def cpu_reference(args, envs: int, steps: int, warmup: int, threads: int) -> dict:
    """The reference CPU backend on this host: env-steps/s over a bounded sample."""
    import random

    from cuju_b200.environment import resolve_asset
    from oracle.driver import OracleBatch

    path, counts = resolve_asset(ASSETS)
    animations = os.path.join(ROOT, 'cuju_b200', 'data', 'animations.bin')
    difficulty = [v for _ in range(envs) for v in DIFFICULTY]
    batch = OracleBatch([path], [counts], envs, 0, animations, threads=threads, difficulty=difficulty)
    rng = random.Random(0)
    batch.reset(list(range(envs)))
    for _ in range(warmup):
        batch.step([rng.randrange(19) for _ in range(envs * batch.agents)])
    start = time.perf_counter()
    for _ in range(steps):
        batch.step([rng.randrange(19) for _ in range(envs * batch.agents)])
    elapsed = time.perf_counter() - start
    batch.close()
    return {'value': envs * steps / elapsed, 'elapsed_s': elapsed, 'envs': envs, 'steps': steps}


def workload_config(envs: int, world: int) -> dict:
    return {'workload': f'{ASSETS}, 1 controlled agent, difficulty {DIFFICULTY}, {envs} envs per GPU, '
                        'auto-reset, seeded uniform int32 actions in [0,19)',
            'envs_per_gpu': envs, 'parallelism': f'env-slice x{world}',
            'l2': 'state larger than L2 (16,384 x ~370 KB worlds), no flush needed'}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args) -> None:
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    threads = host_threads()
    envs = 16 * threads
    steps = max(1, args.steps)
    result = cpu_reference(args, envs, steps, max(1, args.warmup), threads)
    value = result['value']
    line = {
        'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': 'env steps/s', 'n_gpus': args.gpus,
        'steps': steps, 'warmup': args.warmup, 'ms_per_step': 1000 * result['elapsed_s'] / steps,
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'config': workload_config(args.envs, args.gpus),
        'cpu_baseline': {'value': value, 'unit': 'env steps/s', 'cores': threads, 'kind': 'reference',
                         'sample': f'{envs} envs (16 per host thread) x {steps} steps after {args.warmup} '
                                   'warm-up steps of the same workload, reference CPU backend built from source'},
        'e2e': {'value': value, 'unit': 'env steps/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


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

    from cuju_b200 import BatchEnvironment

    envs = args.envs
    batch = BatchEnvironment(ASSETS, environment_count=envs, seed=0, device=device, difficulty=[DIFFICULTY],
                             first_index=rank * envs)
    agents = batch.agents
    generator = torch.Generator(device=device).manual_seed(1000 + rank)
    total_steps = args.warmup + args.steps
    actions = torch.randint(0, 19, (total_steps, envs, agents), generator=generator, device=device, dtype=torch.int32)
    batch.reset(seeds=torch.arange(rank * envs, (rank + 1) * envs))
    stream = torch.cuda.current_stream(device)

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    for step in range(args.warmup):
        batch.step(actions[step], synchronize=False)
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
        end.record(stream)
        batch.synchronize()
    barrier()
    elapsed_ms = begin.elapsed_time(end)
    kernel_ms = [a.elapsed_time(b) for a, b in events]
    clock = clocks.summary()

    # End to end through the public API: pinned host actions in, observation/reward/done out. A
    # fresh batch of the same configuration replays the same seeds, warm-up and actions, so the
    # timed steps are the same simulated steps as above (a step's cost depends on the match
    # situation, and a second episode of the same batch would play the mirrored variant).
    host_actions = actions[args.warmup:].cpu().pin_memory()
    obs_host = torch.empty((envs, agents, 115), dtype=torch.float32, pin_memory=True)
    reward_host = torch.empty((envs, agents), dtype=torch.float32, pin_memory=True)
    done_host = torch.empty((envs,), dtype=torch.bool, pin_memory=True)
    e2e_steps = max(1, min(args.steps, args.e2e_steps if args.e2e_steps else args.steps))
    batch.close()
    batch = BatchEnvironment(ASSETS, environment_count=envs, seed=0, device=device, difficulty=[DIFFICULTY],
                             first_index=rank * envs)
    batch.reset(seeds=torch.arange(rank * envs, (rank + 1) * envs))
    for step in range(args.warmup):
        batch.step(actions[step], synchronize=False)
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
    e_end.record(stream)
    batch.synchronize()
    barrier()
    e2e_ms = e_begin.elapsed_time(e_end)

    times = torch.tensor([elapsed_ms, e2e_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_ms = times.tolist()
    batch.close()

    if rank == 0:
        value = world * envs * args.steps / (elapsed_ms / 1000)
        e2e_value = world * envs * e2e_steps / (e2e_ms / 1000)
        per_step = bytes_per_env_step(agents)
        mean_kernel_s = statistics.mean(kernel_ms) / 1000
        achieved = per_step * envs / mean_kernel_s / 1e9
        peak, peak_kind = measured_peak()
        line = {
            'metric': METRIC, 'value': value, 'unit': 'env steps/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': elapsed_ms / args.steps, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
            'config': workload_config(envs, world),
            'e2e': {'value': e2e_value, 'unit': 'env steps/s', 'h2d_bytes_per_step': 4 * envs * agents,
                    'd2h_bytes_per_step': envs * agents * 115 * 4 + envs * agents * 4 + envs},
            'gpu_launches': args.steps,
            'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': peak, 'unit': 'GB/s',
                         'frac': achieved / peak, 'traffic': TRAFFIC_PER_ENV_STEP * envs / 1e9,
                         'note': f'algorithmic {per_step} B per env-step x {envs} env-steps per launch over the '
                                 f'mean CUDA-event time of a step launch; peak {peak_kind} (of measured); traffic '
                                 'in GB per launch, DRAM read+write of one ncu capture at 4,096 environments '
                                 'scaled by the environments processed'},
            'clocks': clock,
        }
        if args.cpu_baseline:
            threads = host_threads()
            cpu = cpu_reference(args, 16 * threads, args.cpu_steps, 2, threads)
            line['cpu_baseline'] = {'value': cpu['value'], 'unit': 'env steps/s', 'cores': threads,
                                    'kind': 'reference',
                                    'sample': f"{cpu['envs']} envs x {cpu['steps']} steps of the same scenario, "
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
    parser.add_argument('--envs', type=int, default=ENVS_PER_GPU)
    parser.add_argument('--e2e-steps', type=int, default=0, help='end-to-end steps (default: --steps)')
    parser.add_argument('--cpu-steps', type=int, default=60)
    parser.add_argument('--no-cpu-baseline', dest='cpu_baseline', action='store_false')
    args = parser.parse_args()
    if args.impl == 'reference':
        run_reference(args)
    else:
        run_b200(args)


if __name__ == '__main__':
    main()
