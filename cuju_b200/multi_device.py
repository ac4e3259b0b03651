"""One batch of environments over several GPUs, and episode totals summed over ranks.

`MultiDeviceBatch` follows the reference class `cuju.MultiDeviceBatch`
(python/cuju/multi_device.py:52-390): the part on device k is a `BatchEnvironment` of its own that
plays environments `start` to `end - 1` of the seed rule through `first_index`, so environment i
plays exactly as environment i of one batch of `environment_count` environments with the same
options. A step starts on every device before it waits for any. Outputs are gathered into tensors
on `output_device`, which the next call overwrites; `parts` gives each part's own zero-copy outputs.
Unlike the reference, every part runs on a CUDA device: this build has no CPU backend.

`EpisodeTotals` keeps running totals of one batch's steps on its device (episodes ended, goals of
each side, summed reward) and sums them over the ranks of a `torch.distributed` group: the one
collective of a multi-process run, taken once at the end and never on the step path.
"""

from __future__ import annotations

from typing import Any

import torch

from .environment import BatchEnvironment
from .errors import ArgumentError, ChoiceError, ClosedError, ConfigurationError, EnvironmentIndexError

__all__ = ['EpisodeTotals', 'MultiDeviceBatch']


def _per_environment(values, start, end, count, error=ConfigurationError):
    """The values of environments `start` to `end - 1`, or the one value shared by every one
    (reference multi_device.py:38-49)."""
    array = torch.as_tensor(values)
    if array.dim() == 0:
        return array.item()
    if array.shape[0] != count:
        raise error(
            f'expected one value, or one for each of the {count} environments, found the shape {tuple(array.shape)}')
    return array[start:end]


class MultiDeviceBatch:
    """A batch whose environments run on several CUDA devices, each a `BatchEnvironment`.

    Attributes:
        parts: the `BatchEnvironment` of each device, in the order of `devices`.
        ranges: the `(start, end)` environments of each part.
        devices: the device of each part; output_device: where `reset` and `step` outputs live.
        environment_count, agents, action_count, squeeze, stacked: as in `BatchEnvironment`;
        left_agents, right_agents: over every environment.
    """

    def __init__(self, assets: str | list[str], devices: list[Any], environment_count: int = 1024,
                 split: list[int] | None = None, output_device: Any = None, assignment: Any = None,
                 game_engine_random_seed: Any = None, **options: Any) -> None:
        self.devices = [self._device(d) for d in devices]
        if not self.devices:
            raise ConfigurationError('expected at least one device')
        for name in ('device', 'first_index'):
            if name in options:
                raise ConfigurationError(f'expected no {name}, which MultiDeviceBatch sets for each part')
        count = len(self.devices)
        if split is None:
            split = [environment_count // count + (part < environment_count % count) for part in range(count)]
        split = [int(size) for size in split]
        if len(split) != count or sum(split) != environment_count or min(split) < 1:
            raise ConfigurationError(f'expected a split of the {environment_count} environments into {count} parts '
                                     f'of at least one, found {split}')
        self.ranges = []
        start = 0
        for size in split:
            self.ranges.append((start, start + size))
            start += size
        self.output_device = self.devices[0] if output_device is None else self._device(output_device)
        self.environment_count = environment_count
        self.parts = []
        try:
            for device, (start, end) in zip(self.devices, self.ranges):
                part_options = dict(options)
                if assignment is not None:
                    part_options['assignment'] = _per_environment(assignment, start, end, environment_count)
                    if isinstance(part_options['assignment'], int):
                        part_options['assignment'] = [part_options['assignment']] * (end - start)
                    else:
                        part_options['assignment'] = part_options['assignment'].tolist()
                if game_engine_random_seed is not None:
                    seeds = _per_environment(game_engine_random_seed, start, end, environment_count)
                    part_options['game_engine_random_seed'] = seeds if isinstance(seeds, int) else seeds.tolist()
                self.parts.append(self._make_part(assets, device, end - start, start, part_options))
        except BaseException:
            self.close()
            raise
        first = self.parts[0]
        for name in ('agents', 'action_count', 'squeeze', 'stacked'):
            setattr(self, name, getattr(first, name))
        self.left_agents = torch.cat([part.left_agents for part in self.parts])
        self.right_agents = torch.cat([part.right_agents for part in self.parts])
        self._gathered = {}

    @staticmethod
    def _device(device: Any) -> torch.device:
        """A CUDA device with an index, from an index, a name or a `torch.device`."""
        device = torch.device('cuda', device) if isinstance(device, int) else torch.device(device)
        if device.type != 'cuda':
            raise ChoiceError(f'expected a CUDA device (this build has no CPU backend), found {device}')
        if device.index is None:
            device = torch.device('cuda', torch.cuda.current_device())
        return device

    def _make_part(self, assets, device, count, first_index, options):
        return BatchEnvironment(assets, environment_count=count, device=device, first_index=first_index, **options)

    # -- lifetime ------------------------------------------------------------------------------
    def close(self) -> None:
        """Closes every part; a second call does nothing, and other calls then raise."""
        for part in getattr(self, 'parts', []):
            part.close()
        self.parts = []
        self._gathered = {}

    def _open_parts(self):
        if not getattr(self, 'parts', None):
            raise ClosedError('the batch is closed')
        return self.parts

    def __reduce__(self):
        raise TypeError('a batch cannot be pickled; create it inside the worker process that uses it')

    # -- outputs -------------------------------------------------------------------------------
    def _gather(self, key, outputs):
        """The parts' outputs on `output_device`, in tensors that `key` reuses from call to call.
        Copies between devices are ordered after the work on both devices' current streams."""
        if isinstance(outputs[0], dict):
            return {name: self._gather((key, name), [o[name] for o in outputs]) for name in outputs[0]}
        gathered = self._gathered.get(key)
        if gathered is None:
            shape = (self.environment_count, *outputs[0].shape[1:])
            gathered = torch.empty(shape, dtype=outputs[0].dtype, device=self.output_device)
            self._gathered[key] = gathered
        for (start, end), output in zip(self.ranges, outputs):
            gathered[start:end].copy_(output, non_blocking=True)
        return gathered

    def _split(self, values):
        if values is None:
            return [None] * len(self.parts)
        return [_per_environment(values, start, end, self.environment_count, ArgumentError)
                for start, end in self.ranges]

    # -- the environment API -------------------------------------------------------------------
    def reset(self, seeds: Any = None, reverse: Any = None) -> Any:
        """Starts the next episode of every environment; returns every observation."""
        observations = []
        for part, part_seeds, part_reverse in zip(self._open_parts(), self._split(seeds), self._split(reverse)):
            observations.append(part.reset(seeds=part_seeds, reverse=part_reverse))
        return self._gather('observation', observations)

    def reset_done(self) -> None:
        """Starts the next episode of every environment whose episode ended (auto_reset off)."""
        for part in self._open_parts():
            part.reset_done()

    def step(self, actions: Any) -> tuple[Any, Any, Any, dict[str, Any]]:
        """One step of every environment: each part takes its rows of `actions` on its own device,
        every part starts before any is waited for, and the outputs are gathered."""
        parts = self._open_parts()
        actions = torch.as_tensor(actions)
        rows = [actions[start:end].to(device, non_blocking=actions.is_cuda)
                for device, (start, end) in zip(self.devices, self.ranges)]
        started = []
        try:
            for part, part_rows in zip(parts, rows):
                part.step_async(part_rows)
                started.append(part)
        except BaseException:
            for part in started:
                part.step_wait()
            raise
        results = [part.step_wait() for part in parts]
        observation, reward, done, information = zip(*results)
        return (self._gather('observation', observation), self._gather('reward', reward),
                self._gather('done', done),
                {name: self._gather(name, [info[name] for info in information]) for name in information[0]})

    def observation(self) -> Any:
        """Every observation of the last `reset` or `step`."""
        return self._gather('observation', [part.observation() for part in self._open_parts()])

    def _part(self, index: int):
        for part, (start, end) in zip(self._open_parts(), self.ranges):
            if start <= index < end:
                return part, index - start
        raise EnvironmentIndexError(f'expected an environment from 0 to {self.environment_count - 1}, found {index}')

    def get_state(self, index: int) -> bytes:
        part, local = self._part(index)
        return part.get_state(local)

    def set_state(self, index: int, state: bytes) -> None:
        part, local = self._part(index)
        part.set_state(local, state)


class EpisodeTotals:
    """Running totals of one batch's steps, on the batch's device: episodes ended, goals of the left
    and of the right team (from `score_reward`, +1 when the left team scores and -1 when the right
    does), and the reward summed over every agent. `all_reduce` sums them over the ranks of a
    process group (NCCL between GPUs, gloo on the CPU) and returns them as a dict."""

    FIELDS = ('episodes', 'left_goals', 'right_goals', 'reward')

    def __init__(self, device: Any = 'cuda') -> None:
        self.values = torch.zeros(len(self.FIELDS), dtype=torch.float64, device=device)

    def update(self, reward: torch.Tensor, done: torch.Tensor, score_reward: torch.Tensor) -> None:
        """Adds one step's outputs, without a host synchronisation."""
        step = torch.stack([
            done.to(torch.float64).sum(),
            (score_reward > 0).to(torch.float64).sum(),
            (score_reward < 0).to(torch.float64).sum(),
            reward.to(torch.float64).sum(),
        ])
        self.values += step.to(self.values.device)

    def all_reduce(self, group: Any = None) -> dict[str, float]:
        """The totals summed over the ranks of `group` (this rank's alone without a process group)."""
        import torch.distributed as dist

        values = self.values.clone()
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(values, op=dist.ReduceOp.SUM, group=group)
        return dict(zip(self.FIELDS, values.tolist()))
