"""`BatchEnvironment`: the reference's batched GRF environment API on the B200 library.

Names, arguments and results follow the reference class `cuju.BatchEnvironment`
(python/cuju/_batch/environment.py:270-1560) for the simple115 representations: one reset or step
of the whole batch per call, outputs as zero-copy views of device buffers, automatic reset with
`final_observation`, and `get_state` bytes in GRF's format (a pickle of the episode logic, then the
engine state; python/cuju/_batch/state.py:44-77).
"""

from __future__ import annotations

import ctypes
import io
import os
import pickle
import re
import struct
from typing import Any

import torch

from . import _native
from .errors import (ActionRangeError, ArgumentError, ChoiceError, ClosedError, ConfigurationError, LibraryError,
                     MissingFileError, StateError, from_library)

_REPRESENTATIONS = {'simple115': 1, 'simple115v2': 2, 'extracted': 4, 'raw': 8}
_RAW_TYPES = {0: ('<f4', torch.float32), 1: ('<i4', torch.int32), 2: ('|b1', torch.bool), 3: ('|u1', torch.uint8)}
_ACTION_SETS = {'default': 0, 'v2': 1, 'full': 2}
_ACTION_COUNTS = {0: 19, 1: 20, 2: 33}


def bundled_assets() -> list[str]:
    """The asset bundles staged with the package, such as `5_vs_5_l0_r0`."""
    directory = os.path.join(_native.DATA_DIRECTORY, 'assets')
    if not os.path.isdir(directory):
        return []
    return sorted(n[: -len('.cjb')] for n in os.listdir(directory) if n.endswith('.cjb'))


def _split_name(name):
    m = re.fullmatch(r'(.+)_l(\d+)_r(\d+)', name)
    return None if m is None else (m.group(1), int(m.group(2)), int(m.group(3)))


def resolve_asset(asset: str) -> tuple[str, tuple[int, int]]:
    """The bundle path of a path or `<scenario>_l<left>_r<right>` name, and the agents it asks for
    (-1 keeps the bundle's), as python/cuju/_batch/assets.py:39 resolves them."""
    if os.path.isfile(asset):
        return asset, (-1, -1)
    directory = os.path.join(_native.DATA_DIRECTORY, 'assets')
    shipped = os.path.join(directory, asset + '.cjb')
    if os.path.isfile(shipped):
        return shipped, (-1, -1)
    split = _split_name(asset)
    scenarios = {s[0] for s in map(_split_name, bundled_assets()) if s}
    if split is None and asset in scenarios:
        split = (asset, 1, 0)
    if split:
        scenario, left, right = split
        bases = [n for n in bundled_assets() if (_split_name(n) or ('',))[0] == scenario]
        if bases:
            base = min(bases, key=lambda n: sum(_split_name(n)[1:]))
            return os.path.join(directory, base + '.cjb'), (left, right)
    raise MissingFileError(f'expected an asset bundle path or `<scenario>_l<left>_r<right>`, found {asset!r}')


class _DeviceArray:
    """A device buffer as `__cuda_array_interface__`, so torch views it without a copy."""

    def __init__(self, pointer: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {
            'shape': shape, 'typestr': typestr, 'data': (pointer, False), 'version': 3, 'strides': None,
        }


def _pickle_int(v: int) -> bytes:
    return b'J' + struct.pack('<i', v)


def _pickle_str(v: str) -> bytes:
    d = v.encode()
    return b'X' + struct.pack('<I', len(d)) + d


def pickle_episode(episode: list[int], collected: list[int] | None) -> bytes:
    """GRF's state pickle of the episode logic (protocol 2, written by opcode)."""
    logic = b''.join(
        _pickle_str(k) + _pickle_int(v)
        for k, v in zip(('previous_score_diff', 'previous_game_mode', 'prev_ball_owned_team'), episode)
    )
    data = (b'\x80\x02}(' + _pickle_str('FootballEnvCore') + b'cgfootball.env.football_env_core\nEnvState\n'
            + b')\x81}(' + logic + b'ub')
    if collected is not None:
        data += _pickle_str('CheckpointRewardWrapper') + b'}(' + b''.join(
            _pickle_int(a) + _pickle_int(c) for a, c in enumerate(collected) if c) + b'u'
    return data + b'u.'


class _Stub:
    """Stands in for any class a GRF state pickle names; BUILD fills its __dict__."""


class _EpisodeUnpickler(pickle.Unpickler):
    def find_class(self, module, name):
        return _Stub


def unpickle_episode(data: bytes, agents: int) -> list[int]:
    """The episode values (3 + agents) of GRF's state pickle: score difference, game mode and
    ball-owning team after the previous step, then each agent's collected checkpoints."""
    state = _EpisodeUnpickler(io.BytesIO(data)).load()
    core = state['FootballEnvCore'].__dict__
    values = [int(core['previous_score_diff']), int(core['previous_game_mode']), int(core['prev_ball_owned_team'])]
    collected = state.get('CheckpointRewardWrapper', {})
    return values + [int(collected.get(agent, 0)) for agent in range(agents)]


class BatchEnvironment:
    """A batch of GRF environments stepped on one B200, one lane per environment."""

    def __init__(
        self,
        assets: str | list[str],
        animations: str | None = None,
        environment_count: int = 1024,
        representation: str = 'simple115v2',
        rewards: str = 'scoring',
        action_set: str = 'default',
        seed: int = 0,
        numpy_legacy: bool = True,
        auto_reset: bool = True,
        library: str | None = None,
        assignment: Any = None,
        difficulty: list[tuple[float | None, float | None]] | None = None,
        device: str | torch.device = 'cuda',
        physics_steps_per_frame: int = 10,
        stacked: bool = False,
        game_engine_random_seed: Any = None,
        squeeze: bool = False,
        agent_counts: list[tuple[int | None, int | None]] | None = None,
        episode_number: int = 0,
        first_index: int = 0,
        channel_dimensions: tuple[int, int] = (96, 72),
        lanes_per_environment: int | None = None,
    ):
        if representation not in _REPRESENTATIONS:
            raise ChoiceError(f'expected one of {sorted(_REPRESENTATIONS)}, found {representation!r}')
        if action_set not in _ACTION_SETS:
            raise ChoiceError(f'expected one of {sorted(_ACTION_SETS)}, found {action_set!r}')
        reward_names = [r.strip() for r in rewards.split(',') if r.strip()]
        if not reward_names or reward_names[0] != 'scoring' or not set(reward_names) <= {'scoring', 'checkpoints'}:
            raise ConfigurationError(f"expected 'scoring' or 'scoring,checkpoints', found {rewards!r}")
        self._torch_device = torch.device(device)
        if self._torch_device.type != 'cuda':
            raise ChoiceError(f'expected a CUDA device (this build has no CPU backend), found {self._torch_device}')
        if self._torch_device.index is None:
            self._torch_device = torch.device('cuda', torch.cuda.current_device())
        self._library = _native.load(library)
        names = [assets] if isinstance(assets, str) else list(assets)
        resolved = [resolve_asset(a) for a in names]
        counts = []
        for (path, (left, right)), pair in zip(resolved, agent_counts or [(None, None)] * len(resolved)):
            left = left if pair[0] is None else pair[0]
            right = right if pair[1] is None else pair[1]
            counts += [left, right]
        self._requested = names
        self._paths = [p.encode() for p, _ in resolved]
        path_array = (ctypes.c_char_p * len(self._paths))(*self._paths)
        counts_array = (ctypes.c_int * len(counts))(*counts)
        assignment_array = None
        if assignment is not None:
            assignment_array = (ctypes.c_int * environment_count)(*[int(x) for x in assignment])
        fixed_array = None
        if game_engine_random_seed is not None:
            seeds = game_engine_random_seed
            if isinstance(seeds, int):
                seeds = [seeds] * environment_count
            fixed_array = (ctypes.c_longlong * environment_count)(*[int(x) for x in seeds])
        self._checkpoints = 'checkpoints' in reward_names
        self.stacked = bool(stacked)
        self.squeeze = bool(squeeze)
        animations_path = (animations or os.path.join(_native.DATA_DIRECTORY, 'animations.bin')).encode()
        config = _native.Configuration(
            version=_native.CONFIGURATION_VERSION, assets=path_array, asset_count=len(self._paths),
            assignment=ctypes.cast(assignment_array, ctypes.c_void_p) if assignment_array else None,
            animations=animations_path, environment_count=environment_count, seed=seed,
            action_set=_ACTION_SETS[action_set], observation=_REPRESENTATIONS[representation],
            checkpoints=int(self._checkpoints), numpy_legacy=int(numpy_legacy), auto_reset=int(auto_reset),
            threads=0, ticks_per_step=physics_steps_per_frame, smm_width=int(channel_dimensions[0]),
            smm_height=int(channel_dimensions[1]),
            stack=4 if stacked else 1,
            fixed_seeds=ctypes.cast(fixed_array, ctypes.c_void_p) if fixed_array else None,
            agent_counts=ctypes.cast(counts_array, ctypes.c_void_p), episode_number=episode_number,
            first_index=first_index, allocate=None, release=None, allocator_context=None,
            pin_threads=0, numa=0, page_aligned=0,
        )
        with torch.cuda.device(self._torch_device):
            handle = self._library.cuju_environment_create(ctypes.byref(config))
        if not handle:
            raise from_library(self._library.cuju_last_error().decode())
        self._native_handle = handle
        self.environment_count = environment_count
        if lanes_per_environment is not None:
            self.set_lanes_per_environment(lanes_per_environment)
        from . import operators

        self._operator_key = operators.register(self)
        left = (ctypes.c_int * environment_count)()
        right = (ctypes.c_int * environment_count)()
        self.agents = self._library.cuju_environment_agents(handle, left, right)
        self.left_agents = torch.tensor(list(left), dtype=torch.int32)
        self.right_agents = torch.tensor(list(right), dtype=torch.int32)
        self.action_count = _ACTION_COUNTS[_ACTION_SETS[action_set]]
        self.torch_device = self._torch_device
        if difficulty is not None:
            per_bundle = [(-1.0 if l is None else float(l), -1.0 if r is None else float(r)) for l, r in difficulty]
            bundle_of = [0] * environment_count if assignment is None else [int(x) for x in assignment]
            values = (ctypes.c_float * (2 * environment_count))(*[v for b in bundle_of for v in per_bundle[b]])
            self._check(self._library.cuju_environment_set_difficulty(handle, values))
        stack = 4 if stacked else 1
        self._raw = representation == 'raw'
        self._smm = representation == 'extracted'
        if self._smm:
            # GRF's SMM is [height, width, channels] for `channel_dimensions` = (width, height).
            self._observation_shape = (environment_count, self.agents, int(channel_dimensions[1]),
                                       int(channel_dimensions[0]), 4 * stack)
        else:
            self._observation_shape = (environment_count, self.agents, 115 * stack)
        self.channel_dimensions = (int(channel_dimensions[0]), int(channel_dimensions[1]))
        self._views = {}

    # -- plumbing ------------------------------------------------------------------------------
    def _check(self, status: int) -> None:
        if status == -2:
            raise ActionRangeError(self._library.cuju_last_error().decode())
        if status != 0:
            raise from_library(self._library.cuju_last_error().decode())

    @property
    def _handle(self):
        # Every library call goes through here, so a call after close raises instead of passing
        # the library a null batch.
        handle = self.__dict__.get('_native_handle')
        if not handle:
            raise ClosedError('the batch is closed')
        return handle

    def _stream(self) -> int:
        return torch.cuda.current_stream(self._torch_device).cuda_stream

    def _view(self, name: str, shape: tuple[int, ...], typestr: str, dtype: torch.dtype) -> torch.Tensor:
        if name not in self._views:
            pointer = self._library.cuju_environment_buffer(self._handle, name.encode())
            if not pointer:
                raise LibraryError(f'the batch has no buffer {name}')
            self._views[name] = torch.as_tensor(_DeviceArray(pointer, shape, typestr), device=self._torch_device)
        return self._views[name]

    def _raw_arrays(self, buffer: str) -> dict[str, torch.Tensor]:
        """GRF's raw observation as a dict of arrays [environments, agents, ...] over `buffer`."""
        key = ('raw-dict', buffer)
        if key not in self._views:
            base = self._library.cuju_environment_buffer(self._handle, buffer.encode())
            if not base:
                raise LibraryError(f'the batch has no buffer {buffer}')
            arrays = {}
            kind, dims, offset = ctypes.c_int(), (ctypes.c_int * 2)(), ctypes.c_ulonglong()
            for field in range(64):
                name = self._library.cuju_environment_raw_field(
                    self._handle, field, ctypes.byref(kind), dims, ctypes.byref(offset))
                if not name:
                    break
                typestr, dtype = _RAW_TYPES[kind.value]
                shape = (self.environment_count, self.agents) + tuple(d for d in dims if d)
                arrays[name.decode()] = torch.as_tensor(
                    _DeviceArray(base + offset.value, shape, typestr), device=self._torch_device)
            self._views[key] = arrays
        return self._views[key]

    def _outputs(self):
        e, a = self.environment_count, self.agents
        if self._raw:
            obs, final = self._raw_arrays('raw'), self._raw_arrays('final_raw')
        elif self._smm:
            obs = self._view('smm', self._observation_shape, '|u1', torch.uint8)
            final = self._view('final_smm', self._observation_shape, '|u1', torch.uint8)
        else:
            obs = self._view('simple115', self._observation_shape, '<f4', torch.float32)
            final = self._view('final_simple115', self._observation_shape, '<f4', torch.float32)
        reward = self._view('reward', (e, a), '<f4', torch.float32)
        done = self._view('done', (e,), '|b1', torch.bool)
        score = self._view('score_reward', (e,), '<i4', torch.int32)
        if self.squeeze and a == 1 and not self._raw:
            obs, final, reward = obs.squeeze(1), final.squeeze(1), reward.squeeze(1)
        return obs, reward, done, final, score

    # -- the environment API -------------------------------------------------------------------
    def reset(self, seeds: Any = None, reverse: Any = None, mask: Any = None) -> torch.Tensor:
        """Starts the next episode of every environment (or of those `mask` selects).

        Seeds given as a CUDA tensor take the device path (`cuju_b200_environment_reset_masked_device`):
        the mask, if any, must be a CUDA tensor too, nothing is read back to the host and nothing
        synchronises, so the reset can follow a step inside one captured graph. A negative device
        seed draws the next seed, as -1 does; the device path takes no `reverse`.
        """
        e = self.environment_count
        if isinstance(seeds, torch.Tensor) and seeds.is_cuda:
            return self._reset_device(seeds, mask, reverse)
        seed_t = None if seeds is None else torch.as_tensor(seeds, dtype=torch.int64).reshape(-1).expand(e).contiguous()
        rev_t = None if reverse is None else torch.as_tensor(reverse, dtype=torch.int32).reshape(-1).expand(e).contiguous()
        if seed_t is not None and bool(((seed_t < -1) | (seed_t > 4294967295)).any()):
            raise ArgumentError(f'expected seeds from 0 to 4294967295, or -1 to draw, found {seed_t.tolist()}')
        with torch.cuda.device(self._torch_device):
            if mask is not None or (seed_t is not None and bool((seed_t == -1).any())):
                mask_t, on_device = None, 0
                if mask is not None:
                    mask_t = torch.as_tensor(mask).to(torch.uint8)
                    on_device = int(mask_t.is_cuda)
                    mask_t = mask_t.contiguous()
                self._check(self._library.cuju_environment_reset_masked(
                    self._handle, None if mask_t is None else mask_t.data_ptr(), on_device,
                    None if seed_t is None else seed_t.data_ptr(),
                    None if rev_t is None else rev_t.data_ptr(), self._stream(), int(mask is None)))
            else:
                seeds32 = None if seed_t is None else (ctypes.c_uint * e)(*[int(x) for x in seed_t.tolist()])
                self._check(self._library.cuju_environment_reset(
                    self._handle, seeds32, None if rev_t is None else rev_t.data_ptr(), self._stream()))
        return self._outputs()[0]

    def _reset_device(self, seeds: torch.Tensor, mask: Any, reverse: Any) -> torch.Tensor:
        e = self.environment_count
        if reverse is not None:
            raise ArgumentError('a reset with device seeds takes no reverse flags')
        if mask is not None and not (isinstance(mask, torch.Tensor) and mask.is_cuda):
            raise ArgumentError('a reset with device seeds takes its mask on a CUDA device too')
        seed_t = seeds.to(self._torch_device, torch.int64).reshape(-1).expand(e).contiguous()
        mask_t = None if mask is None else mask.to(self._torch_device, torch.uint8).reshape(-1).expand(e).contiguous()
        with torch.cuda.device(self._torch_device):
            self._check(self._library.cuju_b200_environment_reset_masked_device(
                self._handle, None if mask_t is None else mask_t.data_ptr(), seed_t.data_ptr(), self._stream()))
        # The reset reads the staged tensors on the stream; keep them alive until it has run.
        self._device_reset_inputs = (seed_t, mask_t)
        return self._outputs()[0]

    def reset_done(self) -> None:
        """Starts the next episode of every environment whose episode ended (auto_reset off); under
        `torch.compile` through the operator `cuju_b200::reset_done`."""
        if torch.compiler.is_compiling():
            torch.ops.cuju_b200.reset_done(self._operator(), self._operator_tensors())
            return
        with torch.cuda.device(self._torch_device):
            self._check(self._library.cuju_environment_reset_done(self._handle, self._stream()))

    def step(self, actions: Any, synchronize: bool = True):
        """One step of every environment: returns observation, reward, done and an info dict
        with `final_observation` and `score_reward`. Under `torch.compile` the step goes through the
        operator `cuju_b200::step` (operators.py), so the compiled graph keeps it without a break."""
        if torch.compiler.is_compiling():
            return self._compiled_step(actions)
        a = torch.as_tensor(actions)
        if a.dim() == 1:
            a = a.reshape(self.environment_count, -1)
        a = a.to(torch.int32).contiguous()
        with torch.cuda.device(self._torch_device):
            self._check(self._library.cuju_environment_step(
                self._handle, a.data_ptr(), int(a.is_cuda), self._stream(), int(synchronize)))
        obs, reward, done, final, score = self._outputs()
        return obs, reward, done, {'final_observation': final, 'score_reward': score}

    # -- the path of torch.compile (python/cuju/_batch/environment.py:983-1056) ----------------
    def _operator_tensors(self) -> list[torch.Tensor]:
        """The output tensors the operators declare mutated: every array of the observation and
        of the final observation, the reward, done and score_reward."""
        obs, reward, done, final, score = self._outputs()
        tensors = []
        for output in (obs, reward, done, final, score):
            tensors += [output[k] for k in sorted(output)] if isinstance(output, dict) else [output]
        return tensors

    def _operator(self):
        return self._operator_key

    def _device_step(self, actions: torch.Tensor) -> None:
        with torch.cuda.device(self._torch_device):
            self._check(self._library.cuju_environment_step(self._handle, actions.data_ptr(), 1, self._stream(), 0))

    def _device_reset_done(self) -> None:
        with torch.cuda.device(self._torch_device):
            self._check(self._library.cuju_environment_reset_done(self._handle, self._stream()))

    def _compiled_step(self, actions: Any):
        shape = (self.environment_count, self.agents)
        actions = torch.as_tensor(actions)
        if actions.is_floating_point() or actions.is_complex():
            raise TypeError(f'expected integer action indices, found {actions.dtype}')
        if tuple(actions.shape) != shape and not (self.agents == 1 and tuple(actions.shape) == shape[:1]):
            raise ArgumentError(f'expected actions of the shape {shape}, found {tuple(actions.shape)}')
        actions = actions.to(self._torch_device, torch.int32).reshape(shape).contiguous()
        torch.ops.cuju_b200.step(self._operator(), actions, self._operator_tensors())
        obs, reward, done, final, score = self._outputs()
        return obs, reward, done, {'final_observation': final, 'score_reward': score}

    def step_async(self, actions: Any) -> None:
        """Starts one step of every environment on the current stream and returns at once (host
        actions are copied before it returns); `step_wait` gives the outputs."""
        a = torch.as_tensor(actions)
        if a.dim() == 1:
            a = a.reshape(self.environment_count, -1)
        a = a.to(torch.int32).contiguous()
        with torch.cuda.device(self._torch_device):
            self._check(self._library.cuju_environment_step_async(
                self._handle, a.data_ptr(), int(a.is_cuda), self._stream()))
        self._async_actions = a

    def step_wait(self):
        """Waits for the step `step_async` started and returns what `step` returns."""
        self._check(self._library.cuju_environment_step_wait(self._handle))
        self.synchronize()
        self._async_actions = None
        obs, reward, done, final, score = self._outputs()
        return obs, reward, done, {'final_observation': final, 'score_reward': score}

    def observation(self):
        """The observation of every agent that the last reset or step wrote."""
        return self._outputs()[0]

    def raw(self) -> dict[str, torch.Tensor]:
        """GRF's raw observation of every agent from the last reset or step, one tensor per key
        (python/cuju/_batch/environment.py:1268); views of the batch's buffer, which the next call
        overwrites. Raises ConfigurationError unless the batch's representation is `raw`."""
        if not self._raw:
            raise ConfigurationError('expected a batch with the raw representation')
        return self._raw_arrays('raw')

    def final_raw(self) -> dict[str, torch.Tensor]:
        """The raw observation of the step that ended each environment's last episode, as `raw`
        returns it (python/cuju/_batch/environment.py:1278)."""
        if not self._raw:
            raise ConfigurationError('expected a batch with the raw representation')
        return self._raw_arrays('final_raw')

    @property
    def scenario_name(self) -> str:
        """The scenarios the batch was created with, by name without folders or suffixes, each
        once, joined by ', ' (python/cuju/_batch/environment.py:710)."""
        names = []
        for asset in self._requested:
            name = os.path.basename(os.fspath(asset))
            for suffix in ('.cjb', '.py'):
                if name.endswith(suffix):
                    name = name[:-len(suffix)]
            if name not in names:
                names.append(name)
        return ', '.join(names)

    def synchronize(self) -> None:
        with torch.cuda.device(self._torch_device):
            self._check(self._library.cuju_environment_synchronize(self._handle, self._stream()))

    def engine_state(self, index: int) -> tuple[bytes, list[int]]:
        """The engine bytes of environment `index` and its episode values (3 + agents)."""
        episode = (ctypes.c_int * (3 + _native.MAXIMUM_AGENTS))()
        size = ctypes.c_ulonglong()
        torch.cuda.synchronize(self._torch_device)
        with torch.cuda.device(self._torch_device):
            pointer = self._library.cuju_environment_get_state(self._handle, index, ctypes.byref(size), episode)
        if not pointer:
            raise from_library(self._library.cuju_last_error().decode())
        return ctypes.string_at(pointer, size.value), list(episode)

    def get_state(self, index: int) -> bytes:
        """The state of environment `index` in GRF's byte format (episode pickle, then engine)."""
        match, episode = self.engine_state(index)
        collected = episode[3: 3 + self.agents] if self._checkpoints else None
        data = pickle_episode(episode[:3], collected)
        return struct.pack('<i', len(data)) + data + match

    def set_engine_state(self, index: int, match: bytes, episode: list[int]) -> None:
        """Sets environment `index` to GRF engine bytes and its episode values (3 + agents), as
        `engine_state` returns them; the state's scenario and difficulties must be the
        environment's. Reward, done and score restart at zero and the outputs are rewritten."""
        values = (ctypes.c_int * (3 + _native.MAXIMUM_AGENTS))(*list(episode)[:3 + _native.MAXIMUM_AGENTS])
        torch.cuda.synchronize(self._torch_device)
        with torch.cuda.device(self._torch_device):
            status = self._library.cuju_environment_set_state(
                self._handle, index, ctypes.c_char_p(match), len(match), values)
        if status != 0:
            # As the reference does: a refusal of the bytes is a StateError, a CUDA failure stays
            # what it is.
            message = self._library.cuju_last_error().decode()
            error = from_library(message)
            raise StateError(message) if type(error) is LibraryError else error

    def set_state(self, index: int, state: bytes) -> None:
        """Sets environment `index` from GRF's state bytes (episode pickle, then engine), as
        `get_state` writes them."""
        size = struct.unpack_from('<i', state)[0]
        episode = unpickle_episode(state[4:4 + size], self.agents)
        self.set_engine_state(index, state[4 + size:], episode)

    def set_stack(self, index: int, frames: bytes) -> None:
        """Writes the simple115 observation stack of environment `index` after `set_state`:
        float32 `[agents][115 * stack]`, the oldest frame first (a stacked batch only)."""
        data = bytes(frames)
        torch.cuda.synchronize(self._torch_device)
        with torch.cuda.device(self._torch_device):
            self._check(self._library.cuju_environment_set_stack(
                self._handle, index, b'simple115', ctypes.c_char_p(data), len(data)))

    def set_lanes_per_environment(self, lanes: int) -> None:
        """How many lanes of a warp run each environment from the next call: 1, 2, 4, 8, 16 or 32,
        or 0 for the library's choice by batch size. This build's extension (no reference
        counterpart); every layout gives the same results."""
        self._check(self._library.cuju_b200_environment_set_lanes(self._handle, int(lanes)))

    def episode(self, index: int) -> list[int]:
        values = (ctypes.c_longlong * 17)()
        self._check(self._library.cuju_environment_episode(self._handle, index, values, None))
        return list(values)

    @property
    def memory_bytes(self) -> int:
        """The device bytes the batch holds, its tables included (a property, as
        python/cuju/_batch/environment.py:885 has it)."""
        return int(self._library.cuju_environment_memory_bytes(self._handle))

    def close(self) -> None:
        """Frees the batch; a second call does nothing, and other calls then raise ClosedError."""
        handle = self.__dict__.get('_native_handle')
        if handle:
            if self.__dict__.get('_operator_key') is not None:
                from . import operators

                operators.unregister(self._operator_key)
            torch.cuda.synchronize(self._torch_device)
            self.__dict__.get('_views', {}).clear()
            self._native_handle = None
            self._library.cuju_environment_destroy(handle)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
