"""Test infrastructure: a minimal ctypes driver of the reference CPU backend.

`oracle/_ref/libcuju_cpu.so` is the reference's own CPU implementation of the batched step,
compiled from the reference sources by `oracle/Makefile` (cuju src/cuju_cpu.cpp with
include/cuju/batch/*). It exports the same `cuju_*` C-ABI as the B200 library, with host buffers.
Only the parity tests, `__graft_entry__.smoke()` and the CPU legs of `bench.py` use it, as the
checker and the timed reference; the product never loads it.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, '_ref', 'libcuju_cpu.so')


def _configuration_type():
    # The same version-2 configuration struct as the B200 library (cuju src/environment_api.h:49).
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        '_cb_native', os.path.join(os.path.dirname(HERE), 'cuju_b200', '_native.py'))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


class OracleBatch:
    """The reference CPU batch: reset, step and state bytes, outputs as host byte strings."""

    def __init__(self, bundle_paths, agent_counts, environment_count, seed, animations, threads=1,
                 representation=2, checkpoints=False, stack=1, assignment=None, difficulty=None,
                 auto_reset=True, ticks_per_step=10, first_index=0, library=None, fixed_seeds=None,
                 episode_number=0, action_set=0, numpy_legacy=True, smm_size=(96, 72)):
        path = library or LIBRARY
        if not os.path.isfile(path):
            raise RuntimeError(f'the oracle library is missing at {path}; run make -C oracle')
        native = _configuration_type()
        self.lib = native.declare(ctypes.CDLL(path))
        if self.lib.cuju_backend().decode() != 'cpu':
            raise RuntimeError('expected the reference CPU backend')
        self._paths = [p.encode() for p in bundle_paths]
        paths = (ctypes.c_char_p * len(self._paths))(*self._paths)
        counts = (ctypes.c_int * (2 * len(self._paths)))(*[c for pair in agent_counts for c in pair])
        assign = None if assignment is None else (ctypes.c_int * environment_count)(*assignment)
        self._fixed = None if fixed_seeds is None else (ctypes.c_longlong * environment_count)(*fixed_seeds)
        config = native.Configuration(
            version=2, assets=paths, asset_count=len(self._paths),
            assignment=ctypes.cast(assign, ctypes.c_void_p) if assign else None,
            animations=animations.encode(), environment_count=environment_count, seed=seed,
            action_set=action_set, observation=representation, checkpoints=int(checkpoints),
            numpy_legacy=int(numpy_legacy),
            auto_reset=int(auto_reset), threads=threads, ticks_per_step=ticks_per_step, smm_width=smm_size[0], smm_height=smm_size[1],
            stack=stack, fixed_seeds=ctypes.cast(self._fixed, ctypes.c_void_p) if self._fixed else None,
            agent_counts=ctypes.cast(counts, ctypes.c_void_p), episode_number=episode_number, first_index=first_index, allocate=None, release=None, allocator_context=None,
            pin_threads=0, numa=0, page_aligned=0)
        self.handle = self.lib.cuju_environment_create(ctypes.byref(config))
        if not self.handle:
            raise RuntimeError(self.lib.cuju_last_error().decode())
        self.count = environment_count
        self.agents = self.lib.cuju_environment_agents(self.handle, None, None)
        self.checkpoints = checkpoints
        self.width = 115 * stack
        self.representation = representation
        self.smm_size = tuple(smm_size)
        if difficulty is not None:
            values = (ctypes.c_float * (2 * environment_count))(*difficulty)
            if self.lib.cuju_environment_set_difficulty(self.handle, values) != 0:
                raise RuntimeError(self.lib.cuju_last_error().decode())

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(self.lib.cuju_last_error().decode())

    def _buffer(self, name, nbytes):
        return ctypes.string_at(self.lib.cuju_environment_buffer(self.handle, name.encode()), nbytes)

    def _raw_bytes(self, name):
        # Every raw array's bytes, the arrays in name order (as the reference's digest reads them).
        self.lib.cuju_environment_raw_field.restype = ctypes.c_char_p
        self.lib.cuju_environment_raw_field.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                                        ctypes.c_void_p, ctypes.c_void_p]
        base = self.lib.cuju_environment_buffer(self.handle, name.encode())
        kind, dims, offset = ctypes.c_int(), (ctypes.c_int * 2)(), ctypes.c_ulonglong()
        arrays = {}
        for field in range(64):
            field_name = self.lib.cuju_environment_raw_field(self.handle, field, ctypes.byref(kind), dims,
                                                             ctypes.byref(offset))
            if not field_name:
                break
            elements = (dims[0] or 1) * (dims[1] or 1)
            size = 4 if kind.value in (0, 1) else 1
            arrays[field_name.decode()] = ctypes.string_at(base + offset.value, self.count * self.agents * elements * size)
        return b''.join(arrays[k] for k in sorted(arrays))

    def outputs(self):
        e, a = self.count, self.agents
        if self.representation == 8:
            obs = self._raw_bytes('raw')
        elif self.representation == 4:
            obs = self._buffer('smm', e * a * self.smm_size[0] * self.smm_size[1] * 4 * (self.width // 115))
        else:
            obs = self._buffer('simple115', 4 * e * a * self.width)
        return (obs, self._buffer('reward', 4 * e * a), self._buffer('done', e), self._buffer('score_reward', 4 * e))

    def reset(self, seeds=None, reverse=None):
        arr = None if seeds is None else (ctypes.c_uint * self.count)(*seeds)
        rev = None if reverse is None else (ctypes.c_int * self.count)(*reverse)
        self._check(self.lib.cuju_environment_reset(self.handle, arr, rev, None))
        return self.outputs()

    def reset_done(self):
        self._check(self.lib.cuju_environment_reset_done(self.handle, None))
        return self.outputs()

    def step_status(self, actions):
        # The step's return code (0, -1, or -2 for a host action out of range) and its message.
        arr = (ctypes.c_int * (self.count * self.agents))(*actions)
        rc = self.lib.cuju_environment_step(self.handle, arr, 0, None, 1)
        return rc, (self.lib.cuju_last_error() or b'').decode() if rc else ''

    def reset_masked(self, mask, seeds=None):
        m = (ctypes.c_ubyte * self.count)(*mask)
        s = None if seeds is None else (ctypes.c_longlong * self.count)(*seeds)
        self._check(self.lib.cuju_environment_reset_masked(self.handle, m, 0, s, None, None, 1))
        return self.outputs()

    def step(self, actions):
        arr = (ctypes.c_int * (self.count * self.agents))(*actions)
        self._check(self.lib.cuju_environment_step(self.handle, arr, 0, None, 1))
        return self.outputs()

    def engine_state(self, index):
        episode = (ctypes.c_int * 25)()
        size = ctypes.c_ulonglong()
        p = self.lib.cuju_environment_get_state(self.handle, index, ctypes.byref(size), episode)
        if not p:
            raise RuntimeError(self.lib.cuju_last_error().decode())
        return ctypes.string_at(p, size.value), list(episode)

    def set_state(self, index, data, episode):
        values = (ctypes.c_int * 25)(*list(episode)[:25])
        self.lib.cuju_environment_set_state.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p,
                                                        ctypes.c_ulonglong, ctypes.c_void_p]
        self._check(self.lib.cuju_environment_set_state(self.handle, index, data, len(data), values))
        return self.outputs()

    def close(self):
        if self.handle:
            self.lib.cuju_environment_destroy(self.handle)
            self.handle = None
