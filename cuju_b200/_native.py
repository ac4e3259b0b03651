"""Loads the B200 batch library and declares its C entry points.

The library is `cuju_b200/lib/libcuju_b200.so`, built in-tree for sm_100a by `cuju_b200.build`
(or `__graft_entry__.build()`). Its entry points and `cuju_configuration` are those of the
reference CUDA backend (cuju src/environment_api.h:35-520; python/cuju/_batch/library.py:150-276
declares the same argument types). There is no fallback: without the library, or without a CUDA
device, loading fails with the reason.
"""

from __future__ import annotations

import ctypes
import os

PACKAGE_DIRECTORY = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(PACKAGE_DIRECTORY, 'lib', 'libcuju_b200.so')
DATA_DIRECTORY = os.path.join(PACKAGE_DIRECTORY, 'data')

CONFIGURATION_VERSION = 2
MAXIMUM_AGENTS = 22


class Configuration(ctypes.Structure):
    """`cuju_configuration` version 2, field for field."""

    _fields_ = [
        ('version', ctypes.c_int),
        ('assets', ctypes.POINTER(ctypes.c_char_p)),
        ('asset_count', ctypes.c_int),
        ('assignment', ctypes.c_void_p),
        ('animations', ctypes.c_char_p),
        ('environment_count', ctypes.c_int),
        ('seed', ctypes.c_ulonglong),
        ('action_set', ctypes.c_int),
        ('observation', ctypes.c_int),
        ('checkpoints', ctypes.c_int),
        ('numpy_legacy', ctypes.c_int),
        ('auto_reset', ctypes.c_int),
        ('threads', ctypes.c_int),
        ('ticks_per_step', ctypes.c_int),
        ('smm_width', ctypes.c_int),
        ('smm_height', ctypes.c_int),
        ('stack', ctypes.c_int),
        ('fixed_seeds', ctypes.c_void_p),
        ('agent_counts', ctypes.c_void_p),
        ('episode_number', ctypes.c_int),
        ('first_index', ctypes.c_ulonglong),
        ('allocate', ctypes.c_void_p),
        ('release', ctypes.c_void_p),
        ('allocator_context', ctypes.c_void_p),
        ('pin_threads', ctypes.c_int),
        ('numa', ctypes.c_int),
        ('page_aligned', ctypes.c_int),
    ]


EXPORTED = (
    'cuju_last_error', 'cuju_backend', 'cuju_environment_create', 'cuju_memory_estimate',
    'cuju_local_memory_bytes', 'cuju_environment_memory_bytes', 'cuju_environment_destroy',
    'cuju_environment_count', 'cuju_environment_threads', 'cuju_environment_agents',
    'cuju_environment_players', 'cuju_environment_set_difficulty', 'cuju_environment_difficulty',
    'cuju_environment_reset', 'cuju_environment_reset_masked', 'cuju_environment_reset_done',
    'cuju_environment_step', 'cuju_environment_step_async', 'cuju_environment_step_wait',
    'cuju_environment_synchronize', 'cuju_environment_get_state', 'cuju_environment_set_state',
    'cuju_environment_set_stack', 'cuju_environment_buffer', 'cuju_environment_raw_field',
    'cuju_environment_episode', 'cuju_environment_scenario', 'cuju_state_layout',
    'cuju_state_gather', 'cuju_state_padding',
)


def declare(library: ctypes.CDLL) -> ctypes.CDLL:
    """Declares the argument and result types of every entry point of `library`."""
    p, i, s = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p
    library.cuju_last_error.restype = s
    library.cuju_backend.restype = s
    library.cuju_environment_create.restype = p
    library.cuju_environment_create.argtypes = [ctypes.POINTER(Configuration)]
    library.cuju_memory_estimate.argtypes = [ctypes.POINTER(Configuration), ctypes.POINTER(ctypes.c_ulonglong)]
    library.cuju_local_memory_bytes.argtypes = [ctypes.POINTER(ctypes.c_ulonglong)]
    library.cuju_environment_memory_bytes.restype = ctypes.c_ulonglong
    library.cuju_environment_memory_bytes.argtypes = [p]
    library.cuju_environment_destroy.argtypes = [p]
    library.cuju_environment_destroy.restype = None
    library.cuju_environment_count.argtypes = [p]
    library.cuju_environment_threads.argtypes = [p]
    library.cuju_environment_agents.argtypes = [p, p, p]
    library.cuju_environment_players.argtypes = [p, p, p]
    library.cuju_environment_set_difficulty.argtypes = [p, p]
    library.cuju_environment_difficulty.argtypes = [p, p]
    library.cuju_environment_difficulty.restype = None
    library.cuju_environment_reset.argtypes = [p, p, p, p]
    library.cuju_environment_reset_masked.argtypes = [p, p, i, p, p, p, i]
    library.cuju_environment_reset_done.argtypes = [p, p]
    # This build's own extension; the reference libraries that the same declarations serve lack it.
    if hasattr(library, 'cuju_b200_environment_reset_masked_device'):
        library.cuju_b200_environment_reset_masked_device.argtypes = [p, p, p, p]
    if hasattr(library, 'cuju_b200_environment_set_lanes'):
        library.cuju_b200_environment_set_lanes.argtypes = [p, i]
        library.cuju_b200_environment_set_lanes.restype = i
    if hasattr(library, 'cuju_b200_environment_step_static'):
        library.cuju_b200_environment_step_static.argtypes = [p, p, p]
        library.cuju_b200_environment_step_static.restype = i
    library.cuju_environment_step.argtypes = [p, p, i, p, i]
    library.cuju_environment_step_async.argtypes = [p, p, i, p]
    library.cuju_environment_step_wait.argtypes = [p]
    library.cuju_environment_synchronize.argtypes = [p, p]
    library.cuju_environment_get_state.restype = p
    library.cuju_environment_get_state.argtypes = [p, i, ctypes.POINTER(ctypes.c_ulonglong), p]
    library.cuju_environment_set_state.argtypes = [p, i, p, ctypes.c_ulonglong, p]
    library.cuju_environment_set_stack.argtypes = [p, i, s, p, ctypes.c_ulonglong]
    library.cuju_environment_raw_field.restype = s
    library.cuju_environment_raw_field.argtypes = [p, i, p, p, p]
    library.cuju_environment_buffer.restype = p
    library.cuju_environment_buffer.argtypes = [p, s]
    library.cuju_environment_episode.argtypes = [p, i, p, p]
    library.cuju_environment_scenario.restype = s
    library.cuju_environment_scenario.argtypes = [p, i]
    return library


_LOADED = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Returns the declared library at `path` (default: the in-tree build), failing loudly."""
    global _LOADED
    if path is None and _LOADED is not None:
        return _LOADED
    target = path or LIBRARY_PATH
    if not os.path.isfile(target):
        raise RuntimeError(
            f'the cuju-b200 CUDA library is missing at {target}; build it with '
            '`python -c "import cuju_b200.build as b; b.build()"`'
        )
    library = declare(ctypes.CDLL(target))
    backend = library.cuju_backend().decode()
    if backend != 'cuda':
        raise RuntimeError(f'expected the CUDA backend in {target}, found {backend!r}')
    if path is None:
        _LOADED = library
    return library
