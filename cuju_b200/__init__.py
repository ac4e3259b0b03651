"""cuju-b200: Google Research Football's batched environment step on NVIDIA B200 (sm_100a).

A drop-in for the reference's CUDA backend: the C-ABI library `lib/libcuju_b200.so` exports the
reference's `cuju_*` entry points, and `BatchEnvironment` mirrors the reference Python class.
"""

from . import errors
from .environment import BatchEnvironment, bundled_assets, resolve_asset
from .errors import ActionRangeError, LibraryError
from .multi_device import EpisodeTotals, MultiDeviceBatch

__all__ = ['ActionRangeError', 'BatchEnvironment', 'EpisodeTotals', 'LibraryError', 'MultiDeviceBatch',
           'bundled_assets', 'errors', 'resolve_asset']
