"""The exceptions of the batch API, under the reference's names and bases.

Code written against the reference package catches these by name (python/cuju/errors.py:29-92), so
each class keeps the reference's name and the built-in exceptions it derives from: an
`except ValueError:` clause catches a `ConfigurationError`, `ChoiceError` is also a `KeyError`, and
`EnvironmentIndexError` is both an `IndexError` and a `RuntimeError`.
"""

from __future__ import annotations

__all__ = [
    'ActionRangeError', 'ArgumentError', 'ChoiceError', 'ClosedError', 'ConfigurationError', 'DeviceError',
    'EnvironmentIndexError', 'Error', 'LibraryError', 'MissingFileError', 'StateError', 'UndefinedPathError',
    'from_library',
]


class Error(Exception):
    """The base of every failure the batch API raises."""

    # KeyError would quote the message; every class prints it as it is.
    __str__ = Exception.__str__


class ConfigurationError(Error, ValueError):
    """A batch option that is refused."""


class ChoiceError(ConfigurationError, KeyError):
    """A name outside the valid ones: a representation, an action set, a device."""


class ArgumentError(Error, ValueError):
    """A call argument that is refused, such as seeds out of range."""


class ActionRangeError(Error, IndexError):
    """A host action index outside the action set (the library's -2)."""


class EnvironmentIndexError(Error, IndexError, RuntimeError):
    """An environment index outside the batch."""


class StateError(Error, ValueError, RuntimeError):
    """State bytes that do not load into an environment."""


class ClosedError(Error, RuntimeError):
    """A call on a batch after `close`."""


class DeviceError(Error, RuntimeError):
    """A device that cannot run the batch, or a failed CUDA call."""


class UndefinedPathError(Error, RuntimeError):
    """An environment that reached a path GRF leaves undefined."""


class LibraryError(Error, RuntimeError):
    """Any other failure the library reports."""


class MissingFileError(Error, FileNotFoundError):
    """An asset bundle, animation file or library that does not exist."""


def from_library(message: str) -> Error:
    """The exception for a failure message of the library: its CUDA failures start with
    `cuda` (`cuda error in ...`, as the reference's start with the CUDA call's name), and a
    device-side stop on an undefined GRF path says so."""
    if 'reached a path that GRF leaves undefined' in message:
        return UndefinedPathError(message)
    if message.startswith('cuda'):
        return DeviceError(message)
    if message.startswith('expected an environment from'):
        return EnvironmentIndexError(message)
    return LibraryError(message)
