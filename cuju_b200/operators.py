"""The `torch.library` operators through which `torch.compile` traces a batch's step without a graph
break, as the reference's python/cuju/_batch/operators.py:20-55 registers `cuju::step` and
`cuju::reset_done`. Here they are `cuju_b200::step` and `cuju_b200::reset_done` (their own namespace,
so this package and the reference's can share a process). Each takes the integer key of a
registered batch and the list of the batch's output tensors, which it declares mutated; it runs the
same library call as the eager method, on the current stream, without synchronising, and copies the
batch's outputs into any given tensor that is not the batch's own (compiled code may hand over a
functional copy).
"""

from __future__ import annotations

import itertools
import weakref

import torch

_BATCHES: dict[int, weakref.ref] = {}
_KEYS = itertools.count(1)


def register(batch) -> int:
    """Registers a batch with the operators and returns its key."""
    key = next(_KEYS)
    _BATCHES[key] = weakref.ref(batch)
    return key


def unregister(key: int) -> None:
    _BATCHES.pop(key, None)


def _batch(key: int):
    ref = _BATCHES.get(key)
    batch = ref() if ref is not None else None
    if batch is None:
        raise RuntimeError(f'no open batch is registered under key {key}')
    return batch


def _copy_outputs(batch, outputs: list[torch.Tensor]) -> None:
    for given, own in zip(outputs, batch._operator_tensors(), strict=True):
        if given.data_ptr() != own.data_ptr():
            given.copy_(own)


@torch.library.custom_op('cuju_b200::step', mutates_args=('outputs',))
def step(batch: int, actions: torch.Tensor, outputs: list[torch.Tensor]) -> None:
    b = _batch(batch)
    b._device_step(actions)
    _copy_outputs(b, outputs)


@step.register_fake
def _step_fake(batch, actions, outputs):
    return None


@torch.library.custom_op('cuju_b200::reset_done', mutates_args=('outputs',))
def reset_done(batch: int, outputs: list[torch.Tensor]) -> None:
    b = _batch(batch)
    b._device_reset_done()
    _copy_outputs(b, outputs)


@reset_done.register_fake
def _reset_done_fake(batch, outputs):
    return None
