"""The static-scratch step (`cuju_b200_environment_step_static`, no reference counterpart): one step
with device actions and a fixed device scratch array instead of the batch's own, allocating
nothing. Two identical batches, one stepped through `cuju_environment_step` and one through the
static-scratch entry point, must give identical outputs on each of two consecutive calls. Collected
last (file name) and independent of the other tests' state.
"""

import ctypes

import pytest
import torch

from conftest import needs_data

pytestmark = [pytest.mark.gpu, needs_data]

ASSETS = '5_vs_5_l4_r0'


def _declare(library):
    library.cuju_b200_environment_step_static.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    library.cuju_b200_environment_step_static.restype = ctypes.c_int
    return library


def _outputs(batch):
    return tuple(t.cpu().numpy().tobytes() for t in batch._outputs())


def test_static_scratch_step_equals_the_step_entry_point_on_two_consecutive_calls():
    from cuju_b200 import BatchEnvironment

    envs = 8
    regular = BatchEnvironment(ASSETS, environment_count=envs, seed=5)
    static = BatchEnvironment(ASSETS, environment_count=envs, seed=5)
    try:
        library = _declare(static._library)
        regular.reset()
        static.reset()
        assert _outputs(regular) == _outputs(static)
        generator = torch.Generator(device='cuda').manual_seed(11)
        for call in range(2):
            actions = torch.randint(0, 19, (envs, regular.agents), generator=generator, device='cuda',
                                    dtype=torch.int32)
            regular.step(actions)
            with torch.cuda.device(static._torch_device):
                rc = library.cuju_b200_environment_step_static(static._handle, actions.data_ptr(), static._stream())
            assert rc == 0, library.cuju_last_error()
            static.synchronize()
            assert _outputs(regular) == _outputs(static), f'outputs differ after call {call + 1}'
        host = torch.zeros((envs, static.agents), dtype=torch.int32)
        with torch.cuda.device(static._torch_device):
            rc = library.cuju_b200_environment_step_static(static._handle, host.data_ptr(), static._stream())
        assert rc == -1
        assert b'device memory' in library.cuju_last_error()
    finally:
        regular.close()
        static.close()


def test_static_scratch_step_refuses_a_batch_larger_than_its_scratch():
    from cuju_b200 import BatchEnvironment

    batch = BatchEnvironment(ASSETS, environment_count=33, seed=1)
    try:
        library = _declare(batch._library)
        batch.reset()
        actions = torch.zeros((33, batch.agents), dtype=torch.int32, device='cuda')
        with torch.cuda.device(batch._torch_device):
            rc = library.cuju_b200_environment_step_static(batch._handle, actions.data_ptr(), batch._stream())
        assert rc == -1
        assert b'at most 32 environments' in library.cuju_last_error()
    finally:
        batch.close()
