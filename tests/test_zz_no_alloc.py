"""The static-scratch step (`cuju_b200_environment_step_static`, no reference counterpart): one step
with device actions and a fixed device scratch array instead of the batch's own, allocating
nothing. Two identical batches, one stepped through `cuju_environment_step` and one through the
static-scratch entry point, must give identical outputs on each of two consecutive calls. Collected
last (file name) and independent of the other tests' state.
"""

import pytest
import torch

from conftest import needs_data

pytestmark = [pytest.mark.gpu, needs_data]

ASSETS = '5_vs_5_l4_r0'


def _outputs(batch):
    return tuple(t.cpu().numpy().tobytes() for t in batch._outputs())


def test_static_scratch_step_equals_the_step_entry_point_on_two_consecutive_calls():
    from cuju_b200 import BatchEnvironment

    envs = 8
    regular = BatchEnvironment(ASSETS, environment_count=envs, seed=5)
    static = BatchEnvironment(ASSETS, environment_count=envs, seed=5)
    try:
        library = static._library
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
        library = batch._library
        batch.reset()
        actions = torch.zeros((33, batch.agents), dtype=torch.int32, device='cuda')
        with torch.cuda.device(batch._torch_device):
            rc = library.cuju_b200_environment_step_static(batch._handle, actions.data_ptr(), batch._stream())
        assert rc == -1
        assert b'at most 32 environments' in library.cuju_last_error()
    finally:
        batch.close()


@pytest.mark.parametrize('lanes', [None, 1])
def test_static_scratch_step_fills_all_32_slots_through_automatic_restarts(lanes):
    """A batch of exactly 32 environments uses every slot of the static array; a short drill ends
    episodes within the run, so automatic restarts (which sort through the same scratch) happen
    inside static-scratch steps. Every call is compared with the regular step, in the library's
    layout for the size (a warp per environment) and with a lane per environment (the assisted
    branches dealt to crews of one warp)."""
    from cuju_b200 import BatchEnvironment

    envs, assets = 32, 'academy_empty_goal_close_l1_r0'
    regular = BatchEnvironment(assets, environment_count=envs, seed=9, lanes_per_environment=lanes)
    static = BatchEnvironment(assets, environment_count=envs, seed=9, lanes_per_environment=lanes)
    try:
        library = static._library
        regular.reset()
        static.reset()
        generator = torch.Generator(device='cuda').manual_seed(3)
        ended = 0
        for call in range(120):
            actions = torch.randint(0, 19, (envs, regular.agents), generator=generator, device='cuda',
                                    dtype=torch.int32)
            regular.step(actions)
            with torch.cuda.device(static._torch_device):
                rc = library.cuju_b200_environment_step_static(static._handle, actions.data_ptr(), static._stream())
            assert rc == 0, library.cuju_last_error()
            static.synchronize()
            assert _outputs(regular) == _outputs(static), f'outputs differ after call {call + 1}'
            ended += int(static._outputs()[2].sum().item())
        assert ended > 0, 'no episode ended, so no restart went through the static scratch'
        assert static.engine_state(31)[0] == regular.engine_state(31)[0]
    finally:
        regular.close()
        static.close()
