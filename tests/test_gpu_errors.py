"""A path GRF leaves undefined, on the device. The reference traps there; this build ends the
environment's step and records it in a status word instead, and the host raises the reference's
UndefinedPathError at the next synchronising call. The state loaded here has a match generator
with an empty range (minimum equal to maximum, which no valid state holds), so Boost's
uniform-float redraw loop runs to its iteration cap on the next draw instead of forever. The other
environment of the batch keeps stepping. tests/test_host_api.py checks the same path on the host
build."""

import struct

import pytest
import torch

from conftest import needs_data

pytestmark = [pytest.mark.gpu, needs_data]


@pytest.mark.parametrize('lanes', [1, 32])
def test_a_capped_loop_raises_undefined_path_error(lanes):
    from cuju_b200 import BatchEnvironment
    from cuju_b200.errors import UndefinedPathError

    batch = BatchEnvironment('5_vs_5_l4_r0', environment_count=2, seed=7, lanes_per_environment=lanes)
    try:
        batch.reset()
        idle = torch.zeros((2, batch.agents), dtype=torch.int32, device='cuda')
        for _ in range(3):
            batch.step(idle)
        engine, episode = batch.engine_state(0)
        healthy = batch.engine_state(1)[0]
        # The match generator's bytes start at byte 8 of the engine state: 624 words, a 64-bit
        # index, then the range's minimum and maximum floats (0 and 1 in every valid state).
        at = 8 + 624 * 4 + 8
        assert struct.unpack_from('<ff', engine, at) == (0.0, 1.0)
        batch.set_engine_state(0, engine[:at] + struct.pack('<ff', 1.0, 1.0) + engine[at + 8:], episode)
        with pytest.raises(UndefinedPathError):
            for _ in range(20):
                batch.step(idle)
        assert batch.engine_state(1)[0] != healthy, 'the healthy environment stopped stepping'
    finally:
        batch.close()
