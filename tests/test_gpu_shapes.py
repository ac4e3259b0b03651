"""Output shapes on a B200 (reference tests/test_shapes.py, test_squeeze): with `squeeze` a batch
of one agent drops the agent axis of its observation and reward, and its values are those of the
same batch without it."""

import pytest
import torch

from conftest import needs_data

pytestmark = [pytest.mark.gpu, needs_data]


def test_squeeze_drops_the_agent_axis_of_one_agent():
    from cuju_b200 import BatchEnvironment

    plain = BatchEnvironment('academy_empty_goal_close_l1_r0', environment_count=4, seed=3)
    squeezed = BatchEnvironment('academy_empty_goal_close_l1_r0', environment_count=4, seed=3, squeeze=True)
    try:
        first, second = plain.reset(), squeezed.reset()
        assert first.shape == (4, 1, 115) and second.shape == (4, 115)
        assert torch.equal(second, first[:, 0])
        for step in range(5):
            actions = torch.tensor([1, 5, 9, 13], dtype=torch.int32) + step
            a = plain.step(actions.reshape(4, 1).cuda())
            b = squeezed.step(actions.cuda())
            assert b[0].shape == (4, 115) and b[1].shape == (4,) and b[2].shape == (4,)
            assert torch.equal(b[0], a[0][:, 0]) and torch.equal(b[1], a[1][:, 0]) and torch.equal(b[2], a[2])
    finally:
        plain.close()
        squeezed.close()


def test_calls_after_close_raise_closed_error():
    """A closed batch raises ClosedError (a RuntimeError) instead of handing the library a null
    batch; a second close does nothing (reference tests/test_errors.py)."""
    from cuju_b200 import BatchEnvironment
    from cuju_b200.errors import ClosedError

    batch = BatchEnvironment('academy_empty_goal_close_l1_r0', environment_count=2, seed=1)
    batch.reset()
    batch.close()
    batch.close()
    with pytest.raises(ClosedError):
        batch.step(torch.zeros((2, 1), dtype=torch.int32))
    with pytest.raises(ClosedError):
        batch.get_state(0)
    with pytest.raises(ClosedError):
        batch.reset()


def test_minimap_of_another_size_against_the_oracle():
    """`channel_dimensions` = (48, 36): the SMM observation is [environments, agents, 36, 48, 4]
    and equals the reference CPU backend's, byte for byte, over a reset and 20 steps."""
    from conftest import ANIMATIONS, resolve

    from cuju_b200 import BatchEnvironment
    from oracle.driver import OracleBatch

    paths, counts = resolve('5_vs_5_l4_r0')
    mine = BatchEnvironment('5_vs_5_l4_r0', environment_count=3, seed=17, representation='extracted',
                            channel_dimensions=(48, 36))
    ref = OracleBatch(paths, counts, 3, 17, ANIMATIONS, threads=1, representation=4, smm_size=(48, 36))
    try:
        obs = mine.reset()
        assert obs.shape == (3, 4, 36, 48, 4)
        assert obs.cpu().numpy().tobytes() == ref.reset()[0]
        for step in range(20):
            actions = [[(step * 5 + e * 3 + a * 7) % 19 for a in range(4)] for e in range(3)]
            got = mine.step(torch.tensor(actions, dtype=torch.int32).cuda())
            want = ref.step([x for row in actions for x in row])
            assert got[0].cpu().numpy().tobytes() == want[0], f'observation differs at step {step}'
            assert got[1].cpu().numpy().tobytes() == want[1], f'reward differs at step {step}'
    finally:
        mine.close()
        ref.close()
