"""`torch.compile` over a batch's step and reset_done (cuju tests/test_compile.py): the compiled
function traces the calls through the operators `cuju_b200::step` and `cuju_b200::reset_done`
(cuju_b200/operators.py) without a graph break, and its outputs equal eager steps of an identical
batch bit for bit."""

import pytest
import torch

from conftest import needs_data

pytestmark = [pytest.mark.gpu, needs_data]


def _bytes(t):
    return t.detach().cpu().contiguous().numpy().tobytes()


def test_compiled_steps_equal_eager_steps():
    from cuju_b200 import BatchEnvironment

    eager = BatchEnvironment('5_vs_5_l4_r0', environment_count=8, seed=2)
    compiled = BatchEnvironment('5_vs_5_l4_r0', environment_count=8, seed=2)
    try:
        eager.reset()
        compiled.reset()

        @torch.compile(fullgraph=True)
        def play(batch, actions):
            observation, reward, done, info = batch.step(actions)
            return observation * 1.0, reward + 0.0, done.clone(), info['score_reward'] + 0

        generator = torch.Generator(device='cuda').manual_seed(8)
        for step in range(6):
            actions = torch.randint(0, 19, (8, 4), generator=generator, device='cuda', dtype=torch.int32)
            o, r, d, _ = eager.step(actions)
            co, cr, cd, cs = play(compiled, actions)
            assert _bytes(co) == _bytes(o), f'observation differs at step {step}'
            assert _bytes(cr) == _bytes(r), f'reward differs at step {step}'
            assert _bytes(cd) == _bytes(d), f'done differs at step {step}'
        assert eager.engine_state(3)[0] == compiled.engine_state(3)[0]
    finally:
        eager.close()
        compiled.close()


def test_compiled_reset_done_equals_eager():
    from cuju_b200 import BatchEnvironment

    options = dict(environment_count=8, seed=4, auto_reset=False)
    eager = BatchEnvironment('academy_empty_goal_close_l1_r0', **options)
    compiled = BatchEnvironment('academy_empty_goal_close_l1_r0', **options)
    try:
        eager.reset()
        compiled.reset()

        @torch.compile(fullgraph=True)
        def restart(batch):
            batch.reset_done()
            return batch.observation() * 1.0

        generator = torch.Generator(device='cuda').manual_seed(1)
        for step in range(40):
            actions = torch.randint(0, 19, (8, 1), generator=generator, device='cuda', dtype=torch.int32)
            eager.step(actions)
            compiled.step(actions)
            if step % 10 == 9:
                eager.reset_done()
                assert _bytes(restart(compiled)) == _bytes(eager.observation()), f'reset_done differs at {step}'
    finally:
        eager.close()
        compiled.close()
