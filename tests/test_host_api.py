"""The C-ABI's batch options on the host build (tests/host/hostsim.cu) against the reference CPU
backend: fixed seeds with GRF's episode number over many automatic restarts, team order given
at reset, masked resets with given and drawn seeds, first_index, host actions out of range (-2)
or negative (counted from the end), the v2 and full action sets, checkpoint rewards without the
NumPy-legacy rounding, other tick counts per step, episodes without automatic restart, the
device-resident masked reset, and the shapes of the bench's other configurations (all 11 players
controlled with masked resets; mixed bundles, stacked). Every output buffer is compared after every
call, and the state bytes at the end. These are the host-side paths of api.cu and env.cuh that the device
kernels share; the GPU tests cover the device build on shorter runs.
"""

import random

import pytest

from conftest import ANIMATIONS, needs_data, resolve

pytestmark = [needs_data]


def _pair(host_library, assets, envs, seed, **options):
    from oracle.driver import OracleBatch

    paths, counts = resolve(assets)
    return [OracleBatch(paths, counts, envs, seed, ANIMATIONS, threads=1, library=library, **options)
            for library in (None, host_library)]


def _run(batches, steps, rng, masked=False, agents_actions=19):
    ref, mine = batches
    envs = ref.count
    for step in range(steps):
        acts = [rng.randrange(agents_actions) for _ in range(envs * ref.agents)]
        assert mine.step(acts) == ref.step(acts), f'step {step} differs'
        if masked and rng.random() < 0.3:
            mask = [1 if rng.random() < 0.3 else 0 for _ in range(envs)]
            seeds = [rng.randrange(0, 2**32) if rng.random() < 0.5 else -1 for _ in range(envs)]
            assert mine.reset_masked(mask, seeds) == ref.reset_masked(mask, seeds), f'masked reset {step} differs'
    for index in range(envs):
        assert mine.engine_state(index) == ref.engine_state(index), f'state {index} differs'


def test_fixed_seeds_and_episode_number_over_many_episodes(host_library):
    batches = _pair(host_library, 'academy_empty_goal_close_l1_r0', 6, 3, fixed_seeds=[5, -1, 7, -1, 11, 11],
                    episode_number=3, checkpoints=True)
    try:
        assert batches[1].reset() == batches[0].reset()
        _run(batches, 300, random.Random(1))
    finally:
        for b in batches:
            b.close()


def test_reverse_at_reset_and_first_index(host_library):
    batches = _pair(host_library, '5_vs_5_l4_r0', 4, 9, first_index=1000)
    try:
        reverse = [1, 0, 1, 0]
        assert batches[1].reset([4, 4, 8, 8], reverse) == batches[0].reset([4, 4, 8, 8], reverse)
        _run(batches, 40, random.Random(2))
    finally:
        for b in batches:
            b.close()


def test_masked_resets_with_given_and_drawn_seeds(host_library):
    batches = _pair(host_library, '11_vs_11_easy_stochastic_l1_r0', 6, 4, difficulty=[0.3, -1.0] * 6)
    try:
        assert batches[1].reset() == batches[0].reset()
        _run(batches, 40, random.Random(3), masked=True)
    finally:
        for b in batches:
            b.close()


def test_host_actions_out_of_range_and_negative(host_library):
    batches = _pair(host_library, '5_vs_5_l4_r0', 2, 1)
    ref, mine = batches
    try:
        assert mine.reset() == ref.reset()
        n = ref.agents * 2
        for acts in ([-1] * n, [-19] * n, [18] * n):
            assert mine.step(acts) == ref.step(acts)
        for acts in ([19] * n, [-20] * n):
            r, m = ref.step_status(acts), mine.step_status(acts)
            assert r[0] == m[0] == -2, (r, m)
    finally:
        for b in batches:
            b.close()


@pytest.mark.parametrize('action_set,actions', [(1, 20), (2, 33)])
def test_other_action_sets(host_library, action_set, actions):
    batches = _pair(host_library, '5_vs_5_l4_r0', 3, 6, action_set=action_set)
    try:
        assert batches[1].reset() == batches[0].reset()
        _run(batches, 60, random.Random(4), agents_actions=actions)
    finally:
        for b in batches:
            b.close()


def test_checkpoint_rewards_without_the_numpy_legacy_rounding(host_library):
    batches = _pair(host_library, 'academy_counterattack_easy_l1_r0', 4, 8, checkpoints=True, numpy_legacy=False)
    try:
        assert batches[1].reset() == batches[0].reset()
        _run(batches, 200, random.Random(5))
    finally:
        for b in batches:
            b.close()


@pytest.mark.parametrize('ticks', [1, 4])
def test_other_ticks_per_step(host_library, ticks):
    batches = _pair(host_library, '11_vs_11_stochastic_l1_r0', 2, 2, ticks_per_step=ticks)
    try:
        assert batches[1].reset() == batches[0].reset()
        _run(batches, 40, random.Random(6))
    finally:
        for b in batches:
            b.close()


def test_episodes_without_automatic_restart(host_library):
    """auto_reset off: an ended environment keeps its outputs (reward and score zeroed while done)
    until reset_done starts its next episode."""
    batches = _pair(host_library, 'academy_empty_goal_close_l1_r0', 4, 12, auto_reset=False)
    ref, mine = batches
    rng = random.Random(7)
    try:
        assert mine.reset() == ref.reset()
        restarts = 0
        for step in range(250):
            acts = [rng.randrange(19) for _ in range(4 * ref.agents)]
            out = ref.step(acts)
            assert mine.step(acts) == out, f'step {step} differs'
            if any(out[2]) and rng.random() < 0.5:
                assert mine.reset_done() == ref.reset_done(), f'reset_done at {step} differs'
                restarts += 1
        assert restarts > 0
        for index in range(4):
            assert mine.engine_state(index) == ref.engine_state(index)
    finally:
        for b in batches:
            b.close()


def test_masked_reset_with_device_seeds(host_library):
    """`cuju_b200_environment_reset_masked_device` (mask and seeds in device memory, no host check)
    on the host build, where device memory is host memory, against the reference's host-seed masked
    reset: the first call without a mask starts every environment, negative seeds draw as -1 does,
    and a seed of 2^32 or more plays as its low 32 bits. A mask before every environment has
    started is refused."""
    import ctypes

    batches = _pair(host_library, '5_vs_5_l4_r0', 6, 21)
    ref, mine = batches
    mine.lib.cuju_b200_environment_reset_masked_device.argtypes = [ctypes.c_void_p] * 4
    device_reset = mine.lib.cuju_b200_environment_reset_masked_device
    rng = random.Random(11)
    try:
        ones = (ctypes.c_ubyte * 6)(*[1] * 6)
        assert device_reset(mine.handle, ones, None, None) == -1
        assert b'started' in mine.lib.cuju_last_error()
        first = [3, -1, 2**32 + 5, -7, 9, 0]
        given = (ctypes.c_longlong * 6)(*first)
        expected = [s & 0xffffffff if s >= 0 else -1 for s in first]
        ref._check(ref.lib.cuju_environment_reset_masked(
            ref.handle, None, 0, (ctypes.c_longlong * 6)(*expected), None, None, 1))
        assert device_reset(mine.handle, None, given, None) == 0
        assert mine.outputs() == ref.outputs()
        for step in range(60):
            acts = [rng.randrange(19) for _ in range(6 * ref.agents)]
            assert mine.step(acts) == ref.step(acts), f'step {step} differs'
            if step % 7 == 3:
                mask = [1 if rng.random() < 0.4 else 0 for _ in range(6)]
                seeds = [rng.choice((-1, -5, rng.randrange(2**32), 2**32 + rng.randrange(2**32))) for _ in range(6)]
                wanted = ref.reset_masked(mask, [s & 0xffffffff if s >= 0 else -1 for s in seeds])
                rc = device_reset(mine.handle, (ctypes.c_ubyte * 6)(*mask), (ctypes.c_longlong * 6)(*seeds), None)
                assert rc == 0 and mine.outputs() == wanted, f'device masked reset at {step} differs'
        for index in range(6):
            assert mine.engine_state(index) == ref.engine_state(index)
    finally:
        for b in batches:
            b.close()


def test_drawn_seeds_with_first_index_over_restarts(host_library):
    """A part of a larger batch (first_index 20): seeds drawn at reset and at every automatic
    restart follow the seed rule of environments 20 onwards, as in the reference."""
    batches = _pair(host_library, 'academy_empty_goal_close_l1_r0', 12, 5, first_index=20)
    try:
        assert batches[1].reset() == batches[0].reset()
        _run(batches, 120, random.Random(13))
    finally:
        for b in batches:
            b.close()


def test_every_left_player_controlled_at_high_difficulty_with_masked_resets(host_library):
    """The shape of the bench's 65,536-environment configuration at a testable size: 11v11 with all
    11 left players controlled (`11_vs_11_hard_stochastic_l11_r0`, right team at 0.95), and a masked
    reset with fresh seeds after most steps."""
    batches = _pair(host_library, '11_vs_11_hard_stochastic_l11_r0', 4, 0, first_index=4096)
    ref, mine = batches
    rng = random.Random(17)
    try:
        assert ref.agents == 11
        assert mine.reset() == ref.reset()
        for step in range(40):
            acts = [rng.randrange(19) for _ in range(4 * 11)]
            assert mine.step(acts) == ref.step(acts), f'step {step} differs'
            mask = [1 if rng.random() < 0.15 else 0 for _ in range(4)]
            seeds = [rng.randrange(0, 2**32) for _ in range(4)]
            assert mine.reset_masked(mask, seeds) == ref.reset_masked(mask, seeds), f'masked reset {step} differs'
        for index in range(4):
            assert mine.engine_state(index) == ref.engine_state(index)
    finally:
        for b in batches:
            b.close()


def test_mixed_bundles_interleaved_and_stacked(host_library):
    """The shape of the bench's mixed configuration at a testable size: three bundles (11v11 with
    one agent, 5v5 with four, a drill with one) interleaved by index with the assignment
    [0, 1, 0, 1, 2], four-frame stacked observations, and automatic restarts."""
    assets = ['11_vs_11_stochastic_l1_r0', '5_vs_5_l4_r0', 'academy_empty_goal_close_l1_r0']
    assignment = [[0, 1, 0, 1, 2][i % 5] for i in range(10)]
    batches = _pair(host_library, assets, 10, 3, assignment=assignment, stack=4)
    ref, mine = batches
    rng = random.Random(19)
    try:
        assert ref.agents == 4
        assert mine.reset() == ref.reset()
        for step in range(80):
            acts = [rng.randrange(19) for _ in range(10 * 4)]
            assert mine.step(acts) == ref.step(acts), f'step {step} differs'
    finally:
        for b in batches:
            b.close()


def test_device_actions_outside_the_set_step_as_idle(host_library):
    """Actions flagged as device-resident go unchecked: an index outside [-n, n) acts as idle
    (action 0) and a negative one in range counts from the end, as batch_core.h:617-621 decodes
    them. On the host build the device buffer is host memory, so the kernel path reads them."""
    import ctypes

    batches = _pair(host_library, '5_vs_5_l4_r0', 3, 6)
    ref, mine = batches
    try:
        assert mine.reset() == ref.reset()
        n = 3 * ref.agents
        for bad, same in (([19, 1000, -20, -2**31] * 3, [0] * n), ([-1, -19, 5, -7] * 3, [18, 0, 5, 12] * 3)):
            arr = (ctypes.c_int * n)(*bad)
            assert mine.lib.cuju_environment_step(mine.handle, arr, 1, None, 1) == 0
            assert mine.outputs() == ref.step(same)
        for index in range(3):
            assert mine.engine_state(index) == ref.engine_state(index)
    finally:
        for b in batches:
            b.close()


def test_state_bytes_that_stop_short_or_run_on_are_refused(host_library):
    """set_state refuses engine bytes cut short or followed by more, as the reference does
    (tests/test_state_errors.py), and leaves the environment as it was."""
    import ctypes

    batches = _pair(host_library, '5_vs_5_l4_r0', 2, 2)
    ref, mine = batches
    try:
        assert mine.reset() == ref.reset()
        for b in batches:
            b.lib.cuju_environment_set_state.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p,
                                                         ctypes.c_ulonglong, ctypes.c_void_p]
        acts = [3] * (2 * ref.agents)
        assert mine.step(acts) == ref.step(acts)
        data, episode = ref.engine_state(1)
        values = (ctypes.c_int * 25)(*episode[:25])
        for wrong in (data[:-10], data[:len(data) // 2], data + b'\0\0\0'):
            codes = [b.lib.cuju_environment_set_state(b.handle, 0, wrong, len(wrong), values) for b in batches]
            assert codes == [-1, -1], f'{len(wrong)} of {len(data)} bytes: {codes}'
        assert mine.engine_state(0) == ref.engine_state(0)
        assert mine.step(acts) == ref.step(acts)
    finally:
        for b in batches:
            b.close()


def test_an_async_step_equals_a_step(host_library):
    """cuju_environment_step_async followed by cuju_environment_step_wait gives what a step gives,
    and checks host actions the same way (-2 before anything runs)."""
    import ctypes

    batches = _pair(host_library, '5_vs_5_l4_r0', 2, 12)
    ref, mine = batches
    rng = random.Random(23)
    try:
        assert mine.reset() == ref.reset()
        n = 2 * ref.agents
        for step in range(20):
            acts = [rng.randrange(19) for _ in range(n)]
            arr = (ctypes.c_int * n)(*acts)
            assert mine.lib.cuju_environment_step_async(mine.handle, arr, 0, None) == 0
            assert mine.lib.cuju_environment_step_wait(mine.handle) == 0
            assert mine.outputs() == ref.step(acts), f'async step {step} differs'
        arr = (ctypes.c_int * n)(*([19] * n))
        assert mine.lib.cuju_environment_step_async(mine.handle, arr, 0, None) == -2
        assert mine.lib.cuju_environment_step_wait(mine.handle) == 0
        acts = [1] * n
        assert mine.step(acts) == ref.step(acts)
    finally:
        for b in batches:
            b.close()


def test_range_wrap_equals_the_reference_and_ends_on_any_angle(host_library):
    """The device code's range wrap (`common.cuh: wrap_range`, host build) equals the reference's
    ModulateIntoRange bit for bit wherever the reference's loops end (|v| below 2^27 for the
    2*pi span), and returns on the angles where those loops never end (infinities, huge values)."""
    import ctypes
    import math
    import os
    import struct

    units_path = os.path.join(os.path.dirname(__file__), '..', 'oracle', '_ref', 'liboracle_units.so')
    if not os.path.isfile(units_path):
        pytest.skip('run make -C oracle for the unit shim')
    units = ctypes.CDLL(units_path)
    mine = ctypes.CDLL(host_library)
    for fn in (units.oracle_modulate_into_range, mine.hostsim_wrap_range):
        fn.argtypes = [ctypes.c_float] * 3
        fn.restype = ctypes.c_float

    def f32(x):
        return struct.unpack('<f', struct.pack('<f', x))[0]

    def bits(x):
        return struct.pack('<f', x)

    pi = f32(math.pi)
    rng = random.Random(29)
    values = [0.0, -0.0, pi, -pi, f32(pi * 1.0000001), 2 * pi, -2 * pi, 7.0, -7.0, 1e-30, 123456.7, -98765.4]
    values += [rng.uniform(-10, 10) for _ in range(2000)]
    values += [rng.uniform(-1e5, 1e5) for _ in range(200)]
    values += [rng.choice((-1, 1)) * rng.uniform(1e6, 1.3e8) for _ in range(6)]
    below = 2.0 ** 27 - 8  # the largest float below 2^27
    values += [f32(below), -f32(below)]
    for v in values:
        v = f32(v)
        assert bits(mine.hostsim_wrap_range(-pi, pi, v)) == bits(units.oracle_modulate_into_range(-pi, pi, v)), v
    for v in (math.inf, -math.inf, 2.0 ** 28, -1e30, 3e38):
        r = mine.hostsim_wrap_range(-pi, pi, v)
        assert not (-pi <= r <= pi)
    assert math.isnan(mine.hostsim_wrap_range(-pi, pi, math.nan))


def test_episode_values_equal_the_reference(host_library):
    """cuju_environment_episode (seed, team order, resets so far, episode offset, bundle, step of the
    last observation, fixed seed, determinism, ticks, agents, players, designated players, and the
    played and scenario difficulties) equals the reference's for every environment, after resets,
    automatic restarts and masked resets, with mixed bundles, fixed seeds and per-side difficulty."""
    import ctypes

    assets = ['academy_empty_goal_close_l1_r0', '5_vs_5_l4_r0']
    batches = _pair(host_library, assets, 6, 31, assignment=[0, 1, 0, 1, 0, 0],
                    fixed_seeds=[-1, 9, -1, -1, 4, -1], episode_number=2,
                    difficulty=[0.4, -1.0, -1.0, 0.7, 0.1, 0.2, 1.0, -1.0, -1.0, -1.0, 0.5, 0.5])
    ref, mine = batches
    for b in batches:
        b.lib.cuju_environment_episode.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]

    def episode(b, index):
        values, difficulty = (ctypes.c_longlong * 17)(), (ctypes.c_float * 4)()
        assert b.lib.cuju_environment_episode(b.handle, index, values, difficulty) == 0
        return list(values), [ctypes.c_float(x).value for x in difficulty]

    rng = random.Random(37)
    try:
        assert mine.reset() == ref.reset()
        for step in range(90):
            acts = [rng.randrange(19) for _ in range(6 * ref.agents)]
            assert mine.step(acts) == ref.step(acts), f'step {step} differs'
            if step % 15 == 7:
                mask = [1 if rng.random() < 0.5 else 0 for _ in range(6)]
                seeds = [rng.randrange(2**32) if rng.random() < 0.5 else -1 for _ in range(6)]
                assert mine.reset_masked(mask, seeds) == ref.reset_masked(mask, seeds)
            if step % 10 == 0:
                for index in range(6):
                    assert episode(mine, index) == episode(ref, index), f'episode {index} at {step}'
    finally:
        for b in batches:
            b.close()


def test_batch_description_equals_the_reference(host_library):
    """The calls that describe a batch (environment count, agents and players per environment and
    side, the difficulty each environment plays, the scenario name of each bundle, the output
    buffers it has) answer as the reference's do for a mixed batch with per-bundle agent counts."""
    import ctypes

    assets = ['11_vs_11_stochastic_l1_r0', '5_vs_5_l4_r0', 'academy_empty_goal_close_l1_r0']
    batches = _pair(host_library, assets, 7, 2, assignment=[2, 1, 0, 1, 2, 0, 0],
                    difficulty=[0.3, -1.0] * 3 + [-1.0, 0.9] * 4)
    p = ctypes.c_void_p
    for b in batches:
        b.lib.cuju_environment_difficulty.argtypes = [p, p]
        b.lib.cuju_environment_difficulty.restype = None
        b.lib.cuju_environment_scenario.argtypes = [p, ctypes.c_int]
        b.lib.cuju_environment_scenario.restype = ctypes.c_char_p
        b.lib.cuju_environment_buffer.argtypes = [p, ctypes.c_char_p]
        b.lib.cuju_environment_buffer.restype = p

    def describe(b):
        out = {'count': b.lib.cuju_environment_count(b.handle)}
        for name in ('agents', 'players'):
            left, right = (ctypes.c_int * 7)(), (ctypes.c_int * 7)()
            total = getattr(b.lib, f'cuju_environment_{name}')(b.handle, left, right)
            out[name] = (total, list(left), list(right))
        difficulty = (ctypes.c_float * 14)()
        b.lib.cuju_environment_difficulty(b.handle, difficulty)
        out['difficulty'] = list(difficulty)
        out['scenarios'] = [b.lib.cuju_environment_scenario(b.handle, i) for i in range(4)]
        out['buffers'] = {name: bool(b.lib.cuju_environment_buffer(b.handle, name))
                          for name in (b'simple115', b'final_simple115', b'reward', b'done', b'score_reward',
                                       b'smm', b'raw', b'no_such_buffer')}
        return out

    try:
        assert describe(mine := batches[1]) == describe(batches[0])
        assert mine.reset() == batches[0].reset()
        assert describe(mine) == describe(batches[0])
    finally:
        for b in batches:
            b.close()


def test_argument_refusals_equal_the_reference(host_library):
    """Arguments the reference refuses are refused here too, with -1 (or null) and no change to the
    batch: a difficulty above 1 or NaN, a seed below -1 or above 2^32 - 1, a reverse flag other than
    0 or 1, and an environment index outside the batch."""
    import ctypes
    import math

    batches = _pair(host_library, '5_vs_5_l4_r0', 3, 4)
    ref, mine = batches
    p = ctypes.c_void_p
    for b in batches:
        b.lib.cuju_environment_set_difficulty.argtypes = [p, p]
        b.lib.cuju_environment_get_state.argtypes = [p, ctypes.c_int, p, p]
        b.lib.cuju_environment_get_state.restype = p
    try:
        assert mine.reset() == ref.reset()

        def codes(call):
            return [call(b) for b in batches]

        for bad in (1.5, math.nan):
            values = (ctypes.c_float * 6)(*([0.5] * 5 + [bad]))
            assert codes(lambda b: b.lib.cuju_environment_set_difficulty(b.handle, values)) == [-1, -1]
        ones = (ctypes.c_ubyte * 3)(1, 1, 1)
        for seeds in ([-2, 0, 0], [0, 2**32, 0]):
            arr = (ctypes.c_longlong * 3)(*seeds)
            assert codes(lambda b: b.lib.cuju_environment_reset_masked(b.handle, ones, 0, arr, None, None, 1)) == [-1, -1]
        reverse = (ctypes.c_int * 3)(0, 2, 1)
        assert codes(lambda b: b.lib.cuju_environment_reset(b.handle, None, reverse, None)) == [-1, -1]
        size, episode = ctypes.c_ulonglong(), (ctypes.c_int * 25)()
        for index in (-1, 3):
            assert codes(lambda b: b.lib.cuju_environment_get_state(b.handle, index, ctypes.byref(size), episode)) == \
                [None, None]
        acts = [2] * (3 * ref.agents)
        assert mine.step(acts) == ref.step(acts)
        for index in range(3):
            assert mine.engine_state(index) == ref.engine_state(index)
    finally:
        for b in batches:
            b.close()


def test_state_moves_between_batches_of_mixed_bundles(host_library):
    """A state taken from one environment of the reference batch and loaded into the environment
    of the same bundle in both batches gives the same outputs and state from then on; loading it
    into an environment of another bundle is refused by both."""
    import ctypes

    assets = ['academy_empty_goal_close_l1_r0', '5_vs_5_l4_r0']
    batches = _pair(host_library, assets, 4, 8, assignment=[0, 1, 0, 1])
    ref, mine = batches
    rng = random.Random(41)
    p = ctypes.c_void_p
    try:
        assert mine.reset() == ref.reset()
        for step in range(25):
            acts = [rng.randrange(19) for _ in range(4 * ref.agents)]
            assert mine.step(acts) == ref.step(acts)
        data, episode = ref.engine_state(3)
        values = (ctypes.c_int * 25)(*episode[:25])
        for b in batches:
            b.lib.cuju_environment_set_state.argtypes = [p, ctypes.c_int, ctypes.c_char_p, ctypes.c_ulonglong, p]
        assert [b.lib.cuju_environment_set_state(b.handle, 0, data, len(data), values) for b in batches] == [-1, -1]
        assert mine.set_state(1, data, episode) == ref.set_state(1, data, episode)
        for step in range(25):
            acts = [rng.randrange(19) for _ in range(4 * ref.agents)]
            assert mine.step(acts) == ref.step(acts), f'step {step} after the load differs'
        for index in range(4):
            assert mine.engine_state(index) == ref.engine_state(index)
    finally:
        for b in batches:
            b.close()


@pytest.mark.parametrize('assets,representation,stack,checkpoints', [
    ('11_vs_11_stochastic_l1_r1', 4, 4, True),
    ('academy_3_vs_1_with_keeper_l3_r0', 8, 1, True),
    ('5_vs_5_l4_r0', 1, 4, False),
])
def test_option_combinations(host_library, assets, representation, stack, checkpoints):
    """Combinations the golden cases do not hold: stacked SMM with checkpoint rewards and a right
    agent, raw with three agents and checkpoints, stacked simple115 (v1) with four agents."""
    batches = _pair(host_library, assets, 3, 13, representation=representation, stack=stack,
                    checkpoints=checkpoints)
    ref, mine = batches
    rng = random.Random(43)
    try:
        assert mine.reset() == ref.reset()
        for step in range(50):
            acts = [rng.randrange(19) for _ in range(3 * ref.agents)]
            assert mine.step(acts) == ref.step(acts), f'step {step} differs'
    finally:
        for b in batches:
            b.close()


def test_first_index_at_the_end_of_the_seed_range(host_library):
    """The last environments of the seed rule's 2^32 range play as the reference's, and a batch
    that would run past the range is refused by both (reference tests/test_first_index.py)."""
    from oracle.driver import OracleBatch

    from conftest import ANIMATIONS, resolve

    last = 2**32 - 3
    batches = _pair(host_library, 'academy_empty_goal_close_l1_r0', 3, 6, first_index=last)
    ref, mine = batches
    try:
        assert mine.reset() == ref.reset()
        _run(batches, 60, random.Random(47))
    finally:
        for b in batches:
            b.close()
    paths, counts = resolve('academy_empty_goal_close_l1_r0')
    for library in (None, host_library):
        with pytest.raises(RuntimeError):
            OracleBatch(paths, counts, 3, 6, ANIMATIONS, threads=1, library=library, first_index=last + 1)


@pytest.mark.parametrize('size', [(48, 36), (120, 80)])
def test_minimap_of_another_size(host_library, size):
    """The SMM (`extracted`) minimap at a width and height other than GRF's default 96 x 72, stacked,
    as the reference draws it (configuration smm_width / smm_height)."""
    batches = _pair(host_library, '5_vs_5_l4_r0', 3, 17, representation=4, stack=4, smm_size=size)
    ref, mine = batches
    rng = random.Random(53)
    try:
        assert mine.reset() == ref.reset()
        for step in range(40):
            acts = [rng.randrange(19) for _ in range(3 * ref.agents)]
            assert mine.step(acts) == ref.step(acts), f'step {step} differs'
    finally:
        for b in batches:
            b.close()


@pytest.mark.parametrize('representation,stack', [(2, 1), (1, 4), (4, 1)])
def test_final_observation_buffers_equal_the_reference(host_library, representation, stack):
    """The observation that ended each episode (`final_simple115`, `final_smm`), which the automatic
    restart keeps beside the new episode's first observation, equals the reference's after every
    step of a drill that ends many episodes."""
    batches = _pair(host_library, 'academy_empty_goal_close_l1_r0', 6, 59, representation=representation,
                    stack=stack)
    ref, mine = batches
    name = 'final_smm' if representation == 4 else 'final_simple115'
    per_env = (96 * 72 * 4 * stack) if representation == 4 else 4 * 115 * stack
    rng = random.Random(61)
    ended = 0
    try:
        assert mine.reset() == ref.reset()
        for step in range(120):
            acts = [rng.randrange(19) for _ in range(6 * ref.agents)]
            out = ref.step(acts)
            assert mine.step(acts) == out, f'step {step} differs'
            ended += sum(out[2])
            size = 6 * ref.agents * per_env
            assert mine._buffer(name, size) == ref._buffer(name, size), f'{name} differs at step {step}'
        assert ended > 0
    finally:
        for b in batches:
            b.close()


def test_final_raw_equals_the_reference(host_library):
    """`final_raw` (every raw array of each ended episode's last observation) equals the
    reference's after every step of a drill that ends many episodes."""
    batches = _pair(host_library, 'academy_empty_goal_close_l1_r0', 4, 67, representation=8)
    ref, mine = batches
    rng = random.Random(71)
    try:
        assert mine.reset() == ref.reset()
        ended = 0
        for step in range(100):
            acts = [rng.randrange(19) for _ in range(4 * ref.agents)]
            out = ref.step(acts)
            assert mine.step(acts) == out, f'step {step} differs'
            ended += sum(out[2])
            assert mine._raw_bytes('final_raw') == ref._raw_bytes('final_raw'), f'final_raw differs at step {step}'
        assert ended > 0
    finally:
        for b in batches:
            b.close()


def test_a_difficulty_set_between_episodes_applies_from_the_next_reset(host_library):
    """cuju_environment_set_difficulty during play changes nothing until an environment's next
    reset, and then only the side it names (negative keeps the scenario's), as in the reference
    (tests/test_difficulty.py)."""
    import ctypes

    batches = _pair(host_library, '11_vs_11_easy_stochastic_l1_r0', 3, 73)
    ref, mine = batches
    p = ctypes.c_void_p
    for b in batches:
        b.lib.cuju_environment_set_difficulty.argtypes = [p, p]
    rng = random.Random(79)
    try:
        assert mine.reset() == ref.reset()
        for step in range(30):
            acts = [rng.randrange(19) for _ in range(3 * ref.agents)]
            assert mine.step(acts) == ref.step(acts)
            if step == 5:
                values = (ctypes.c_float * 6)(0.9, -1.0, -1.0, 0.05, 0.5, 0.5)
                assert [b.lib.cuju_environment_set_difficulty(b.handle, values) for b in batches] == [0, 0]
            if step == 15:
                assert mine.reset_masked([1, 0, 1], [5, -1, 7]) == ref.reset_masked([1, 0, 1], [5, -1, 7])
        for index in range(3):
            assert mine.engine_state(index) == ref.engine_state(index)
    finally:
        for b in batches:
            b.close()


def test_a_capped_loop_ends_the_step_with_the_undefined_path_error(host_library):
    """A state whose match generator has an empty range (minimum equal to maximum, which no valid
    state holds) makes Boost's uniform-float redraw loop run to its cap on the next draw: the loop
    gives up, the environment's status records a path GRF leaves undefined, and the step returns an
    error that the Python layer raises as UndefinedPathError. The other environment keeps its state.
    The reference's own loop never ends on such a state, so it is not run here."""
    import struct

    from cuju_b200.errors import UndefinedPathError, from_library
    from oracle.driver import OracleBatch

    paths, counts = resolve('5_vs_5_l4_r0')
    batch = OracleBatch(paths, counts, 2, 7, ANIMATIONS, threads=1, library=host_library)
    try:
        batch.reset()
        for _ in range(3):
            batch.step([0] * (2 * batch.agents))
        engine, episode = batch.engine_state(0)
        healthy = batch.engine_state(1)
        # The match generator's bytes start at byte 8 of the engine state: 624 words, a 64-bit
        # index, then the range's minimum and maximum floats (0 and 1 in every valid state).
        at = 8 + 624 * 4 + 8
        assert struct.unpack_from('<ff', engine, at) == (0.0, 1.0)
        broken = engine[:at] + struct.pack('<ff', 1.0, 1.0) + engine[at + 8:]
        batch.set_state(0, broken, episode)
        rc, message = 0, ''
        for _ in range(20):
            rc, message = batch.step_status([0] * (2 * batch.agents))
            if rc:
                break
        assert rc == -1
        assert isinstance(from_library(message), UndefinedPathError), message
        assert batch.engine_state(1) != healthy  # the healthy environment stepped on
    finally:
        batch.close()


def test_the_repeated_ball_prediction_shortcut_equals_a_second_prediction(host_library):
    """ball_touch predicts the ball's flight twice on unchanged inputs; the build replaces the
    second run by its exact outcome (touch.cuh: ball_recalc_again). On seeded balls on the ground,
    in flight, at rest, against a post and in the goal's net, both give the same ball, byte for
    byte: where the second run recomputes every entry, and where its cache shifts the list (half
    the trials set up a ball that stays put between 10 and 20 ms)."""
    import ctypes

    lib = ctypes.CDLL(host_library)
    shifted = ctypes.c_int()
    bad = lib.hostsim_check_recalc_again(ctypes.c_uint(2024), 1000, ctypes.byref(shifted))
    assert bad == 0
    assert shifted.value >= 500
