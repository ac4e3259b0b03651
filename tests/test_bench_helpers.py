"""Host logic of bench.py (no GPU): each rank's slice of a configuration, the interleaved bundle
assignment of configuration 5, and the number of kernel launches a step takes (waves), which the
bench line reports as `gpu_launches`."""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_slices_split_or_repeat_by_configuration():
    # Configuration 3 repeats its 16,384 environments per rank (weak scaling); 4 and 5 split theirs.
    assert bench.slice_of(bench.CONFIGS[3], 8, 5) == (16384, 5 * 16384)
    assert bench.slice_of(bench.CONFIGS[4], 8, 3) == (8192, 3 * 8192)
    assert bench.slice_of(bench.CONFIGS[5], 8, 7) == (16384, 7 * 16384)
    slices = [bench.slice_of(bench.CONFIGS[4], 4, rank) for rank in range(4)]
    covered = sorted(e for count, first in slices for e in range(first, first + count))
    assert covered == list(range(65536))


def test_mixed_assignment_follows_the_global_index():
    cfg = bench.CONFIGS[5]
    whole = bench.assignment_of(cfg, 20, 0)
    assert whole == [0, 1, 0, 1, 2] * 4
    assert bench.assignment_of(cfg, 7, 13) == whole[13:20]
    assert bench.assignment_of(bench.CONFIGS[3], 10, 0) is None


def test_waves_per_step():
    sms = 148
    assert bench.waves_for(16384, 0, sms) == 1      # 3-4 warps per SM, one launch
    assert bench.waves_for(18944, 0, sms) == 1      # exactly four warps on every SM
    assert bench.waves_for(18945, 0, sms) == 2
    assert bench.waves_for(20000, 0, sms) == 2
    assert bench.waves_for(32768, 0, sms) == 2
    assert bench.waves_for(65536, 0, sms) == 4
    assert bench.waves_for(131072, 0, sms) == 7
    assert bench.waves_for(4096, 0, sms) == 1       # four lanes per environment
    assert bench.waves_for(4096, 32, sms) == 7      # a warp each: 592 environments a wave
    assert bench.waves_for(64, 0, sms) == 1
