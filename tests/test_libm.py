"""The library's restatements of glibc's math functions (cuju_b200/csrc/libm.cuh), compiled for the
host, against the reference's own restatements of the same functions (cuju include/cuju/libm/*.h,
built into oracle/_ref/liboracle_units.so), function by function and bit for bit: sinf, cosf and
their pair, powf (and its positive-base form), acosf, asinf, atanf, atan2f, and the double sin,
cos, acos and pow. The arguments are seeded: special values, the ranges the simulation uses and
wide magnitudes. tests/test_gpu_libm.py runs the same check on the device build."""

import ctypes

import pytest

from conftest import LIBM_NAMES, libm_compare, libm_inputs


@pytest.mark.parametrize('which', sorted(LIBM_NAMES), ids=[LIBM_NAMES[k] for k in sorted(LIBM_NAMES)])
def test_host_build_equals_the_reference(host_library, which):
    lib = ctypes.CDLL(host_library)
    xs, ys = libm_inputs(which)
    bad = libm_compare(lib.hostsim_libm, which, xs, ys)
    assert bad is None, f'{LIBM_NAMES[which]}{bad[:2]}: this build {bad[2]!r}, reference {bad[3]!r}'
