"""The library's restatements of glibc's math functions on a B200, against the reference's own
restatements (cuju include/cuju/libm/*.h in oracle/_ref/liboracle_units.so), function by function
and bit for bit on the arguments tests/test_libm.py uses for the host build. The device side is
tests/host/libm_device.cu, built here for sm_100a with the library's floating-point flags
(cuju_b200/build.py), so it runs the same compiled arithmetic as the kernels."""

import ctypes
import os
import shutil
import subprocess

import pytest

from conftest import LIBM_NAMES, ROOT, libm_compare, libm_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def device_library(tmp_path_factory):
    from cuju_b200.build import NVCC_FLAGS

    nvcc = shutil.which('nvcc') or '/usr/local/cuda/bin/nvcc'
    out = str(tmp_path_factory.mktemp('libm') / 'liblibm_device.so')
    subprocess.run([nvcc, *NVCC_FLAGS, '-I', os.path.join(ROOT, 'cuju_b200', 'csrc'), '-shared',
                    os.path.join(ROOT, 'tests', 'host', 'libm_device.cu'), '-o', out], check=True, capture_output=True)
    return ctypes.CDLL(out)


@pytest.mark.parametrize('which', sorted(LIBM_NAMES), ids=[LIBM_NAMES[k] for k in sorted(LIBM_NAMES)])
def test_device_build_equals_the_reference(device_library, which):
    xs, ys = libm_inputs(which)
    bad = libm_compare(device_library.libm_device_eval, which, xs, ys)
    assert bad is None, f'{LIBM_NAMES[which]}{bad[:2]}: this build {bad[2]!r}, reference {bad[3]!r}'
