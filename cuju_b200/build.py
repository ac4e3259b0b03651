"""Builds the B200 library in-tree and stages the read-only data it loads.

* `lib/libcuju_b200.so` from `csrc/kernels.cu` (the device kernels) and `csrc/api.cu` (host batch
  and C-ABI), for sm_100a only, with IEEE float semantics (no FMA contraction, exact division and
  square root, no flush to zero) because every environment must match the reference bit for bit.
* `data/`: the asset bundles (`assets/*.cjb`) and `animations.bin` the library reads, copied from
  the reference package when it is present (the GPU box receives the staged copy).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, 'csrc')
LIB_DIR = os.path.join(HERE, 'lib')
LIBRARY = os.path.join(LIB_DIR, 'libcuju_b200.so')
DATA = os.path.join(HERE, 'data')
# The reference checkout: CUJU_REFERENCE, else a `reference` directory beside the repository.
REFERENCE = os.environ.get('CUJU_REFERENCE') or os.path.normpath(os.path.join(ROOT, '..', 'reference'))

NVCC_FLAGS = [
    '-std=c++17', '-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '-lineinfo',
    '--fmad=false', '-prec-div=true', '-prec-sqrt=true', '-ftz=false',
    '-Xcompiler', '-ffp-contract=off,-fPIC,-fvisibility=hidden',
]
SOURCES = ['kernels.cu', 'api.cu']


def _nvcc() -> str:
    for candidate in (os.environ.get('NVCC'), '/usr/local/cuda/bin/nvcc', shutil.which('nvcc')):
        if candidate and os.path.isfile(candidate):
            return candidate
    raise RuntimeError('nvcc not found')


def _sources_mtime() -> float:
    latest = 0.0
    for name in os.listdir(CSRC):
        latest = max(latest, os.path.getmtime(os.path.join(CSRC, name)))
    header = os.path.join(ROOT, 'include', 'cuju_b200.h')
    if os.path.isfile(header):
        latest = max(latest, os.path.getmtime(header))
    return latest


def build_library(force: bool = False) -> str:
    """Compiles the library unless it is newer than every source."""
    if not force and os.path.isfile(LIBRARY) and os.path.getmtime(LIBRARY) >= _sources_mtime():
        return LIBRARY
    os.makedirs(LIB_DIR, exist_ok=True)
    obj_dir = os.path.join(ROOT, '_build')
    os.makedirs(obj_dir, exist_ok=True)
    nvcc = _nvcc()
    procs, objects = [], []
    for src in SOURCES:
        obj = os.path.join(obj_dir, src.replace('.cu', '.o'))
        objects.append(obj)
        procs.append(subprocess.Popen([nvcc, *NVCC_FLAGS, '-c', os.path.join(CSRC, src), '-o', obj],
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    for proc, src in zip(procs, SOURCES):
        out, _ = proc.communicate()
        if proc.returncode != 0:
            raise RuntimeError(f'nvcc failed on {src}:\n{out.decode(errors="replace")[-4000:]}')
    tmp = LIBRARY + '.tmp'
    subprocess.run([nvcc, '-shared', '-gencode', 'arch=compute_100a,code=sm_100a', *objects, '-o', tmp,
                    '-Xlinker', '--exclude-libs,ALL'], check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


def stage_data() -> str:
    """Copies the bundles and animation tables from the reference package, when present."""
    source = os.path.join(REFERENCE, 'python', 'cuju', 'data')
    if not os.path.isdir(source):
        if not os.path.isfile(os.path.join(DATA, 'animations.bin')):
            raise RuntimeError(f'no staged data in {DATA} and no reference package at {source}')
        return DATA
    os.makedirs(os.path.join(DATA, 'assets'), exist_ok=True)
    shutil.copyfile(os.path.join(source, 'animations.bin'), os.path.join(DATA, 'animations.bin'))
    for name in os.listdir(os.path.join(source, 'assets')):
        if name.endswith('.cjb'):
            shutil.copyfile(os.path.join(source, 'assets', name), os.path.join(DATA, 'assets', name))
    return DATA


def build_oracle() -> None:
    """Builds the reference CPU backend (the parity checker) into oracle/_ref, when the reference
    sources are present."""
    if not os.path.isdir(os.path.join(REFERENCE, 'include', 'cuju')):
        return
    subprocess.run(['make', '-s', '-C', os.path.join(ROOT, 'oracle'), f'REF={REFERENCE}'], check=True)


def build(force: bool = False) -> None:
    stage_data()
    build_library(force)
    build_oracle()


if __name__ == '__main__':
    build(force='--force' in sys.argv)
    print(LIBRARY)
