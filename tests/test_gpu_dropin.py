"""The drop-in claim, checked through the reference's own Python package: its unmodified
`cuju.BatchEnvironment` (copied beside the oracle by oracle/Makefile) loads libcuju_b200.so through
CUJU_CUDA_LIBRARY, exactly as a user of the reference would switch backends
(python/cuju/_batch/library.py:194-276), and reproduces every short golden digest (every output of
100 steps, then the state bytes), and a batch with masked resets on host seeds steps bit for bit
like the same package driving the reference CPU backend. Runs in a fresh interpreter so that
`import cuju` is the reference's package and the environment variables are read at its load."""

import json
import os
import subprocess
import sys

import pytest

from conftest import GOLDEN, ROOT, needs_data

pytestmark = [pytest.mark.gpu, needs_data]

PACKAGE = os.path.join(ROOT, 'oracle', '_ref', 'pkg')
LIBRARY = os.path.join(ROOT, 'cuju_b200', 'lib', 'libcuju_b200.so')
CPU_LIBRARY = os.path.join(ROOT, 'oracle', '_ref', 'libcuju_cpu.so')


@pytest.mark.skipif(not os.path.isfile(os.path.join(PACKAGE, 'cuju', '__init__.py')),
                    reason='run make -C oracle to stage the reference package')
def test_reference_package_binds_this_library():
    env = dict(os.environ, CUJU_CUDA_LIBRARY=LIBRARY, CUJU_CPU_LIBRARY=CPU_LIBRARY,
               PYTHONPATH=PACKAGE + os.pathsep + os.environ.get('PYTHONPATH', ''))
    run = subprocess.run([sys.executable, os.path.join(ROOT, 'tests', 'dropin_reference_package.py'), GOLDEN],
                         env=env, capture_output=True, text=True, timeout=1500, cwd=os.path.join(ROOT, 'tests'))
    assert run.returncode == 0, run.stderr[-4000:]
    report = json.loads(run.stdout.strip().splitlines()[-1])
    assert report['package'].startswith(PACKAGE), report['package']
    with open(GOLDEN, encoding='utf-8') as handle:
        golden = json.load(handle)
    wrong = [case for case, entry in golden['cases'].items() if report['digests'][case] != entry['digest']]
    assert not wrong, f'digests differ through the reference package: {wrong}'
    assert report['masked']['difference'] is None, report['masked']
    assert report['masked']['steps'] == 60
