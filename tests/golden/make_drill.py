"""Builds the drill bundle of the benchmark's second configuration from the repository's scenario
file (academy_attacker_vs_keeper.py), with the reference's own host-side bundle builder: its
Python scenario runner (python/cuju/scenarios.py, build_bundle) over the reference CPU library
built by oracle/Makefile (its cuju_scenario_build_bundle). Run where the reference checkout is
(CUJU_REFERENCE, else a `reference` directory beside the repository); the bundle it writes,
academy_attacker_vs_keeper_l0_r0.cjb, is committed beside this script.
"""

import os
import shutil
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REFERENCE = os.environ.get('CUJU_REFERENCE') or os.path.normpath(os.path.join(ROOT, '..', 'reference'))
NAME = 'academy_attacker_vs_keeper'


def main():
    package = os.path.join(REFERENCE, 'python')
    library = os.path.join(ROOT, 'oracle', '_ref', 'libcuju_cpu.so')
    animations = os.path.join(ROOT, 'cuju_b200', 'data', 'animations.bin')
    for path in (package, library, animations):
        if not os.path.exists(path):
            raise SystemExit(f'missing {path}')
    sys.path.insert(0, package)
    from cuju import scenarios

    with tempfile.TemporaryDirectory() as tmp:
        # The scenario file imports the builder's names relatively, as GRF's scenario files do:
        # run it from a copy inside the reference's scenario package namespace.
        target = os.path.join(HERE, NAME + '_l0_r0.cjb')
        scenario = os.path.join(tmp, NAME + '.py')
        shutil.copyfile(os.path.join(HERE, NAME + '.py'), scenario)
        scenarios.build_bundle(scenario, target, name=NAME, device='cpu', library=library, animations=animations)
    print(target, os.path.getsize(target), 'bytes')


if __name__ == '__main__':
    main()
