"""Writes tests/golden/digests.json from the reference package (run where the reference is).

The file is the reference's own known-answer set for the batched step (cuju
python/cuju/data/digests.json): SHA-256 digests of every observation, reward and done flag of
every step, then every environment's `get_state`, for seed 7, 4 environments and the actions
(step * 7 + environment * 3 + agent * 5) % action_count of cuju tests/conftest.py:60-66. It is
copied unchanged so the GPU tests compare against the reference's published answers.
"""

import json
import os
import sys

# The reference checkout: CUJU_REFERENCE, else a `reference` directory beside the repository.
REFERENCE = os.environ.get('CUJU_REFERENCE') or os.path.normpath(
    os.path.join(os.path.dirname(os.path.abspath(__file__)), '..', '..', '..', 'reference'))


def main():
    source = os.path.join(REFERENCE, 'python', 'cuju', 'data', 'digests.json')
    with open(source, encoding='utf-8') as handle:
        digests = json.load(handle)
    target = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'digests.json')
    with open(target, 'w', encoding='utf-8') as handle:
        json.dump(digests, handle, indent=1, sort_keys=True)
        handle.write('\n')
    print(target, len(digests['cases']), 'cases', len(digests['long_cases']), 'long cases')


if __name__ == '__main__':
    sys.exit(main())
