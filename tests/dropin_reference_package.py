"""Run by tests/test_gpu_dropin.py in a fresh interpreter: drives this repository's library through
the reference's own, unmodified Python package (`cuju.BatchEnvironment`, copied beside the oracle
by oracle/Makefile), with CUJU_CUDA_LIBRARY naming libcuju_b200.so and CUJU_CPU_LIBRARY the
reference CPU backend. Prints one JSON object:

* `digests`: the golden digest of every short case, played as the reference's tests play them
  (seed 7, 4 environments, 100 steps of its arithmetic actions; every observation, reward and done,
  then every environment's state bytes);
* `masked`: a 5-a-side batch stepped on `cuda` (this library) and on `cpu` (the reference CPU
  backend) through the same package, with masked resets that take host seeds; every output and
  the final state bytes compared, the number of compared steps and the first difference if any.
"""

import hashlib
import json
import os
import sys

import torch

import cuju


def tensor_bytes(tensor):
    return tensor.detach().to('cpu').contiguous().numpy().tobytes()


def actions_at(step, environments, agents, action_count):
    return torch.tensor([[(step * 7 + e * 3 + a * 5) % action_count for a in range(agents)]
                         for e in range(environments)], dtype=torch.int32)


def digest(assets, steps, seed, environments, options):
    batch = cuju.BatchEnvironment(assets, environment_count=environments, device='cuda', seed=seed, **options)
    h = hashlib.sha256()

    def add(observation):
        if isinstance(observation, dict):
            for name in sorted(observation):
                h.update(tensor_bytes(observation[name]))
        else:
            h.update(tensor_bytes(observation))

    add(batch.reset())
    for step in range(steps):
        observation, reward, done, _ = batch.step(actions_at(step, environments, batch.agents,
                                                             batch.action_count).to(batch.torch_device))
        add(observation)
        h.update(tensor_bytes(reward))
        h.update(tensor_bytes(done))
    if not batch.stacked:
        for index in range(environments):
            h.update(batch.get_state(index))
    batch.close()
    return h.hexdigest()


def outputs(observation, reward, done):
    return tensor_bytes(observation), tensor_bytes(reward), tensor_bytes(done)


def masked_resets(environments=8, steps=60):
    batches = {d: cuju.BatchEnvironment('5_vs_5_l4_r0', environment_count=environments, device=d, seed=3)
               for d in ('cuda', 'cpu')}
    generator = torch.Generator().manual_seed(5)
    result = {'steps': 0, 'difference': None}
    try:
        first = {d: tensor_bytes(b.reset()) for d, b in batches.items()}
        if first['cuda'] != first['cpu']:
            result['difference'] = 'reset'
            return result
        for step in range(steps):
            actions = torch.randint(0, 19, (environments, 4), generator=generator, dtype=torch.int32)
            got = {}
            for d, b in batches.items():
                observation, reward, done, _ = b.step(actions.to(b.torch_device))
                got[d] = outputs(observation, reward, done)
            if got['cuda'] != got['cpu']:
                result['difference'] = f'step {step}'
                return result
            if step % 7 == 3:
                mask = torch.rand(environments, generator=generator) < 0.4
                seeds = [int(x) if m else -1 for x, m in
                         zip(torch.randint(0, 2**32 - 1, (environments,), generator=generator, dtype=torch.int64), mask)]
                reset = {d: tensor_bytes(b.reset(seeds=seeds, mask=mask.tolist())) for d, b in batches.items()}
                if reset['cuda'] != reset['cpu']:
                    result['difference'] = f'masked reset after step {step}'
                    return result
            result['steps'] = step + 1
        for index in range(environments):
            if batches['cuda'].get_state(index) != batches['cpu'].get_state(index):
                result['difference'] = f'state {index}'
                return result
    finally:
        for b in batches.values():
            b.close()
    return result


def main():
    golden = json.load(open(sys.argv[1], encoding='utf-8'))
    cases = [c for c in golden['cases']]
    report = {'library': os.environ.get('CUJU_CUDA_LIBRARY'), 'package': os.path.dirname(cuju.__file__),
              'digests': {}, 'masked': None}
    for case in cases:
        entry = golden['cases'][case]
        report['digests'][case] = digest(entry['assets'], golden['steps'], golden['seed'], golden['environments'],
                                         entry['options'])
    report['masked'] = masked_resets()
    print(json.dumps(report))


if __name__ == '__main__':
    main()
