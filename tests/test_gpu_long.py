"""The reference's long golden matches on the B200 (cuju tests/test_long.py; digests.json
`long_cases`): full 3,010-step 11-a-side matches with their automatic restart (simple115v2 and the
raw representation), a full 5-a-side match with checkpoint rewards, and academy drills over many
episodes (the extracted minimap, checkpoints). Every observation, reward and done flag of every
step goes into the digest, then every environment's GRF state bytes.

An environment's step is a long serial computation, so these matches are latency-bound: the five
batches run at once, each on a CUDA stream of its own, and each step's outputs are copied to the
host on that stream without waiting; the digests are taken as the copies land.
"""

import hashlib

import pytest
import torch

from conftest import actions_at, golden, needs_data

pytestmark = [pytest.mark.gpu, needs_data]

CHUNK = 50  # steps between the host's reads of one batch's outputs


class _Run:
    def __init__(self, name, entry, seed, environments):
        from cuju_b200 import BatchEnvironment

        self.name = name
        self.steps = entry['steps']
        self.stream = torch.cuda.Stream()
        with torch.cuda.stream(self.stream):
            self.batch = BatchEnvironment(entry['assets'], environment_count=environments, seed=seed, **entry['options'])
            self.actions = torch.tensor([actions_at(step, environments, self.batch.agents, self.batch.action_count)
                                         for step in range(self.steps)], dtype=torch.int32).cuda()
        self.digest = hashlib.sha256()
        self.pending = []

    def _record(self, observation, reward, done):
        tensors = [observation[k] for k in sorted(observation)] if isinstance(observation, dict) else [observation]
        tensors += [reward, done]
        if not hasattr(self, 'slots'):
            # CHUNK sets of pinned host buffers, reused after every drain.
            self.slots = [[torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in tensors]
                          for _ in range(CHUNK)]
        copies = self.slots[len(self.pending)]
        for host, t in zip(copies, tensors):
            host.copy_(t, non_blocking=True)
        self.pending.append(copies)

    def _drain(self):
        self.stream.synchronize()
        for copies in self.pending:
            for host in copies:
                self.digest.update(host.contiguous().numpy().tobytes())
        self.pending = []

    def reset(self):
        with torch.cuda.stream(self.stream):
            observation = self.batch.reset()
        self.stream.synchronize()
        for t in ([observation[k] for k in sorted(observation)] if isinstance(observation, dict) else [observation]):
            self.digest.update(t.cpu().contiguous().numpy().tobytes())

    def step(self, step):
        if step >= self.steps:
            return
        with torch.cuda.stream(self.stream):
            observation, reward, done, _ = self.batch.step(self.actions[step], synchronize=False)
            self._record(observation, reward, done)
        if len(self.pending) >= CHUNK or step == self.steps - 1:
            self._drain()

    def finish(self, environments):
        self._drain()
        self.batch.synchronize()
        if not self.batch.stacked:
            for index in range(environments):
                self.digest.update(self.batch.get_state(index))
        self.batch.close()
        return self.digest.hexdigest()


def test_long_golden_digests():
    g = golden()
    environments = g['environments']
    runs = [_Run(name, entry, g['seed'], environments) for name, entry in sorted(g['long_cases'].items())]
    try:
        for run in runs:
            run.reset()
        for step in range(max(run.steps for run in runs)):
            for run in runs:
                run.step(step)
        results = {run.name: run.finish(environments) for run in runs}
    finally:
        for run in runs:
            run.batch.close()
    for name, entry in g['long_cases'].items():
        assert results[name] == entry['digest'], f'{name} differs from the golden digest'
