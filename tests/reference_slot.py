"""The reference's slot (`streamvoxel/stream/slot.py:50-176`, `LowEntropyLastSlot`) for the GPU parity tests
(TEST INFRASTRUCTURE ONLY).

The host bookkeeping, the quotas and the block-quota selection are the oracle's (`oracle/sampler.py`, pinned to
the reference's fixtures); the two device decisions are the reference's own torch calls on the device that holds the
logits and the slot generator:

* marking: `logits.float().softmax(0)[air].sum(0)` (`slot.py:126`);
* the draw: `torch.multinomial(logits.permute(1, 2, 3, 0)[chosen].float().softmax(-1), 1, generator)`
  (`slot.py:149-150`) on a CUDA generator seeded with the window seed (`slot.py:100`).

The entropy that ranks voxels inside a block is passed in (`scores`): the parity contract compares the sampler given
the same fp32 scores, and the kernel's scores are checked against `entropy_scores` within 1e-5 separately.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import sampler as osm


class ReferenceSlot:
    def __init__(self, shape, classes, air_ids=(0,), air_token=0, last_eps=1e-4, block_size=4, device='cuda'):
        self.slot = osm.Slot(shape, classes, air_ids, air_token, last_eps, block_size)
        self.shape, self.classes, self.air_ids = tuple(shape), int(classes), tuple(air_ids)
        self.device = torch.device(device)
        self.generator = None

    @property
    def idle(self):
        return self.slot.idle

    @property
    def phase(self):
        return self.slot.phase

    def arm(self, seed, cap, target, order):
        self.slot.arm(seed, cap, target, np.asarray(order))
        self.generator = torch.Generator(device=self.device).manual_seed(int(seed))

    def consume(self, logits, tokens, scores=None):
        """logits: device tensor [C, Y, Z, X] (any float dtype); tokens: host int array [Y, Z, X], updated in place;
        scores: host fp32 [Y, Z, X] (needed for solid steps)."""
        slot = self.slot
        if slot.phase == 'marking':
            air = logits.float().softmax(0)[list(self.air_ids)].sum(0).cpu().numpy()
            return slot.consume(None, tokens, air=air)
        flat = logits.reshape(self.classes, -1)

        def draw(positions):
            index = torch.as_tensor(positions, dtype=torch.long, device=logits.device)
            p = flat.index_select(1, index).t().contiguous().float().softmax(-1)
            return torch.multinomial(p, 1, generator=self.generator).squeeze(-1).cpu().numpy()

        return slot.consume(None, tokens, scores=scores, draw=draw)
