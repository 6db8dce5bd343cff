"""Single-column decoding from an all-MASK column: the BASELINE config-1 driver.

`decode_low_entropy_last` restates `streamvoxel/eval/samplers.py:118-134`: one slot of the shipped sampler driven by a
model forward until its window finishes (one marking forward, then the solid steps of the quartercos schedule, the
low-entropy-last voxels committed at finish). `UnconditionalForward` is the time-free DiT-B/4 alone on our engine
(`streamvoxel/models/unconditional_md4_timefree.py`), batch 1.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from streamvoxel_b200.stream.fast_ops import FastLowEntropyLastSlot


class UnconditionalForward:
    """Callable (tokens [1, Y, Z, X] int16, timestep) -> logits [1, V, Y, Z, X] bf16 of the time-free model (the
    timestep is accepted for the reference's call shape; the model ignores it)."""

    def __init__(self, cfg, state_dict, device='cuda'):
        from streamvoxel_b200.model import Engine, PreparedModel
        self.cfg, self.device = cfg, torch.device(device)
        self.engine = Engine(PreparedModel(cfg, state_dict, self.device), 1, 0)
        self.logits = torch.empty((1, cfg.classes, *cfg.voxel_shape), dtype=torch.bfloat16, device=self.device)

    def __call__(self, tokens, timestep=None):
        tokens = tokens.to(torch.int16).contiguous()
        return self.engine.forward(1, tokens, self.logits)


@torch.inference_mode()
def decode_low_entropy_last(forward, spec, seed, device, shape, classes, sampling='parity'):
    """Decode one column: returns (dict(compact=[Y,Z,X] int16, commit_step=[Y,Z,X] step map), info) with info keys
    spec, complete, remaining, nfe, last_count, last_frac, seconds (`samplers.py:130-134`)."""
    device = torch.device(device)
    slot = FastLowEntropyLastSlot(tuple(shape), classes, spec['air_ids'], spec['air_token'], spec['last_eps'],
                                  spec['block_size'], device, sampling=sampling)
    tokens = torch.full(tuple(shape), classes, device=device, dtype=torch.int16)
    slot.arm(seed, spec['steps'], ())
    began = time.perf_counter()
    record = None
    while record is None:
        logits = forward(tokens[None], slot.time())[0]
        record, _ = slot.consume(logits, tokens)
    if device.type == 'cuda':
        torch.cuda.synchronize(device)
    result = dict(compact=tokens.cpu().numpy().astype(np.int16), commit_step=record['step_map'].numpy())
    return result, dict(spec=spec, complete=True, remaining=0, nfe=record['nfe'], last_count=record['last_count'],
                        last_frac=record['last_frac'], seconds=time.perf_counter() - began)
