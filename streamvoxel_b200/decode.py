"""Single-column decoding from an all-MASK column: the BASELINE config-1 driver and the evaluation decoders.

`decode` mirrors `streamvoxel/eval/samplers.py:69-115`: the random, entropy, mixed and block baselines (and the
native_quarter threshold schedule) with every schedule of `streamvoxel/sampling/schedule.py`, on libsvx's entropy,
selection (`svx_eval_select`) and categorical-draw kernels; the decoder's random stream is the reference's (one
torch generator on `seed` for the draws and the multinomial noise, the block order on `seed + 9173`), so a decode
equals the reference's given the same logits. `decode_low_entropy_last` restates `samplers.py:118-134`: one slot of
the shipped sampler driven by a model forward until its window finishes (one marking forward, then the solid steps of
the quartercos schedule, the low-entropy-last voxels committed at finish). `UnconditionalForward` is the time-free
DiT-B/4 alone on our engine (`streamvoxel/models/unconditional_md4_timefree.py`), batch 1.
"""
from __future__ import annotations

import math
import time

import numpy as np
import torch

from streamvoxel_b200 import _lib, ops
from streamvoxel_b200.sampling import actual_time, counts, curve
from streamvoxel_b200.stream.fast_ops import FastLowEntropyLastSlot


class UnconditionalForward:
    """Callable (tokens [1, Y, Z, X] int16, timestep) -> logits [1, V, Y, Z, X] bf16 of the time-free model (the
    timestep is accepted for the reference's call shape; the model ignores it)."""

    def __init__(self, cfg, state_dict, device='cuda'):
        from streamvoxel_b200.model import Engine, PreparedModel
        if cfg.layer_indices:
            raise ValueError('UnconditionalForward runs the backbone alone (layer_indices=())')
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


def reveal_fraction(u, schedule):
    """`streamvoxel/sampling/schedule.py:8-12`."""
    if schedule == 'linear':
        return u
    if schedule == 'halfcos':
        return (1 - math.cos(math.pi * u)) / 2
    if schedule == 'reversequarter':
        return math.sin(math.pi * u / 2)
    raise ValueError(schedule)


def schedule_counts(total, spec):
    """`streamvoxel/sampling/schedule.py:15-18,37-43`: per-step reveal counts (None for native_quarter; 'legacy'
    rounding may reveal nothing in a step)."""
    if spec['schedule'] == 'native_quarter':
        return None
    steps = spec['steps']
    if spec.get('rounding') == 'legacy':
        cumulative = [0] + [min(total, max(0, math.floor(total * reveal_fraction(s / steps, spec['schedule']) + 1e-9)))
                            for s in range(1, steps + 1)]
        cumulative[-1] = total
        return [b - a for a, b in zip(cumulative, cumulative[1:])]
    curve(0.5, spec['schedule'])   # unknown schedule names raise ValueError, as the reference does
    return counts(total, steps, spec['schedule'])


def native_probability(s, steps):
    """`streamvoxel/eval/samplers.py:98-100`: the reveal probability of step s of the native quarter schedule."""
    i = steps - s
    if i == 1:
        return 1.
    return (math.sin(math.pi * i / (2 * steps)) - math.sin(math.pi * (i - 1) / (2 * steps))) / \
        math.sin(math.pi * i / (2 * steps))


@torch.inference_mode()
def decode(forward, spec, seed, device, *, shape=(256, 16, 16), classes=304, trace=False):
    """One window from an all-MASK canvas (`streamvoxel/eval/samplers.py:69-115`). `forward(tokens [1, Y, Z, X]
    int16, t) -> logits [1, C, Y, Z, X]` (bf16 or fp32, class-major). Returns (result, meta): result has `compact`
    ([Y, Z, X] int16) and, with `trace`, `commit_step` (0 = never); meta has spec, complete, remaining, nfe,
    seconds, events (per step: step, model_t, committed, remaining and the selection's info)."""
    device = torch.device(device)
    if spec['selection'] == 'low_entropy_last':
        return decode_low_entropy_last(forward, spec, seed, device, shape, classes)
    mode = spec['selection']
    if mode not in ('random', 'entropy', 'mixed', 'block'):
        raise ValueError(mode)
    if mode == 'block' and spec['block_size'] != 4:
        raise ValueError('the selection kernel implements 4^3 blocks')
    if mode == 'mixed':
        c = spec['candidate_multiplier']
        if not math.isfinite(c) or c < 1:
            raise ValueError('candidate multiplier must be finite and >=1')
    _lib.require_device(device)
    shape = tuple(shape)
    total = int(np.prod(shape))
    tokens = torch.full((1, *shape), classes, device=device, dtype=torch.int16)
    rng = torch.Generator(device=device).manual_seed(seed)
    native = spec['schedule'] == 'native_quarter'
    quotas = schedule_counts(total, spec)
    blocks = total // 64
    pos = torch.zeros((1, blocks), dtype=torch.int32, device=device)
    if mode == 'block':
        bg = torch.Generator(device=device).manual_seed(seed + 9173)
        order = torch.randperm(blocks, device=device, generator=bg)
        pos[0, order] = torch.arange(blocks, device=device, dtype=torch.int32)
    commit = torch.zeros((1, *shape), device=device, dtype=torch.int32)
    scores = torch.zeros((1, *shape), device=device, dtype=torch.float32)
    chosen = torch.zeros((1, *shape), device=device, dtype=torch.uint8)
    index = torch.zeros((1, total), device=device, dtype=torch.int32)
    count = torch.zeros(1, device=device, dtype=torch.int32)
    status = torch.zeros(1, device=device, dtype=torch.int32)
    quota_range = torch.zeros((1, 2), device=device, dtype=torch.int32)
    values = torch.zeros((1, total), device=device, dtype=torch.int16)
    events = []
    remaining = total
    began = time.perf_counter()
    for s in range(spec['steps']):
        if remaining == 0:
            break
        t = (spec['steps'] - s) / spec['steps'] if native else actual_time(remaining / total)
        logits = forward(tokens, t)
        draw = torch.rand(shape, device=device, generator=rng)
        status.zero_()
        if mode != 'random':
            ops.ease_scores(logits, status, out=scores)
        info = {}
        if native:
            row = ('threshold', 0, 0, 0, float(np.float32(native_probability(s, spec['steps']))), s + 1)
        else:
            q = min(quotas[s], remaining)
            if mode == 'mixed':
                cand = min(remaining, math.ceil(c * q))
                row = (mode, q, cand, 0, 0., s + 1)
                info = dict(candidate_count=cand, candidate_multiplier=c)
            elif mode == 'block':
                row = (mode, q, 0, total - remaining, 0., s + 1)
            else:
                row = (mode, q, 0, 0, 0., s + 1)
        ops.eval_select(scores, draw[None], tokens, pos, ops.eval_params([row], device), classes, chosen=chosen,
                        index=index, count=count, commit_step=commit, quota_range=quota_range, status=status)
        k = int(count.item())
        if int(status.item()) & _lib.STATUS_QUOTA_MISSED:
            raise AssertionError(f'{mode} selection did not meet its quota at step {s + 1}')
        if mode == 'block' and not native:
            low, high = quota_range[0].tolist()
            info = dict(block_size=4, global_cumulative_target=total - remaining + q, per_block_quota_min=low,
                        per_block_quota_max=high)
        if k:
            # The exponential draws torch.multinomial(probabilities, 1, generator) makes (`samplers.py:108`).
            noise = torch.empty((1, k, classes), device=device).exponential_(generator=rng)
            ops.ease_sample(logits, index, ops.step_params([(k, s + 1, 0, 0., seed)], device), tokens, noise=noise,
                            values=values, status=status)
        remaining -= k
        events.append(dict(step=s + 1, model_t=t, committed=k, remaining=remaining, **info))
    if device.type == 'cuda':
        torch.cuda.synchronize(device)
    result = dict(compact=tokens[0].cpu().numpy().astype(np.int16))
    if trace:
        result['commit_step'] = commit[0].cpu().numpy()
    return result, dict(spec=spec, complete=remaining == 0, remaining=remaining, nfe=len(events),
                        seconds=time.perf_counter() - began, events=events)
