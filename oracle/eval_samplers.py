"""Evaluation decoders restated in numpy (TEST INFRASTRUCTURE ONLY; see `oracle/__init__.py`).

Follows `streamvoxel/eval/samplers.py` (random, entropy, mixed and block selections, the native_quarter threshold)
and the schedules of `streamvoxel/sampling/schedule.py`. The decoder's random stream is an input: `draw()` returns
the step's `torch.rand(shape, generator)` values and `noise(k, classes)` the exponential noise behind
`torch.multinomial(p, 1, generator)` (`argmax(p / q)`, see `oracle/sampler.py`), in the order the reference calls
them; the block order (`torch.randperm`) is an input too.
"""
from __future__ import annotations

import math

import numpy as np

from oracle.sampler import actual_time, block_unview, block_view, categorical_from_noise, counts, entropy_scores, \
    softmax0, top_mask, _descending_stable


def reveal_fraction(u, schedule):
    """`streamvoxel/sampling/schedule.py:8-12`."""
    if schedule == 'linear':
        return u
    if schedule == 'halfcos':
        return (1 - math.cos(math.pi * u)) / 2
    if schedule == 'reversequarter':
        return math.sin(math.pi * u / 2)
    raise ValueError(schedule)


def quota_counts(total, steps, schedule):
    """`streamvoxel/sampling/schedule.py:15-18` (rounding 'legacy': steps may reveal nothing)."""
    cumulative = [0] + [min(total, max(0, math.floor(total * reveal_fraction(s / steps, schedule) + 1e-9)))
                        for s in range(1, steps + 1)]
    cumulative[-1] = total
    return [b - a for a, b in zip(cumulative, cumulative[1:])]


def schedule_counts(total, spec):
    """`streamvoxel/sampling/schedule.py:37-43`: None for native_quarter."""
    if spec['schedule'] == 'native_quarter':
        return None
    if spec.get('rounding') == 'legacy':
        return quota_counts(total, spec['steps'], spec['schedule'])
    return counts(total, spec['steps'], spec['schedule'])


def native_probability(s, steps):
    """`streamvoxel/eval/samplers.py:98-100`: the reveal probability of step s of the 1024-step reference."""
    i = steps - s
    if i == 1:
        return 1.
    return (math.sin(math.pi * i / (2 * steps)) - math.sin(math.pi * (i - 1) / (2 * steps))) / \
        math.sin(math.pi * i / (2 * steps))


def mixed_select(score, mask, position_draw, k, c):
    """`streamvoxel/eval/samplers.py:23-28`."""
    if not math.isfinite(c) or c < 1:
        raise ValueError('candidate multiplier must be finite and >=1')
    candidate_count = min(int(mask.sum()), math.ceil(c * k))
    candidates = top_mask(position_draw, mask, candidate_count)
    return top_mask(score, candidates, k), dict(candidate_count=candidate_count, candidate_multiplier=c)


def block_select(score, mask, k, b, order, committed_before):
    """`streamvoxel/eval/samplers.py:31-48`: the global cumulative count apportioned linearly over equal blocks (the
    first `rem` blocks of the seeded order take one more), the lowest-entropy masked voxels of each block."""
    mb = block_view(mask, b)
    nb = len(order)
    after = committed_before + k
    q, rem = divmod(after, nb)
    target = np.full(nb, q, np.int64)
    target[np.asarray(order)[:rem]] += 1
    already = (~mb).sum(1)
    quota = target - already
    legal = mb.sum(1)
    assert (quota >= 0).all() and (quota <= legal).all() and int(quota.sum()) == k
    sm = np.where(mb, block_view(score, b), -np.inf)
    bc = np.zeros_like(mb)
    for j in range(nb):
        bc[j, _descending_stable(sm[j])[:quota[j]]] = True
    chosen = block_unview(bc, mask.shape, b)
    assert int(chosen.sum()) == k and not (chosen & ~mask).any()
    return chosen, dict(block_size=b, global_cumulative_target=after, per_block_quota_min=int(quota.min()),
                        per_block_quota_max=int(quota.max()))


def choose(score, mask, draw, q, spec, order=None, committed=0):
    """`streamvoxel/eval/samplers.py:51-66`."""
    mode = spec['selection']
    q = min(q, int(mask.sum()))
    info = {}
    if mode == 'random':
        chosen = top_mask(draw, mask, q)
    elif mode == 'entropy':
        chosen = top_mask(score, mask, q)
    elif mode == 'mixed':
        chosen, info = mixed_select(score, mask, draw, q, spec['candidate_multiplier'])
    elif mode == 'block':
        chosen, info = block_select(score, mask, q, spec['block_size'], order, committed)
    else:
        raise ValueError(mode)
    assert not (chosen & ~mask).any()
    return chosen, info


def decode(forward, spec, draw, noise, *, order=None, shape=(256, 16, 16), classes=304, score_fn=None):
    """`streamvoxel/eval/samplers.py:69-115` from an all-MASK canvas: `forward(tokens[Y,Z,X] int64, t)` returns
    fp32 logits [C, Y, Z, X]; `order` is the block order (`torch.randperm` on seed + 9173) for block selection;
    `score_fn` overrides the entropy (test feed). Returns (tokens, commit_step, events)."""
    tokens = np.full(shape, classes, np.int64)
    total = tokens.size
    native = spec['schedule'] == 'native_quarter'
    quotas = schedule_counts(total, spec)
    commit = np.zeros(shape, np.int32)
    events = []
    remaining = total
    for s in range(spec['steps']):
        if remaining == 0:
            break
        mask = tokens == classes
        t = (spec['steps'] - s) / spec['steps'] if native else actual_time(remaining / total)
        logits = np.asarray(forward(tokens, t), np.float32)
        d = np.asarray(draw(), np.float32)
        score = None
        if spec['selection'] != 'random':
            score = entropy_scores(logits) if score_fn is None else np.asarray(score_fn(logits), np.float32)
        if native:
            p = np.float32(native_probability(s, spec['steps']))
            chosen, info = mask & (d < p), {}
        else:
            chosen, info = choose(score, mask, d, quotas[s], spec, order=order, committed=total - remaining)
        k = int(chosen.sum())
        if k:
            positions = np.flatnonzero(chosen)
            columns = logits.reshape(classes, -1)[:, positions]
            values = categorical_from_noise(softmax0(columns).T, noise(k, classes))
            tokens.reshape(-1)[positions] = values
            commit.reshape(-1)[positions] = s + 1
        remaining -= k
        events.append(dict(step=s + 1, model_t=t, committed=k, remaining=remaining, **info))
    return tokens, commit, events
