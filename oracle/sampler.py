"""EASE sampler restated in numpy (TEST INFRASTRUCTURE ONLY; see `oracle/__init__.py`).

Every function follows one reference function; the citation is `path:line` in zzf1955/StreamVoxel. Index and
integer work is exact (int64 / float64 where the reference uses them); floating point follows the reference's
precision (fp32 log-softmax and softmax, fp64 apportioning).

Third-party arithmetic the reference relies on (torch 2.11.0): `torch.randperm` (block order) and the generator
stream behind `torch.multinomial`. Neither is restated: the block order is an input (`order`), and the categorical
draw takes its exponential noise `q` as an input, using the identity `multinomial(p, 1) == argmax(p / q)` with
`q = empty_like(p).exponential_(generator)` that torch's multinomial uses for a single draw
(checked against the reference by `tests/golden/make_golden.py`).
"""
from __future__ import annotations

import math

import numpy as np

# ----------------------------------------------------------------------------------------------- schedule

def curve(u, name):
    """`streamvoxel/sampling/schedule.py:17-25` (quartercos and the other named reveal curves)."""
    if name == 'linear':
        return u
    if name == 'quartercos':
        return 1 - math.cos(math.pi * u / 2)
    if name == 'reversequarter':
        return math.sin(math.pi * u / 2)
    if name == 'halfcos':
        return (1 - math.cos(math.pi * u)) / 2
    if name == 'arccos':
        return 2 / math.pi * math.acos(1 - u)
    if name.startswith('front'):
        return 1 - (1 - u) ** float(name[5:])
    if name.startswith('power'):
        return u ** float(name[5:])
    raise ValueError(name)


def counts(total, steps, schedule='quartercos'):
    """`streamvoxel/sampling/schedule.py:28-34` with rounding='positive': every step reveals at least one voxel."""
    if not 1 <= steps <= total:
        raise ValueError((total, steps))
    cumulative = [0] + [s + math.floor((total - steps) * curve(s / steps, schedule) + 1e-10) for s in range(1, steps + 1)]
    cumulative[-1] = total
    q = [b - a for a, b in zip(cumulative, cumulative[1:])]
    assert min(q) >= 1 and sum(q) == total
    return q


def actual_time(mask_fraction):
    """`streamvoxel/sampling/schedule.py:4-5`."""
    return 2 * math.asin(min(1., max(0., mask_fraction))) / math.pi


def low_entropy_last_quotas(total, steps, n_last, schedule='quartercos'):
    """`streamvoxel/sampling/low_entropy_last.py:20-33`: the deferred voxels are taken from the schedule's tail."""
    n_last = int(n_last)
    if steps < 1 or not 0 <= n_last <= total:
        raise ValueError((total, steps, n_last))
    quotas = counts(total, int(steps), schedule)
    air, solid = n_last, []
    for q in reversed(quotas):
        take = min(q, air)
        air -= take
        solid.append(q - take)
    solid.reverse()
    assert air == 0 and sum(solid) == total - n_last
    return [q for q in solid if q > 0]


# ------------------------------------------------------------------------------------------------ scores

def log_softmax0(logits):
    """fp32 log-softmax over axis 0 (the class axis), as `Tensor.log_softmax(0)` in fp32."""
    x = np.asarray(logits, np.float32)
    m = x.max(0)
    shifted = x - m
    return shifted - np.log(np.exp(shifted).sum(0, dtype=np.float32))


def entropy_scores(logits):
    """`streamvoxel/sampling/entropy.py:1-4`: negative Shannon entropy per voxel (nats), fp32. logits [C, ...]."""
    logp = log_softmax0(logits)
    return (np.exp(logp) * logp).sum(0, dtype=np.float32)


def softmax0(logits):
    """fp32 softmax over axis 0, as `Tensor.softmax(0)` in fp32."""
    x = np.asarray(logits, np.float32)
    e = np.exp(x - x.max(0))
    return e / e.sum(0, dtype=np.float32)


def air_probability(logits, air_ids):
    """`streamvoxel/stream/slot.py:126`: `softmax(0)[air].sum(0)` in fp32."""
    p = softmax0(logits)
    return p[list(air_ids)].sum(0, dtype=np.float32)


# ----------------------------------------------------------------------------------------------- selection

def block_view(a, b):
    """`streamvoxel/sampling/block_quota.py:15-17`: [Y,Z,X] -> [blocks, b^3], blocks in YZX order, offsets YZX."""
    y, z, x = a.shape
    return a.reshape(y // b, b, z // b, b, x // b, b).transpose(0, 2, 4, 1, 3, 5).reshape(-1, b ** 3)


def block_unview(a, shape, b):
    """Inverse of `block_view` (the reshape/permute at `block_quota.py:33`)."""
    y, z, x = shape
    return a.reshape(y // b, z // b, x // b, b, b, b).transpose(0, 3, 1, 4, 2, 5).reshape(shape)


def _descending_stable(values):
    """Indices of `values` sorted high to low; equal values keep their index order (`argsort(stable=True)`)."""
    return np.argsort(-np.asarray(values), kind='stable')


def top_mask(scores, eligible, count):
    """`streamvoxel/sampling/block_quota.py:4-12`: the `count` best eligible scores, ties to the lower YZX index."""
    result = np.zeros(eligible.shape, bool)
    indices = np.flatnonzero(eligible)
    count = min(int(count), len(indices))
    if count > 0:
        order = _descending_stable(scores.reshape(-1)[indices])
        result.reshape(-1)[indices[order[:count]]] = True
    return result


def block_targets(mask, b, pos, frac, n_total, goal):
    """The per-block quota of `block_quota_select` (`streamvoxel/sampling/block_quota.py:24-30`).

    `pos` is the inverse block order, `goal` = already-committed non-deferred voxels + k."""
    mb = block_view(mask, b)
    nbk = mb.shape[0]
    legal = mb.sum(1).astype(np.int64)
    n_total = np.asarray(n_total, np.int64)
    already = n_total - legal
    ideal = float(frac) * n_total.astype(np.float64)
    base = np.floor(ideal + 1e-9).astype(np.int64)
    extra = max(int(goal) - int(base.sum()), 0)
    key = -(ideal - base.astype(np.float64)) * 1e6 + np.asarray(pos, np.float64)
    frac_rank = np.argsort(key, kind='stable')
    target = base.copy()
    target[frac_rank[:extra]] += 1
    quota = np.minimum(np.maximum(target - already, 0), legal)
    assert quota.shape == (nbk,)
    return quota


def block_quota_select(score, mask, k, b, order, frac, n_total):
    """`streamvoxel/sampling/block_quota.py:20-38`: exactly k voxels of `mask`, balanced over b^3 blocks.

    order: the seeded block permutation; frac: target committed fraction after this step (float64)."""
    score = np.asarray(score, np.float32)
    mask = np.asarray(mask, bool)
    order = np.asarray(order, np.int64)
    mb = block_view(mask, b)
    legal = mb.sum(1).astype(np.int64)
    already = np.asarray(n_total, np.int64) - legal
    pos = np.empty_like(order)
    pos[order] = np.arange(len(order))
    quota = block_targets(mask, b, pos, frac, n_total, int(already.sum()) + int(k))
    sm = np.where(mb, block_view(score, b), np.float32(-np.inf))
    ranks = np.argsort(-sm, axis=1, kind='stable')
    bc = np.zeros(mb.shape, bool)
    rows = np.arange(mb.shape[0])[:, None]
    bc[rows, ranks] = np.arange(b ** 3)[None, :] < quota[:, None]
    sel = block_unview(bc, mask.shape, b) & mask
    got = int(sel.sum())
    if got > k:
        sel = top_mask(score, sel, k)
    elif got < k:
        sel = sel | top_mask(score, mask & ~sel, k - got)
    return sel


def low_entropy_last_update(last, mask, air, solid, eps, band=False, col=False):
    """`streamvoxel/sampling/low_entropy_last.py:8-17`. The threshold is compared in fp32 (torch casts the Python
    float to the fp32 tensor's dtype)."""
    bad = (mask & (np.asarray(air, np.float32) <= np.float32(1 - eps))) | solid
    if col:
        run = np.flip(np.cumprod(np.flip(~bad, 0).astype(np.int64), 0), 0).astype(bool)
        return last | run
    clean = ~bad.reshape(bad.shape[0], -1).any(1)
    if band:
        clean = np.repeat(clean.reshape(-1, 8).all(1), 8)
    top_run = np.flip(np.cumprod(np.flip(clean, 0).astype(np.int64), 0), 0).astype(bool)
    return last | top_run[:, None, None]


# ------------------------------------------------------------------------------------------------- sampling

def categorical_from_noise(probabilities, q):
    """`torch.multinomial(p, 1)` for one draw per row (`streamvoxel/stream/slot.py:150`) given its exponential
    noise q: `argmax(p / q)`, the first index among equal maxima. fp32 division."""
    ratio = np.asarray(probabilities, np.float32) / np.asarray(q, np.float32)
    return ratio.argmax(-1).astype(np.int64)


PHILOX_M0, PHILOX_M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
PHILOX_W0, PHILOX_W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
NATIVE_STREAM = 0x53564F58  # counter word 3 of the native draw


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011):
    ten rounds of two 32x32->64 multiplies, key bumped by the Weyl constants between rounds. Vectorised."""
    c = [np.asarray(v, np.uint32).copy() for v in (c0, c1, c2, c3)]
    k = [np.asarray(k0, np.uint32).copy(), np.asarray(k1, np.uint32).copy()]
    mask = np.uint64(0xFFFFFFFF)
    with np.errstate(over='ignore'):
        for r in range(10):
            if r:
                k[0] = (k[0] + PHILOX_W0).astype(np.uint32)
                k[1] = (k[1] + PHILOX_W1).astype(np.uint32)
            p0 = PHILOX_M0 * c[0].astype(np.uint64)
            p1 = PHILOX_M1 * c[2].astype(np.uint64)
            hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & mask).astype(np.uint32)
            hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & mask).astype(np.uint32)
            c = [hi1 ^ c[1] ^ k[0], lo1, hi0 ^ c[3] ^ k[1], lo0]
    return c


def native_uniforms(seed, step, voxels, classes):
    """Uniforms in (0,1) of the native draw for `voxels` (flat YZX indexes) x `classes`, float32 [n, classes].

    Counter (class // 4, voxel, step, NATIVE_STREAM), key (seed low, seed high); output word class % 4;
    u = (2 (word >> 9) + 1) * 2^-24: odd multiples of 2^-24, exactly representable in fp32, never 0 or 1."""
    voxels = np.asarray(voxels, np.int64)
    groups = (classes + 3) // 4
    g = np.arange(groups, dtype=np.uint32)[None, :]
    n = voxels.astype(np.uint32)[:, None]
    seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    words = philox4x32_10(np.broadcast_to(g, (len(voxels), groups)), np.broadcast_to(n, (len(voxels), groups)),
                          np.full((len(voxels), groups), step & 0xFFFFFFFF, np.uint32),
                          np.full((len(voxels), groups), NATIVE_STREAM, np.uint32),
                          np.uint32(seed & 0xFFFFFFFF), np.uint32(seed >> 32))
    stacked = np.stack(words, -1).reshape(len(voxels), groups * 4)[:, :classes]
    odd = ((stacked >> np.uint32(9)) << np.uint32(1)) | np.uint32(1)
    return (odd.astype(np.float32) * np.float32(2.0 ** -24)).astype(np.float32)


# 1/11, 1/9, 1/7, 1/5, 1/3 and ln 2 rounded to the nearest fp32 value (the kernel writes the same hexadecimal literals)
_SERIES = [np.float32(float.fromhex(h)) for h in ('0x1.745d18p-4', '0x1.c71c72p-4', '0x1.24924ap-3', '0x1.99999ap-3',
                                                  '0x1.555556p-2')]
_LN2 = np.float32(float.fromhex('0x1.62e430p-1'))


def series_log(a):
    """Natural log of positive normal fp32 values by the atanh series, with exactly the fp32 operations of the native
    draw kernel's `series_log`: a = m 2^e with m in [sqrt(1/2), sqrt(2)), s = (m - 1) / (m + 1), z = s^2,
    log a = e ln 2 + 2 s (1 + z (1/3 + z (1/5 + z (1/7 + z (1/9 + z/11))))), each operation rounded once to fp32."""
    a = np.asarray(a, np.float32)
    bits = a.view(np.int32)
    e = (bits >> 23) - 127
    mbits = (bits & 0x007FFFFF) | 0x3F800000
    high = mbits > 0x3FB504F3
    mbits = np.where(high, mbits - 0x00800000, mbits).astype(np.int32)
    e = np.where(high, e + 1, e)
    m = mbits.view(np.float32)
    one = np.float32(1)
    s = (m - one) / (m + one)
    z = s * s
    t = _SERIES[0]
    for c in _SERIES[1:]:
        t = c + z * t
    t = one + z * t
    return (e.astype(np.float32) * _LN2 + (np.float32(2) * s) * t).astype(np.float32)


def native_sample(logits_cn, voxels, seed, step):
    """Native (graph-capturable) draw, Gumbel-max: argmax_v x_v - log(-log u_v) with `series_log` for both logs and
    one fp32 subtraction, ties to the lower class; distributed as `multinomial(softmax(x), 1)`. Bit-exact with the
    kernel given the same fp32 logits. logits_cn is [C, n] for the voxels."""
    x = np.asarray(logits_cn, np.float32).T
    u = native_uniforms(seed, step, voxels, x.shape[1])
    key = (x - series_log(-series_log(u))).astype(np.float32)
    return key.argmax(1).astype(np.int64)


# ------------------------------------------------------------------------------------------------ the slot

class Slot:
    """`streamvoxel/stream/slot.py:50-176` (`LowEntropyLastSlot`) with the torch RNG made explicit.

    `arm(..., order=)` takes the block permutation the reference draws with `randperm(Generator(seed + 9173))`.
    `consume(..., noise=)` takes `noise(k, C) -> q[k, C]`, the exponential draws `torch.multinomial` would take from
    the slot generator (`slot.py:150`), or `native=True` for the Philox draw of `native_sample`.
    """

    def __init__(self, shape, classes, air_ids, air_token, last_eps, block_size):
        self.shape = tuple(shape)
        self.total = int(np.prod(self.shape))
        self.classes = int(classes)
        self.air_ids = tuple(air_ids)
        self.air_token = int(air_token)
        self.last_eps = float(last_eps)
        self.block_size = int(block_size)
        self.phase = 'idle'

    @property
    def idle(self):
        return self.phase == 'idle'

    def arm(self, seed, cap, target, order):
        """`slot.py:86-103`."""
        self.phase = 'marking'
        self.seed, self.cap, self.target = int(seed), int(cap), tuple(target)
        self.nfe = self.actual = self.solid_calls = 0
        self.quotas = None
        self.last_count = 0
        self.last = np.zeros(self.shape, bool)
        self.order = np.asarray(order, np.int64)
        self.step_map = np.zeros(self.shape, np.int16)
        self.values = np.full(self.shape, -1, np.int16)

    def time(self):
        """`slot.py:110-115`."""
        if self.phase == 'idle':
            return 1.0
        committed = sum(self.quotas[:self.solid_calls]) if self.quotas else 0
        return actual_time((self.total - committed) / self.total)

    def mark(self, logits, air=None):
        """Marking forward, `slot.py:124-136`; `air` overrides the air probability (a test feed of the reference's
        `softmax(0)[air].sum(0)` computed elsewhere)."""
        self.nfe += 1
        air = air_probability(logits, self.air_ids) if air is None else np.asarray(air, np.float32)
        ones = np.ones(self.shape, bool)
        self.last = low_entropy_last_update(self.last, ones, air, ~ones, self.last_eps, False, True)
        self.last_count = int(self.last.sum())
        self.quotas = low_entropy_last_quotas(self.total, self.cap, self.last_count, 'quartercos')
        self.phase = 'solid'
        self.solid_calls = 0

    def select(self, logits, tokens, scores=None):
        """The selection half of a solid step (`slot.py:139-148`); `scores` overrides the entropy (test feed)."""
        k = self.quotas[self.solid_calls]
        selectable = (tokens == self.classes) & ~self.last
        committed = sum(self.quotas[:self.solid_calls])
        frac = (committed + k) / (self.total - self.last_count)
        n_total = block_view(~self.last, self.block_size).sum(1)
        score = entropy_scores(logits) if scores is None else scores
        chosen = block_quota_select(score, selectable, k, self.block_size, self.order, frac, n_total)
        if int(chosen.sum()) != k or (chosen & ~selectable).any():
            raise AssertionError('low-entropy-last solid step did not meet its quota')
        return chosen

    def consume(self, logits, tokens, noise=None, native=False, scores=None, air=None, draw=None):
        """One forward (`slot.py:117-164`); `tokens` [Y,Z,X] is updated in place. Returns (record|None, commit|None).

        Test feeds: `scores` (the entropy), `air` (the marking probability), and `draw(positions) -> values`, which
        replaces the categorical draw (for instance the reference's own `torch.multinomial` call on the device that
        holds the logits and the slot generator); `logits` may then be None for solid steps."""
        if self.phase == 'idle':
            return None, None
        if self.phase == 'marking':
            self.mark(logits, air)
            if not self.quotas:
                return self._finish(tokens), None
            return None, None
        if self.solid_calls >= len(self.quotas):
            return self._finish(tokens), None
        chosen = self.select(logits, tokens, scores)
        positions = np.flatnonzero(chosen)
        if draw is not None:
            values = np.asarray(draw(positions), np.int64)
        elif native:
            columns = np.asarray(logits, np.float32).reshape(self.classes, -1)[:, positions]
            values = native_sample(columns, positions, self.seed, self.nfe + 1)
        else:
            columns = np.asarray(logits, np.float32).reshape(self.classes, -1)[:, positions]
            q = noise(len(positions), self.classes)
            values = categorical_from_noise(softmax0(columns).T, q)
        tokens.reshape(-1)[positions] = values
        self.solid_calls += 1
        self.actual += 1
        self.nfe += 1
        self.step_map.reshape(-1)[positions] = self.nfe
        self.values.reshape(-1)[positions] = values.astype(np.int16)
        commit = dict(positions=positions.astype(np.int32), values=values.astype(np.int16), step=int(self.nfe))
        if self.solid_calls >= len(self.quotas):
            return self._finish(tokens), commit
        return None, commit

    def _finish(self, tokens):
        """`slot.py:166-176`."""
        tokens[self.last] = self.air_token
        self.step_map[self.last] = self.nfe
        self.values[self.last] = self.air_token
        record = dict(target=self.target, seed=self.seed, cap=self.cap, nfe=int(self.nfe), actual=int(self.actual),
                      last_count=int(self.last_count), last_frac=float(self.last_count) / self.total,
                      step_map=self.step_map.copy(), values=self.values.copy())
        self.phase = 'idle'
        self.target = None
        return record
