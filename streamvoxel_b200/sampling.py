"""Host-side EASE schedule: quartercos quota counts, the low-entropy-last quota list and the model time.

Pure Python integer/float64 arithmetic, identical to the reference:
`streamvoxel/sampling/schedule.py:4-38` and `streamvoxel/sampling/low_entropy_last.py:20-33`.
"""
from __future__ import annotations

import math


def actual_time(mask_fraction):
    """`streamvoxel/sampling/schedule.py:4-5`."""
    return 2 * math.asin(min(1., max(0., mask_fraction))) / math.pi


def curve(u, name):
    """`streamvoxel/sampling/schedule.py:17-25`."""
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
    """`streamvoxel/sampling/schedule.py:28-34` (rounding 'positive'): per-step reveal counts summing to total."""
    if not 1 <= steps <= total:
        raise ValueError((total, steps))
    cumulative = [0] + [s + math.floor((total - steps) * curve(s / steps, schedule) + 1e-10) for s in range(1, steps + 1)]
    cumulative[-1] = total
    q = [b - a for a, b in zip(cumulative, cumulative[1:])]
    assert min(q) >= 1 and sum(q) == total
    return q


def low_entropy_last_quotas(total, steps, n_last, schedule='quartercos'):
    """`streamvoxel/sampling/low_entropy_last.py:20-33`: the schedule with n_last voxels removed from its tail,
    positive quotas only (their sum is total - n_last)."""
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
