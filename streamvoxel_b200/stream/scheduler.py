"""Window admission for a world expansion, and the split of the slot batch over GPUs.

The rules of the reference (`streamvoxel/stream/scheduler.py:1-151`, `streamvoxel/common/colored_frontier.py:97-106`):
a candidate window is an uncommitted cell with at least one committed 8-neighbour, it must not be in flight and must
keep Chebyshev distance >= 2 from every in-flight window (Manhattan >= 2 with `diagonal`), and the nearest such cell
to the player wins (ties on (z, x)). Conditions come only from the committed snapshot. With these rules windows in
flight never condition on each other, so GPUs sample independent windows and only committed columns are exchanged.
"""
from __future__ import annotations

import hashlib

import numpy as np

from .condition import Item

BIOME_PERIOD = 64   # biome quarts per world side (labels repeat), the biome array carries a one-quart halo


def ready_cells(committed):
    """Uncommitted cells with at least one committed 8-neighbour (`colored_frontier.py:97-106`)."""
    ready = set()
    for z, x in committed:
        for a in (z - 1, z, z + 1):
            for b in (x - 1, x, x + 1):
                if (a, b) not in committed:
                    ready.add((a, b))
    return ready


def chebyshev(a, b):
    return max(abs(a[0] - b[0]), abs(a[1] - b[1]))


def separated(cell, others, gap=2, diagonal=False):
    """`scheduler.py:37-40`: Chebyshev distance >= gap to every other cell; with `diagonal`, Manhattan >= 2."""
    if diagonal:
        return all(abs(cell[0] - o[0]) + abs(cell[1] - o[1]) >= 2 for o in others)
    return all(chebyshev(cell, o) >= gap for o in others)


def rank_share(batch, ranks, rank):
    """`scheduler.py:43-48`: equal split of a global batch, the remainder to the first ranks."""
    batch, ranks = max(0, int(batch)), max(1, int(ranks))
    base, extra = divmod(batch, ranks)
    return base + (1 if int(rank) < extra else 0)


def plan_inserts(idle_indexes, active_count, batch, mode):
    """`scheduler.py:51-64`: idle slots that may start a window now ('dynamic' refills, 'fixed' waits for all)."""
    batch = max(0, int(batch))
    idle = list(idle_indexes)
    if mode == 'fixed':
        return [] if active_count else idle[:batch]
    return idle[:max(0, batch - int(active_count))]


def pick_window(committed, inflight, player_zx, *, cell_size=16, diagonal=False):
    """`scheduler.py:66-79`: the nearest admissible cell to the player, or None when the frontier is blocked."""
    pz, px = player_zx
    blocked = set(inflight)
    best_key, best = None, None
    for cell in ready_cells(committed):
        if cell in blocked or not separated(cell, blocked, diagonal=diagonal):
            continue
        z, x = cell
        key = (((z + .5) * cell_size - pz) ** 2 + ((x + .5) * cell_size - px) ** 2, z, x)
        if best_key is None or key < best_key:
            best_key, best = key, cell
    return best


def member_shares(batch, members):
    """`scheduler.py:126-151`: split `batch` over `[(wid, capacity, weight)]` by weight (integer largest remainder,
    ties to the smaller wid), then clamp to capacity and hand the excess to the members with room, in wid order."""
    batch = max(0, int(batch))
    if not members:
        return {}
    total = sum(w for _, _, w in members)
    numer = {wid: batch * w for wid, _, w in members}
    share = {wid: numer[wid] // total for wid, _, _ in members}
    left = batch - sum(share.values())
    for wid, _, _ in sorted(members, key=lambda m: (-(numer[m[0]] % total), m[0]))[:left]:
        share[wid] += 1
    excess = 0
    for wid, cap, _ in members:
        if share[wid] > cap:
            excess += share[wid] - cap
            share[wid] = cap
    for wid, cap, _ in members:
        moved = min(excess, cap - share[wid])
        share[wid] += moved
        excess -= moved
    return share


def window_seed(world, z, x):
    """The window's sampler seed (`scheduler.py:31-32`): the first 8 bytes (little endian) of
    sha256('player-frontier-v1:{world}:{z}:{x}') modulo 2^63 - 1, so every rank derives the same seed."""
    digest = hashlib.sha256(f'player-frontier-v1:{world}:{z}:{x}'.encode()).digest()
    return int.from_bytes(digest[:8], 'little') % (2 ** 63 - 1)


def tiled_biome_crop(biomes, z, x):
    """`scheduler.py:19-27`: the 6x6-quart crop (one-quart halo) of cell (z, x), wrapping with the label period."""
    zi = (np.arange(4 * z - 1, 4 * z + 5) % BIOME_PERIOD) + 1
    xi = (np.arange(4 * x - 1, 4 * x + 5) % BIOME_PERIOD) + 1
    return biomes[:, zi][:, :, xi]


def biome_volume(biomes, z, x, spec):
    """`scheduler.py:86-100`: the halo crop centred in the 12x12 biome tensor the condition encoder reads."""
    if spec.biome_halo == 4:
        crop = tiled_biome_crop(biomes, z, x)
    else:
        pad = spec.biome_halo // 4
        zi = (np.arange(4 * z - pad, 4 * z + 4 + pad) % BIOME_PERIOD) + 1
        xi = (np.arange(4 * x - pad, 4 * x + 4 + pad) % BIOME_PERIOD) + 1
        crop = biomes[:, zi][:, :, xi]
    if crop.shape != spec.biome_shape:
        raise ValueError(f'Biome crop {crop.shape} != {spec.biome_shape}')
    out = np.zeros((spec.height // 4, 12, 12), np.int64)
    lo = (12 - crop.shape[1]) // 2
    out[:, lo:lo + crop.shape[1], lo:lo + crop.shape[2]] = crop.astype(np.int64)
    return out


def nearest_cells(cells, target, count):
    """The `count` committed cells nearest to `target` by (squared distance, cell), as `make_item` picks its L2 tiles
    (`scheduler.py:114`), found by growing a square around the target instead of sorting the whole snapshot: once
    the square of radius r holds at least `count` cells within distance r, every cell at or below the count-th
    distance lies inside it (ties included), so sorting the square's cells gives the same answer."""
    z, x = target
    total = len(cells)
    r = max(1, int((count / 3.0) ** 0.5))
    while True:
        box = [(a, b) for a in range(z - r, z + r + 1) for b in range(x - r, x + r + 1) if (a, b) in cells]
        within = sum(1 for a, b in box if (a - z) ** 2 + (b - x) ** 2 <= r * r)
        if within >= count or len(box) == total:
            box.sort(key=lambda c: ((c[0] - z) ** 2 + (c[1] - x) ** 2, c))
            return box[:count]
        r += 1


class ColumnStack:
    """The L2 tiles of an item as a lazy stack over the committed snapshot: `len`, fancy indexing (`stack[[i, j]]`)
    and `np.asarray` give what the stacked [n, H, T, T] array would, but only the columns asked for are copied (the
    encoder asks only for columns its L2 cache has not seen)."""

    def __init__(self, cells, keys, shape):
        self.cells, self.keys, self.shape_one = cells, list(keys), tuple(shape)

    def __len__(self):
        return len(self.keys)

    @property
    def shape(self):
        return (len(self.keys),) + self.shape_one

    def __getitem__(self, index):
        picks = np.arange(len(self.keys))[index]
        if np.ndim(picks) == 0:
            return np.asarray(self.cells[self.keys[int(picks)]], np.int16)
        if len(picks) == 0:
            return np.zeros((0,) + self.shape_one, np.int16)
        return np.stack([np.asarray(self.cells[self.keys[int(i)]], np.int16) for i in picks])

    def __array__(self, dtype=None, copy=None):
        out = self[np.arange(len(self.keys))]
        return out if dtype is None else out.astype(dtype)


def fast_item(cells, target, biomes, spec, world, cap, l2_cap):
    """`make_item` with the same result for a driver that builds an item per window from a large snapshot: the L2
    cells by `nearest_cells` and the L2 tiles as a `ColumnStack` (the L1 tiles, positions, seed and biome crop are
    built exactly as `make_item` builds them)."""
    z, x = target
    if target in cells:
        raise ValueError('Target already committed')
    near = sorted((a, b) for a in (z - 1, z, z + 1) for b in (x - 1, x, x + 1) if (a, b) != target and (a, b) in cells)
    if not near:
        raise ValueError('Target has no committed neighbor')
    far = sorted(nearest_cells(cells, target, l2_cap))
    shape = (spec.height, spec.tile, spec.tile)
    l1 = np.stack([np.asarray(cells[c], np.int16) for c in near])
    if l1.shape[1:] != shape:
        raise ValueError('Condition tile has the wrong shape')
    return Item(id=f'{z}_{x}', seed=window_seed(world, z, x), steps=int(cap), temperature=1.0,
                l1_blocks=l1, l1_xz=_relative_xz(near, z, x), l2_blocks=ColumnStack(cells, far, shape),
                l2_xz=_relative_xz(far, z, x), biomes=biome_volume(biomes, z, x, spec), known=None,
                l2_keys=[(world,) + c for c in far])


def _relative_xz(cells, z, x):
    return np.asarray([[(b - x) * 16, (a - z) * 16] for a, b in cells], np.int64).reshape(-1, 2)


def make_item(cells, target, biomes, spec, world, cap, l2_cap):
    """`scheduler.py:103-123`: the `Item` of window `target` from the committed snapshot `cells` ({(z, x): tokens}):
    committed 8-neighbours as L1 tiles (sorted by cell), the `l2_cap` nearest committed cells as L2 tiles (nearest by
    squared distance then cell, listed sorted by cell), the biome crop; XZ relative to the target in voxels."""
    z, x = target
    if target in cells:
        raise ValueError('Target already committed')
    near = sorted((a, b) for a in (z - 1, z, z + 1) for b in (x - 1, x, x + 1) if (a, b) != target and (a, b) in cells)
    if not near:
        raise ValueError('Target has no committed neighbor')
    far = sorted(sorted(cells, key=lambda c: ((c[0] - z) ** 2 + (c[1] - x) ** 2, c))[:l2_cap])
    shape = (spec.height, spec.tile, spec.tile)
    l1 = np.stack([np.asarray(cells[c], np.int16) for c in near])
    l2 = np.stack([np.asarray(cells[c], np.int16) for c in far])
    if l1.shape[1:] != shape or l2.shape[1:] != shape:
        raise ValueError('Condition tile has the wrong shape')
    return Item(id=f'{z}_{x}', seed=window_seed(world, z, x), steps=int(cap), temperature=1.0,
                l1_blocks=l1, l1_xz=_relative_xz(near, z, x), l2_blocks=l2, l2_xz=_relative_xz(far, z, x),
                biomes=biome_volume(biomes, z, x, spec), known=None, l2_keys=[(world,) + c for c in far])
