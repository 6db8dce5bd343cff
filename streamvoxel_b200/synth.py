"""Seeded synthetic columns, windows and conditions with the shapes and distributions of the benchmark configs.

No dataset or checkpoint of the reference exists outside its authors' pipeline, so every run uses these stand-ins:

* world: a smoothed-noise heightmap h(z, x) in [40, 120] (voxel y), block ids 1..4 below the surface, air (0) above,
  and 2% random ids 5..255 within 8 voxels of the surface;
* a slot's target column is masked with a per-slot ratio r ~ U[0, 1];
* conditions: k ~ U{0..8} committed neighbour columns (L1, 4^3 patches), the other 80 columns of the 9x9 around the
  target (L2, 16^3 patches) and an 8x8 biome grid of 16 classes (the centre 6x6 of the [H/4, 12, 12] biome window).
"""
from __future__ import annotations

import numpy as np

from streamvoxel_b200.stream.condition import Item


def heightmap(rng, cells_z, cells_x, tile=16, low=40, high=120, coarse=2):
    """Bilinear upsampling of a coarse uniform grid (one knot every `coarse` cells) to voxel resolution."""
    gz, gx = cells_z // coarse + 2, cells_x // coarse + 2
    knots = rng.random((gz, gx))
    vz = np.arange(cells_z * tile) / (coarse * tile)
    vx = np.arange(cells_x * tile) / (coarse * tile)
    z0, x0 = np.floor(vz).astype(int), np.floor(vx).astype(int)
    fz, fx = (vz - z0)[:, None], (vx - x0)[None, :]
    a = knots[z0][:, x0]
    b = knots[z0][:, x0 + 1]
    c = knots[z0 + 1][:, x0]
    d = knots[z0 + 1][:, x0 + 1]
    smooth = (a * (1 - fx) + b * fx) * (1 - fz) + (c * (1 - fx) + d * fx) * fz
    return np.rint(low + (high - low) * smooth).astype(np.int64)


def world(seed, cells_z, cells_x, height=256, tile=16):
    """Columns {(z, x): [height, tile, tile] int16} of a synthetic region."""
    rng = np.random.default_rng(seed)
    h = heightmap(rng, cells_z, cells_x, tile)
    y = np.arange(height)[:, None, None]
    cells = {}
    for z in range(cells_z):
        for x in range(cells_x):
            top = h[z * tile:(z + 1) * tile, x * tile:(x + 1) * tile][None]
            col = np.where(y < top, rng.integers(1, 5, (height, tile, tile)), 0)
            near = (np.abs(y - top) <= 8) & (rng.random((height, tile, tile)) < 0.02)
            col = np.where(near, rng.integers(5, 256, (height, tile, tile)), col)
            cells[(z, x)] = col.astype(np.int16)
    return cells


def clip_classes(column, classes):
    """Map ids >= classes (small test vocabularies) into range."""
    return np.where(column >= classes, column % classes, column).astype(np.int16)


def masked(rng, column, mask_id):
    """A partially masked column: each voxel masked with a per-column ratio r ~ U[0, 1]."""
    ratio = rng.random()
    return np.where(rng.random(column.shape) < ratio, mask_id, column).astype(np.int16)


def biome_window(rng, height, classes=16):
    """[H/4, 12, 12] int64 biome labels, zero outside the centre 6x6 (`streamvoxel/stream/condition.py:154-156`)."""
    biomes = np.zeros((height // 4, 12, 12), np.int64)
    biomes[:, 3:9, 3:9] = rng.integers(0, classes, (height // 4, 6, 6))
    return biomes


NEIGHBOURS = [(-1, -1), (-1, 0), (-1, 1), (0, -1), (0, 1), (1, -1), (1, 0), (1, 1)]


def item(seed, spec, k=None, far=80, classes=None):
    """One window's conditions in the target frame (x, z offsets in voxels), like `make_item` would build."""
    rng = np.random.default_rng(seed)
    height, tile = spec.height, spec.tile
    classes = spec.num_classes if classes is None else classes
    k = int(rng.integers(0, 9)) if k is None else int(k)
    region = world(int(rng.integers(1 << 30)), 9, 9, height, tile)
    cells = {key: clip_classes(col, classes) for key, col in region.items()}
    near = [NEIGHBOURS[i] for i in sorted(rng.choice(8, size=k, replace=False))] if k else []
    others = [(dz, dx) for dz in range(-4, 5) for dx in range(-4, 5) if (dz, dx) != (0, 0)][:far]
    l1 = np.stack([cells[(4 + dz, 4 + dx)] for dz, dx in near]) if near else np.zeros((0, height, tile, tile), np.int16)
    l2 = np.stack([cells[(4 + dz, 4 + dx)] for dz, dx in others]) if others else np.zeros((0, height, tile, tile), np.int16)
    xz = lambda offs: np.asarray([[dx * tile, dz * tile] for dz, dx in offs], np.int64).reshape(-1, 2)
    return Item(f'synthetic{seed}', seed, 32, 1.0, l1, xz(near), l2, xz(others),
                biome_window(rng, height, spec.biome_classes), None)


def target_tokens(seed, spec, classes=None):
    """A partially masked target column (ground truth from the same world generator)."""
    rng = np.random.default_rng(seed + 7919)
    classes = spec.num_classes if classes is None else classes
    column = clip_classes(world(int(rng.integers(1 << 30)), 1, 1, spec.height, spec.tile)[(0, 0)], classes)
    return masked(rng, column, spec.num_classes), column


def ease_logits(seed, slots, classes=256, voxels=65536, sigma=2 ** 0.5, boost=6.0, fraction=0.7, truth=None):
    """BASELINE config 3 logits: N(0, sigma^2) with +boost on the ground-truth id of a seeded 70% of voxels.
    Returns fp32 [slots, classes, voxels] and the ground truth [slots, voxels]."""
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((slots, classes, voxels), dtype=np.float32) * np.float32(sigma)
    if truth is None:
        truth = rng.integers(0, classes, (slots, voxels))
    pick = rng.random((slots, voxels)) < fraction
    s, v = np.nonzero(pick)
    logits[s, truth[s, v], v] += np.float32(boost)
    return logits, truth
