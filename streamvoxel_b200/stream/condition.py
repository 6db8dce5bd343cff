"""Condition types of a generation window (`streamvoxel/stream/condition.py:21-85`): the model spec and one item.

Only the in-memory types the engine consumes are mirrored; request parsing and the wire format are not on the path.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass(frozen=True)
class ModelSpec:
    """`streamvoxel/stream/condition.py:21-34`."""
    height: int
    tile: int
    num_classes: int        # the MASK token id equals num_classes
    biome_classes: int
    biome_halo: int
    y_origin: float
    trained_l1: tuple = (1, 3)

    @property
    def biome_shape(self):
        side = 6 if self.biome_halo == 4 else 12
        return (self.height // 4, side, side)

    @classmethod
    def of(cls, cfg):
        """The spec of a `ModelConfig` (`streamvoxel/stream/engine.py:289-296`)."""
        return cls(height=cfg.voxel_shape[0], tile=cfg.voxel_shape[1], num_classes=cfg.classes,
                   biome_classes=cfg.biome_classes, biome_halo=cfg.biome_halo, y_origin=float(cfg.y_range[0]))


@dataclass
class Item:
    """`streamvoxel/stream/condition.py:68-85`: one window's conditions, XZ relative to the target tile."""
    id: str
    seed: int
    steps: int
    temperature: float
    l1_blocks: np.ndarray    # [n1,H,T,T] int16
    l1_xz: np.ndarray        # [n1,2] int64 voxels
    l2_blocks: np.ndarray    # [n2,H,T,T]
    l2_xz: np.ndarray        # [n2,2]
    biomes: np.ndarray       # [H/4,12,12] int64, zero padded outside the supplied window
    known: np.ndarray | None = None
    warnings: list = field(default_factory=list)
    # Absolute (world, z, x) keys of the L2 columns, when the item was built from a committed snapshot: committed
    # columns never change, so the engine may reuse their encoded tokens across windows (None: encode every time).
    l2_keys: list | None = None


def probe_item(spec):
    """`streamvoxel/stream/engine.py:275-280`: a minimal item used to size and warm the engine."""
    height, tile = spec.height, spec.tile
    blocks = np.zeros((1, height, tile, tile), np.int16)
    biomes = np.zeros((height // 4, 12, 12), np.int64)
    return Item('probe', 0, 1, 1.0, blocks, np.asarray([[-tile, 0]], np.int64), blocks.copy(),
                np.asarray([[-2 * tile, 0]], np.int64), biomes, None)


def largest_item(spec, l1_cap, l2_cap):
    """An item with the most conditions a slot holds (`l1_cap` L1 tiles, `l2_cap` L2 columns), all-air columns."""
    height, tile = spec.height, spec.tile
    l1 = np.zeros((max(1, l1_cap), height, tile, tile), np.int16)
    l2 = np.zeros((max(1, l2_cap), height, tile, tile), np.int16)
    offsets = lambda n, r: np.asarray([[(i % 9 - 4) * tile, (i // 9 - r) * tile] for i in range(n)], np.int64)
    return Item('largest', 0, 1, 1.0, l1, offsets(len(l1), 6), l2, offsets(len(l2), 4),
                np.zeros((height // 4, 12, 12), np.int64), None)
