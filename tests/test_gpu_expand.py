"""The world-expansion driver through the real engine (small model): windows conditioned on committed columns via
`make_item`, sampled by the whole-step graph, committed and re-admitted until the region is full."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_small_expansion_through_the_engine():
    from streamvoxel_b200 import model as sm
    from streamvoxel_b200.stream import expand
    from streamvoxel_b200.stream.batch import SlotBatch
    from streamvoxel_b200.stream.condition import ModelSpec
    from streamvoxel_b200.stream.fast_ops import FastSlotForward
    cfg = sm.small_test_config()
    spec = ModelSpec.of(cfg)
    forward = FastSlotForward((cfg, sm.synthetic_state_dict(cfg, seed=0)), spec, 'cuda', 4, 8, 24)
    engine = SlotBatch(forward)
    committed, region, biomes, player = expand.start_region(3, 2, 4, spec, classes=cfg.classes)
    exp = expand.Expansion(committed, biomes, spec, player, region, slots=4, l2_cap=24)
    stats = expand.run(engine, exp, 0)
    assert exp.done and stats['windows'] == 12 and len(exp.committed) == 16
    for cell in region - set(committed):
        col = exp.committed[cell]
        assert col.shape == (spec.height, spec.tile, spec.tile)
        assert col.min() >= 0 and col.max() < cfg.classes   # no mask id left: every voxel committed
    assert stats['forwards'] > 0 and stats['blocked_admissions'] >= 0


def test_l2_token_cache_gives_identical_keys_and_values():
    import torch
    from streamvoxel_b200 import model as sm
    from streamvoxel_b200.model import L2TokenCache, PreparedModel
    from streamvoxel_b200.stream import expand
    from streamvoxel_b200.stream.condition import ModelSpec
    cfg = sm.small_test_config()
    spec = ModelSpec.of(cfg)
    model = PreparedModel(cfg, sm.synthetic_state_dict(cfg, seed=0), 'cuda')
    committed, region, biomes, player = expand.start_region(3, 4, 6, spec, classes=cfg.classes)
    exp = expand.Expansion(committed, biomes, spec, player, region, slots=4, l2_cap=12)
    cache = L2TokenCache()
    for cell in sorted(exp.ready)[:3]:
        item = exp.item(cell)
        args = (item.l1_blocks, item.l1_xz, item.l2_blocks, item.l2_xz, item.biomes)
        plain = model.encode_item(*args)
        cached = model.encode_item(*args, l2_keys=item.l2_keys, cache=cache)
        for (k0, v0), (k1, v1) in zip(plain, cached):
            assert torch.equal(k0, k1) and torch.equal(v0, v1)
    assert cache.hits > 0 and cache.misses <= len(committed)


def test_device_exchange_two_ranks():
    """`DeviceExchange` (finished columns and free-slot counts all-gathered over NCCL) gives every rank the same
    rounds, including rounds where nobody or only one rank finished."""
    import torch
    from exchange_worker import check_rounds, run_two_ranks
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two GPUs')
    check_rounds(run_two_ranks('nccl'))
