"""The world-expansion driver through the real engine (small model): windows conditioned on committed columns via
`make_item`, sampled by the whole-step graph, committed and re-admitted until the region is full."""
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
