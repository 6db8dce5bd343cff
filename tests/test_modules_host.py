"""The module boundary on the CPU: a reference model object becomes the engine's configuration and state dict.

With the reference checkout present (the build container), the reference's own `CompactStreamingControlNet` and
time-free `UnconditionalMD4DiT` are built and read; the GPU box has no checkout, and these cases skip there.
"""
import os
import sys

import pytest
import torch

from streamvoxel_b200 import model as sm
from streamvoxel_b200.modules import model_config, prepare

REFERENCE = os.environ.get('STREAMVOXEL_REFERENCE', '/root/reference')


def _reference():
    if not os.path.isdir(os.path.join(REFERENCE, 'streamvoxel')):
        pytest.skip('reference checkout not present')
    if REFERENCE not in sys.path:
        sys.path.insert(0, REFERENCE)
    from streamvoxel.models.compact_controlnet import CompactStreamingControlNet
    from streamvoxel.models.unconditional_md4_timefree import UnconditionalMD4DiT
    return CompactStreamingControlNet, UnconditionalMD4DiT


def test_reference_controlnet_gives_the_small_config_and_every_parameter():
    Control, DiT = _reference()
    torch.manual_seed(0)
    base = DiT(num_classes=32, voxel_shape=(64, 16, 16), hidden_dim=192, depth=3, num_heads=2, time_free=True)
    model = Control(base, control_depth=2, control_hidden_dim=192, checkpointing=False, biome_halo=4, biome_patch=4,
                    biome_classes=16, struct_classes=0)
    cfg, state = prepare(model)
    assert cfg == sm.small_test_config()
    assert set(state) == set(sm.state_dict_shapes(cfg))
    reference_state = model.state_dict()
    for name, value in state.items():
        assert torch.equal(value, reference_state[name]), name
    from module_standin import reference_like
    assert model_config(reference_like(cfg, sm.synthetic_state_dict(cfg))) == cfg


def test_reference_dit_gives_the_unconditional_config():
    _, DiT = _reference()
    base = DiT(num_classes=32, voxel_shape=(64, 16, 16), hidden_dim=192, depth=3, num_heads=2, time_free=True)
    cfg, state = prepare(base)
    assert cfg == sm.small_test_config(layer_indices=())
    assert set(state) == set(sm.state_dict_shapes(cfg))
    assert torch.equal(state['backbone.blocks.2.mlp.0.weight'], base.blocks[2].mlp[0].weight)


def test_unsupported_reference_models_are_rejected():
    Control, DiT = _reference()
    timed = DiT(num_classes=8, voxel_shape=(16, 16, 16), hidden_dim=48, depth=2, num_heads=4, time_free=False)
    with pytest.raises(ValueError, match='time-free'):
        model_config(timed)
    base = DiT(num_classes=8, voxel_shape=(16, 16, 16), hidden_dim=48, depth=2, num_heads=4, time_free=True)
    narrow = Control(base, control_depth=2, control_hidden_dim=24, checkpointing=False, struct_classes=0)
    with pytest.raises(ValueError, match='width'):
        model_config(narrow)


def test_standin_round_trip_without_reference():
    from module_standin import reference_like
    for cfg in (sm.small_test_config(), sm.small_test_config(layer_indices=())):
        sd = sm.synthetic_state_dict(cfg, seed=1)
        got_cfg, got = prepare(reference_like(cfg, sd))
        assert got_cfg == cfg and set(got) == set(sd)
        assert all(torch.equal(got[k], sd[k]) for k in sd)
