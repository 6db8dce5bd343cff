"""The module-level drop-ins on the GPU (`streamvoxel_b200.modules`): the reference model object at the engine
boundary, `CompactStreamingControlNet.forward` and `UnconditionalMD4DiT.forward` against the oracle's bf16 forward.

Tolerance (BASELINE contract): logits within 2e-2 abs + 1e-2 rel of the bf16 forward on the same weights and inputs.
"""
import numpy as np
import pytest
import torch

from oracle import model as om

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _cfg_dict(cfg):
    return dict(num_classes=cfg.classes, voxel_shape=cfg.voxel_shape, patch_size=4, depth=cfg.depth,
                num_heads=cfg.heads, y_range=cfg.y_range, layer_indices=list(cfg.layer_indices),
                biome_halo=cfg.biome_halo, biome_patch=cfg.biome_patch)


def test_fast_slot_forward_takes_the_reference_model_object():
    """`FastSlotForward(model, spec, ...)` with a reference-shaped module (as `worker.py:272` passes it) gives the
    same logits, bit for bit, as the engine built from the (config, state dict) pair."""
    from module_standin import reference_like
    from streamvoxel_b200 import model as sm, synth
    from streamvoxel_b200.stream.condition import ModelSpec
    from streamvoxel_b200.stream.fast_ops import FastSlotForward
    cfg = sm.small_test_config()
    sd = sm.synthetic_state_dict(cfg, seed=6, std=0.05)
    spec = ModelSpec.of(cfg)
    outs = []
    for model in (reference_like(cfg, sd), (cfg, sd)):
        engine = FastSlotForward(model, spec, 'cuda', 2, 3, 8)
        for i in range(2):
            engine.load_slot(i, synth.item(60 + i, spec, k=1 + i, far=8))
        engine.wait_loads()
        engine.tokens.copy_(torch.from_numpy(np.stack([synth.target_tokens(70 + i, spec)[0] for i in range(2)])))
        outs.append(engine.replay(torch.ones(2)).clone())
    assert torch.equal(outs[0], outs[1])


def test_controlnet_forward_matches_oracle():
    """`ControlNetForward(model)(tokens, timestep=, origin_xyz=, group_origin_xyz=, prefix_kv=, local=,
    local_positions=)`: the prefix K/V, local tokens and positions as `engine.unpadded_logits` passes them (made by
    the oracle encoder), for windows with 0 and 3 L1 tiles through one engine."""
    from module_standin import reference_like
    from streamvoxel_b200 import model as sm, synth
    from streamvoxel_b200.modules import ControlNetForward
    from streamvoxel_b200.stream.condition import ModelSpec
    cfg = sm.small_test_config()
    sd = sm.synthetic_state_dict(cfg, seed=8, std=0.05)
    spec = ModelSpec.of(cfg)
    forward = ControlNetForward(reference_like(cfg, sd))
    origin = torch.tensor([[0., cfg.y_range[0], 0.]])
    for k in (0, 3):
        item = synth.item(80 + k, spec, k=k, far=8)
        prefix_kv, (_, local, positions) = om.encode_condition(sd, item.l1_blocks, item.l1_xz, item.l2_blocks,
                                                               item.l2_xz, item.biomes, _cfg_dict(cfg), bf16=True)
        tokens = torch.from_numpy(synth.target_tokens(90 + k, spec)[0][None]).long()
        got = forward(tokens.cuda(), timestep=torch.ones(1), origin_xyz=origin, group_origin_xyz=origin[0],
                      prefix_kv=[(pk.cuda(), pv.cuda()) for pk, pv in prefix_kv], local=local.cuda(),
                      local_positions=positions.cuda())
        kv = om.encode_kv(sd, item.l1_blocks, item.l1_xz, item.l2_blocks, item.l2_xz, item.biomes, _cfg_dict(cfg),
                          bf16=True)
        want = om.control_forward(sd, tokens, kv, _cfg_dict(cfg), bf16=True)
        torch.testing.assert_close(got.float().cpu(), want, atol=ATOL, rtol=RTOL)
    with pytest.raises(ValueError):
        forward(tokens.cuda(), timestep=torch.ones(1), origin_xyz=origin, group_origin_xyz=origin[0],
                prefix_kv=[(pk.cuda(), pv.cuda()) for pk, pv in prefix_kv], local=local.cuda(),
                local_positions=positions.cuda(), scale=0.5)


def test_dit_forward_matches_oracle():
    """`DiTForward(model)(tokens, timestep=, origin_xyz=)`: the time-free backbone alone, batch 2."""
    from module_standin import reference_like
    from streamvoxel_b200 import model as sm, synth
    from streamvoxel_b200.modules import DiTForward
    from streamvoxel_b200.stream.condition import ModelSpec
    cfg = sm.small_test_config(layer_indices=())
    sd = sm.synthetic_state_dict(cfg, seed=9, std=0.05)
    forward = DiTForward(reference_like(cfg, sd))
    spec = ModelSpec.of(cfg)
    tokens = torch.from_numpy(np.stack([synth.target_tokens(100 + i, spec)[0] for i in range(2)])).long()
    origin = torch.tensor([[0., cfg.y_range[0], 0.]] * 2)
    got = forward(tokens.cuda(), timestep=torch.ones(2), origin_xyz=origin)
    want = om.unconditional_forward(sd, tokens, _cfg_dict(cfg), bf16=True)
    torch.testing.assert_close(got.float().cpu(), want, atol=ATOL, rtol=RTOL)
    with pytest.raises(ValueError):
        forward(tokens.cuda(), timestep=torch.ones(3))
