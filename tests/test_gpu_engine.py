"""The slot-batched forward (svx_engine_forward through FastSlotForward) against the CPU oracle's bf16 forward.

Tolerance (BASELINE contract): logits within 2e-2 abs + 1e-2 rel of the reference bf16 forward on the same
random-init weights and inputs. The oracle runs the reference's forward in fp32 arithmetic with the bf16 rounding points
of CUDA autocast (`oracle/model.py`); it is fed the same packed K/V the engine holds, so this isolates the forward.
The encoder is checked separately against the oracle encoder.
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


def _engine(cfg, slots, seed=0, std=0.02, l1_cap=3, l2_cap=80):
    from streamvoxel_b200 import model as sm
    from streamvoxel_b200.stream.condition import ModelSpec
    from streamvoxel_b200.stream.fast_ops import FastSlotForward
    sd = sm.synthetic_state_dict(cfg, seed=seed, std=std)
    spec = ModelSpec.of(cfg)
    engine = FastSlotForward((cfg, sd), spec, 'cuda', slots, l1_cap, l2_cap)
    return engine, sd, spec


def _kv_of_slot(engine, slot):
    length = int(engine.packed.lengths[slot])
    return [(k[slot:slot + 1, :, :length].float().cpu(), v[slot:slot + 1, :, :length].float().cpu())
            for k, v in engine.packed.kv]


def _assert_logits(got, want, outlier_ppm=0.0, min_agree=0.99):
    """Every logit within ATOL + RTOL |want|. A full-size 24-block forward may leave `outlier_ppm` parts per million of
    its 16.7 M logits up to 1.5 times that bound: two bf16 forwards with identical rounding points that differ only in
    fp32 accumulation order already reach 0.94 of the bound there (`tests/test_forward_noise_floor.py`), and the
    kernels round the folded LayerNorm's weights where the oracle rounds the modulated activations.
    Random-init logits have near-tied top classes, so bf16 noise alone flips some argmaxes (1.4% between the two
    valid full-size forwards above); a gross error flips most."""
    d = (got - want).abs()
    bound = ATOL + RTOL * want.abs()
    bad = int((d > bound).sum())
    print(f'logits: max |d| {float(d.max()):.4g}, mean |d| {float(d.mean()):.3g}, out of tolerance {bad} / '
          f'{got.numel()}, max |d| / bound {float((d / bound).max()):.3f}')
    if outlier_ppm == 0.0:
        torch.testing.assert_close(got, want, atol=ATOL, rtol=RTOL)
    else:
        assert bad <= outlier_ppm * 1e-6 * got.numel(), bad
        assert bool((d <= 1.5 * bound).all()), float((d / bound).max())
    assert float((got - want).abs().mean()) <= 5e-3
    agree = float((got.argmax(0) == want.argmax(0)).float().mean())
    print(f'argmax agreement {agree:.4f}')
    assert agree >= min_agree, agree


def test_small_forward_matches_oracle_per_slot():
    from streamvoxel_b200 import model as sm, synth
    cfg = sm.small_test_config()
    engine, sd, spec = _engine(cfg, 3, std=0.05, l1_cap=3, l2_cap=8)
    tokens = []
    for i, k in enumerate((0, 2, 3)):
        engine.load_slot(i, synth.item(100 + i, spec, k=k, far=8))
        t, _ = synth.target_tokens(200 + i, spec)
        tokens.append(t)
    engine.wait_loads()
    engine.tokens.copy_(torch.from_numpy(np.stack(tokens)).cuda())
    got = engine.eager(torch.ones(3)).float().cpu()
    for i in range(3):
        want = om.control_forward(sd, torch.from_numpy(tokens[i][None]).long(), _kv_of_slot(engine, i),
                                  _cfg_dict(cfg), bf16=True)[0]
        _assert_logits(got[i], want)


def test_wide_forward_matches_oracle_per_slot():
    """The BASELINE config-5 width (d = 1152, 12 heads x 96, MLP 4608): 36 row-statistics chunks per LayerNorm fold,
    18-block K loops, 12-head attention plans; two backbone layers, both fed by control layers."""
    from streamvoxel_b200 import model as sm, synth
    cfg = sm.small_test_config(d=1152, heads=12, mlp=4608, depth=2, layer_indices=(0, 1))
    engine, sd, spec = _engine(cfg, 2, std=0.02, l1_cap=3, l2_cap=8)
    tokens = []
    for i, k in enumerate((1, 3)):
        engine.load_slot(i, synth.item(300 + i, spec, k=k, far=8))
        t, _ = synth.target_tokens(400 + i, spec)
        tokens.append(t)
    engine.wait_loads()
    engine.tokens.copy_(torch.from_numpy(np.stack(tokens)).cuda())
    got = engine.eager(torch.ones(2)).float().cpu()
    for i in range(2):
        want = om.control_forward(sd, torch.from_numpy(tokens[i][None]).long(), _kv_of_slot(engine, i),
                                  _cfg_dict(cfg), bf16=True)[0]
        _assert_logits(got[i], want)


def test_graph_replay_equals_eager_and_buckets_agree():
    from streamvoxel_b200 import model as sm, synth
    cfg = sm.small_test_config()
    engine, sd, spec = _engine(cfg, 4, std=0.05, l1_cap=2, l2_cap=8)
    for i in range(4):
        engine.load_slot(i, synth.item(300 + i, spec, k=i % 3, far=8))
    engine.wait_loads()
    engine.tokens.copy_(torch.from_numpy(np.stack([synth.target_tokens(400 + i, spec)[0] for i in range(4)])).cuda())
    assert sorted(engine.graphs) == [1, 2, 4]
    eager = engine.eager(torch.ones(4)).clone()
    replayed = engine.replay(torch.ones(4)).clone()
    assert torch.equal(eager, replayed)
    small = engine.replay(torch.ones(4), 2)[:2].clone()
    assert torch.equal(small, eager[:2])   # row-independent kernels: the bucket does not change slot results
    report = engine.numerical_gate(synth.item(500, spec, k=1, far=8), synth.item(501, spec, k=2, far=8))
    assert report['graph_equal'] and report['padded_close'] and report['bucket_close']


def test_encoder_matches_oracle_encoder():
    from streamvoxel_b200 import model as sm, synth
    cfg = sm.small_test_config()
    engine, sd, spec = _engine(cfg, 1, std=0.05, l1_cap=3, l2_cap=8)
    item = synth.item(600, spec, k=3, far=8)
    got = engine.encode(item)
    want = om.encode_kv(sd, item.l1_blocks, item.l1_xz, item.l2_blocks, item.l2_xz, item.biomes, _cfg_dict(cfg),
                        bf16=True)
    l1, l2, biome = cfg.condition_widths()
    assert got[0][0].shape[1] == want[0][0].shape[2] == 8 * l2 + 3 * l1 + biome
    for (gk, gv), (wk, wv) in zip(got, want):
        torch.testing.assert_close(gk.float().cpu(), wk[0], atol=3e-2, rtol=2e-2)
        torch.testing.assert_close(gv.float().cpu(), wv[0], atol=3e-2, rtol=2e-2)


@pytest.mark.slow
def test_full_size_control_forward_matches_oracle():
    """DiT-B/4 + 12-layer ControlNet (BASELINE config 2 model), slot 1 of a 2-slot batch, k=2 L1 + 80 L2 + biome."""
    from streamvoxel_b200 import model as sm, synth
    cfg = sm.dit_b4_control()
    engine, sd, spec = _engine(cfg, 2, l1_cap=8, l2_cap=81)
    engine.load_slot(0, synth.item(700, spec, k=5))
    engine.load_slot(1, synth.item(701, spec, k=2))
    engine.wait_loads()
    tokens = np.stack([synth.target_tokens(800 + i, spec)[0] for i in range(2)])
    engine.tokens.copy_(torch.from_numpy(tokens).cuda())
    got = engine.replay(torch.ones(2))[1].float().cpu()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    want = om.control_forward(sd, torch.from_numpy(tokens[1:2]).long(), _kv_of_slot(engine, 1), _cfg_dict(cfg),
                              bf16=True)[0]
    _assert_logits(got, want, outlier_ppm=1.0, min_agree=0.98)


@pytest.mark.slow
def test_full_size_unconditional_forward_matches_oracle():
    """BASELINE config 1 model: the time-free DiT-B/4 alone, batch 1, a partially masked column."""
    from streamvoxel_b200 import model as sm, synth
    from streamvoxel_b200.model import Engine, PreparedModel
    cfg = sm.dit_b4_unconditional()
    sd = sm.synthetic_state_dict(cfg, seed=3)
    model = PreparedModel(cfg, sd, 'cuda')
    engine = Engine(model, 1, 0)
    from streamvoxel_b200.stream.condition import ModelSpec
    tokens, _ = synth.target_tokens(900, ModelSpec.of(cfg))
    t = torch.from_numpy(tokens[None]).cuda()
    logits = torch.empty((1, cfg.classes, *cfg.voxel_shape), dtype=torch.bfloat16, device='cuda')
    got = engine.forward(1, t, logits)[0].float().cpu()
    want = om.unconditional_forward(sd, torch.from_numpy(tokens[None]).long(), _cfg_dict(cfg), bf16=True)[0]
    _assert_logits(got, want, min_agree=0.98)


@pytest.mark.slow
def test_full_size_forward_against_reference_fp32_logits():
    """The engine's bf16 forward of the full-size config-2 model against the reference's own fp32 forward
    (`engine.unpadded_logits` run on the CPU, fixture `tests/golden/control_full.npz`: 512 voxels x 256 classes, the
    window `synth.item(701, k=2)` encoded by our encoder). A bf16 forward cannot equal an fp32 one: the oracle's bf16
    forward sits at mean |d| 0.0044, max |d| 0.023 (1.09 of the 2e-2 / 1e-2 bound) and 98% argmax agreement from these
    same logits, so the engine must stay within 1.4 times that mean, twice the bound and 97% agreement."""
    import os
    from streamvoxel_b200 import model as sm, synth
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden', 'control_full.npz'))
    cfg = sm.dit_b4_control()
    engine, sd, spec = _engine(cfg, 1, l1_cap=8, l2_cap=81)
    engine.load_slot(0, synth.item(701, spec, k=2))
    engine.wait_loads()
    engine.tokens.copy_(torch.from_numpy(g['tokens'][None]).cuda())
    got = engine.replay(torch.ones(1))[0].float().reshape(cfg.classes, -1)[:, torch.from_numpy(g['voxels']).cuda()]
    want = torch.from_numpy(g['logits']).cuda()
    d = (got - want).abs()
    ratio = float((d / (ATOL + RTOL * want.abs())).max())
    agree = float((got.argmax(0) == want.argmax(0)).float().mean())
    print(f'vs reference fp32: max |d| {float(d.max()):.4g}, mean |d| {float(d.mean()):.4g}, max |d| / bound '
          f'{ratio:.3f}, argmax agreement {agree:.4f}')
    assert float(d.mean()) <= 1.4 * 0.0044 and ratio <= 2.0 and agree >= 0.97


@pytest.mark.slow
def test_full_size_config5_forward_matches_oracle():
    """BASELINE config 5 model at full size: the DiT-L/4-class backbone (d = 1152, 12 x 96 heads, 24 layers, MLP 4608)
    + 24-layer ControlNet, slot 1 of a 2-slot batch (k = 3 L1 tiles, 80 L2 columns, the biome window), against the
    oracle's bf16-rounding forward. 48 blocks and 24 cross-attentions put this model's bf16 noise floor above the
    bound: two forwards with identical rounding points and fp32 versus float64 accumulation differ by mean |d| 0.0052,
    leave 493 ppm of logits outside the bound, reach 1.63 times it and disagree on 1.7% of argmaxes
    (`tests/test_forward_noise_floor.py` with SVX_NOISE_FLOOR_CONFIG5=1). The engine must stay within 1.25 times that
    mean, twice that outlier share and 2 times the bound, and agree on 97.5% of argmaxes."""
    from streamvoxel_b200 import model as sm, synth
    cfg = sm.dit_l4_control()
    engine, sd, spec = _engine(cfg, 2, l1_cap=8, l2_cap=81)
    engine.load_slot(0, synth.item(710, spec, k=6))
    engine.load_slot(1, synth.item(711, spec, k=3))
    engine.wait_loads()
    tokens = np.stack([synth.target_tokens(810 + i, spec)[0] for i in range(2)])
    engine.tokens.copy_(torch.from_numpy(tokens).cuda())
    got = engine.replay(torch.ones(2))[1].float().cpu()
    want = om.control_forward(sd, torch.from_numpy(tokens[1:2]).long(), _kv_of_slot(engine, 1), _cfg_dict(cfg),
                              bf16=True)[0]
    d = (got - want).abs()
    bound = ATOL + RTOL * want.abs()
    ppm = float((d > bound).sum()) / got.numel() * 1e6
    ratio = float((d / bound).max())
    agree = float((got.argmax(0) == want.argmax(0)).float().mean())
    print(f'config 5 logits: max |d| {float(d.max()):.4g}, mean |d| {float(d.mean()):.4g}, outside the bound {ppm:.0f} '
          f'ppm, max |d| / bound {ratio:.3f}, argmax agreement {agree:.4f}')
    assert float(d.mean()) <= 1.25 * 0.0052 and ppm <= 2 * 493 and ratio <= 2.0 and agree >= 0.975
