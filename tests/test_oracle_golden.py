"""Pin the CPU oracle to the reference: every fixture under tests/golden/ was produced by the reference itself
(`tests/golden/make_golden.py`). Integer/index results must be equal; fp32 results agree to rounding."""
import os

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import sampler as osm

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_block_quota_select_matches_reference():
    g = _load('quota_select.npz')
    for i in range(int(g['count'])):
        p = f'c{i}_'
        got = osm.block_quota_select(g[p + 'score'], g[p + 'selectable'], int(g[p + 'k']), 4, g[p + 'order'],
                                     float(g[p + 'frac']), g[p + 'n_total'])
        assert np.array_equal(got, g[p + 'chosen']), i
        assert int(got.sum()) == int(g[p + 'k'])


def test_top_mask_matches_reference_with_ties():
    g = _load('top_mask.npz')
    for i in range(int(g['count'])):
        got = osm.top_mask(g[f't{i}_scores'], g[f't{i}_eligible'], int(g[f't{i}_count']))
        assert np.array_equal(got, g[f't{i}_mask']), i


def test_quotas_and_schedule_match_reference():
    g = _load('schedule.npz')
    for i in range(int(g['count'])):
        total, steps, n_last = (int(v) for v in g[f's{i}_args'])
        assert osm.low_entropy_last_quotas(total, steps, n_last) == g[f's{i}_quotas'].tolist()
        assert osm.counts(total, steps) == g[f's{i}_counts'].tolist()
    assert np.array_equal(np.asarray([osm.actual_time(f) for f in g['time_in']]), g['time_out'])


def test_scores_air_and_last_mask_match_reference():
    g = _load('scores.npz')
    for i in range(int(g['count'])):
        logits = g[f'e{i}_logits']
        np.testing.assert_allclose(osm.entropy_scores(logits), g[f'e{i}_entropy'], atol=2e-6, rtol=1e-5)
        air = osm.air_probability(logits, (0,))
        np.testing.assert_allclose(air, g[f'e{i}_air'], atol=1e-6, rtol=1e-6)
        ones = np.ones(air.shape, bool)
        last = osm.low_entropy_last_update(np.zeros(air.shape, bool), ones, g[f'e{i}_air'], ~ones, float(g[f'e{i}_eps']),
                                           False, True)
        assert np.array_equal(last, g[f'e{i}_last']), i


def _fixture_logits(step, ground):
    generator = torch.Generator().manual_seed(step + 1)
    logits = torch.randn((6, 16, 8, 8), generator=generator)
    logits[0, ground:] += 30.
    return logits.numpy()


def test_slot_windows_match_reference_given_its_draws():
    g = _load('slot_windows.npz')
    for i in range(int(g['count'])):
        seed, cap, ground = (int(v) for v in g[f'w{i}_args'])
        slot = osm.Slot((16, 8, 8), 6, (0,), 0, 1e-3, 4)
        slot.arm(seed, cap, (i, 0), g[f'w{i}_order'])
        tokens = np.full((16, 8, 8), 6, np.int64)
        step = 0
        while not slot.idle:
            logits = _fixture_logits(step + 31 * i, ground)
            key = f'w{i}_s{step}_noise'
            noise = (lambda k, c, key=key: g[key]) if key in g.files else None
            record, commit = slot.consume(logits, tokens, noise=noise)
            if commit is not None:
                assert np.array_equal(commit['positions'], g[f'w{i}_s{step}_positions'])
                assert np.array_equal(commit['values'], g[f'w{i}_s{step}_values'])
            step += 1
        assert step == int(g[f'w{i}_steps'])
        assert np.array_equal(tokens, g[f'w{i}_tokens'])
        assert np.array_equal(record['step_map'], g[f'w{i}_step_map'])
        assert np.array_equal(record['values'], g[f'w{i}_values'])
        assert [record['nfe'], record['actual'], record['last_count']] == g[f'w{i}_record'].tolist()


def _sd(g, prefix=''):
    return {prefix + k[3:]: torch.from_numpy(np.asarray(g[k])) for k in g.files if k.startswith('sd.')}


def test_dit_forward_matches_reference_fp32():
    g = _load('dit_tiny.npz')
    cfg = dict(num_classes=5, voxel_shape=(16, 16, 16), patch_size=4, depth=3, num_heads=4, y_range=(-64., 192.))
    got = om.unconditional_forward(_sd(g, 'backbone.'), torch.from_numpy(g['tokens']), cfg)
    torch.testing.assert_close(got, torch.from_numpy(g['logits']), atol=1e-5, rtol=1e-5)


def test_dit_bf16_rounding_points_track_autocast():
    """The bf16 emulation stays within bf16 noise of the reference run under CPU bf16 autocast."""
    g = _load('dit_tiny.npz')
    want = torch.from_numpy(_load('dit_tiny_cpu_autocast.npz')['logits'])
    cfg = dict(num_classes=5, voxel_shape=(16, 16, 16), patch_size=4, depth=3, num_heads=4, y_range=(-64., 192.))
    got = om.unconditional_forward(_sd(g, 'backbone.'), torch.from_numpy(g['tokens']), cfg, bf16=True)
    fp32 = torch.from_numpy(g['logits'])
    assert (got - want).abs().max() < 0.1 * max(1e-3, float(fp32.abs().max()))


def test_control_forward_and_encoder_match_reference_fp32():
    g = _load('control_tiny.npz')
    sd = _sd(g)
    cfg = dict(num_classes=3, voxel_shape=(16, 16, 16), patch_size=4, depth=5, num_heads=4, y_range=(-64., 192.),
               layer_indices=g['layer_indices'].tolist(), biome_halo=4, biome_patch=2)
    tokens = torch.from_numpy(g['tokens'])
    lengths = []
    for i in range(3):
        layers = om.encode_kv(sd, g[f'i{i}_l1'], g[f'i{i}_l1_xz'], g[f'i{i}_l2'], g[f'i{i}_l2_xz'], g[f'i{i}_biomes'], cfg)
        for j in (0, 2):
            torch.testing.assert_close(layers[j][0][0], torch.from_numpy(g[f'i{i}_k{j}']), atol=1e-5, rtol=1e-5)
            torch.testing.assert_close(layers[j][1][0], torch.from_numpy(g[f'i{i}_v{j}']), atol=1e-5, rtol=1e-5)
        lengths.append(layers[0][0].shape[2])
        got = om.control_forward(sd, tokens[i:i + 1], layers, cfg)[0]
        torch.testing.assert_close(got, torch.from_numpy(g[f'i{i}_logits']), atol=1e-4, rtol=1e-4)
    assert lengths == g['lengths'].tolist()


def test_philox_known_answers():
    """Philox4x32-10 known-answer vectors from the Random123 distribution (kat_vectors)."""
    zero = osm.philox4x32_10(0, 0, 0, 0, 0, 0)
    assert [int(v) for v in zero] == [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]
    ones = osm.philox4x32_10(0xffffffff, 0xffffffff, 0xffffffff, 0xffffffff, 0xffffffff, 0xffffffff)
    assert [int(v) for v in ones] == [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]
    pi = osm.philox4x32_10(0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344, 0xa4093822, 0x299f31d0)
    assert [int(v) for v in pi] == [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]


def _eval_fixture_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location('make_golden', os.path.join(GOLDEN, 'make_golden.py'))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_eval_decoders_match_reference_given_its_draws():
    """The evaluation decoders (`streamvoxel/eval/samplers.py`: random, entropy, mixed, block, native_quarter; linear,
    quartercos, halfcos, reversequarter, front/power and legacy-rounded schedules) reproduce the reference's whole
    decodes: tokens, commit steps and per-step events, given its draws."""
    from oracle import eval_samplers as oes
    mg = _eval_fixture_module()
    g = _load('eval_decode.npz')
    assert int(g['count']) == len(mg.EVAL_SPECS)
    for i, spec in enumerate(mg.EVAL_SPECS):
        step = {'draw': 0, 'noise': 0}

        def draw(i=i):
            key = f'e{i}_s{step["draw"]}_draw'
            step['noise'] = step['draw']
            step['draw'] += 1
            return g[key]

        def noise(k, c, i=i):
            q = g[f'e{i}_s{step["noise"]}_noise']
            assert q.shape == (k, c)
            return q

        order = g[f'e{i}_order'] if f'e{i}_order' in g.files else None
        forward = lambda tokens, t: mg.eval_logits(torch.from_numpy(tokens)).numpy()
        tokens, commit, events = oes.decode(forward, dict(spec), draw, noise, order=order, shape=(16, 8, 8), classes=6)
        assert np.array_equal(tokens, g[f'e{i}_tokens']), spec
        assert np.array_equal(commit, g[f'e{i}_commit']), spec
        keys = [str(k) for k in g[f'e{i}_event_keys']]
        got = np.asarray([[float(ev.get(k, np.nan)) for k in keys] for ev in events])
        np.testing.assert_array_equal(got, g[f'e{i}_events'])


def test_series_log_and_native_draw():
    """The native draw's logarithm (atanh series in single-rounded fp32) is within 4e-7 relative of log over the range
    the draw uses, and the Gumbel-max draw is distributed as softmax(x): 400,000 draws of one 8-class row land within
    five standard errors of p in every class."""
    rng = np.random.default_rng(0)
    a = rng.uniform(2.0 ** -25, 17.0, 200_000).astype(np.float32)
    a = np.concatenate([a, np.float32(1) - np.arange(1, 64, dtype=np.float32) * np.float32(2.0 ** -24)])
    got = osm.series_log(a).astype(np.float64)
    want = np.log(a.astype(np.float64))
    assert np.all(np.abs(got - want) <= 4e-7 * np.maximum(np.abs(want), 2.0 ** -24))
    u = osm.native_uniforms(3, 1, np.arange(4096), 256)
    assert u.min() > 0 and u.max() < 1 and np.all(np.mod(u * 2 ** 24, 2) == 1)
    x = rng.normal(0, 1, (8, 1)).astype(np.float32)
    n = 400_000
    values = osm.native_sample(np.repeat(x, n, 1), np.arange(n), 9, 1)
    p = np.exp(x[:, 0] - x.max())
    p /= p.sum()
    freq = np.bincount(values, minlength=8) / n
    assert np.all(np.abs(freq - p) <= 5 * np.sqrt(p * (1 - p) / n))


@pytest.mark.slow
def test_full_size_forward_matches_reference_fp32():
    """The oracle's fp32 encoder + forward of the full-size config-2 model equals the reference's own
    `engine.unpadded_logits` (fixture `control_full.npz`: 512 voxels x 256 classes) within 1e-4."""
    from streamvoxel_b200 import model as sm, synth
    from streamvoxel_b200.stream.condition import ModelSpec
    g = _load('control_full.npz')
    cfg = sm.dit_b4_control()
    sd = sm.synthetic_state_dict(cfg, seed=0)
    spec = ModelSpec.of(cfg)
    cfgd = dict(num_classes=cfg.classes, voxel_shape=cfg.voxel_shape, patch_size=4, depth=cfg.depth,
                num_heads=cfg.heads, y_range=cfg.y_range, layer_indices=list(cfg.layer_indices),
                biome_halo=cfg.biome_halo, biome_patch=cfg.biome_patch)
    item = synth.item(701, spec, k=2)
    tokens, _ = synth.target_tokens(801, spec)
    assert np.array_equal(tokens, g['tokens'])
    with torch.no_grad():
        kv = om.encode_kv(sd, item.l1_blocks, item.l1_xz, item.l2_blocks, item.l2_xz, item.biomes, cfgd)
        got = om.control_forward(sd, torch.from_numpy(tokens[None]).long(), kv, cfgd)[0]
    torch.testing.assert_close(got.reshape(256, -1)[:, g['voxels']], torch.from_numpy(g['logits']), atol=1e-4,
                               rtol=1e-4)
