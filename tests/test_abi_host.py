"""CPU checks of the boundary and the host logic: libsvx.so loads and exports every function include/svx.h declares,
the ctypes structs match the C layout, and the host-side schedule and weight naming match the reference."""
import ctypes
import os

import numpy as np
import pytest
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')


@pytest.fixture(scope='module')
def lib():
    from streamvoxel_b200 import _lib, build
    build.build()
    return _lib.load()


def test_library_exports_every_header_symbol(lib):
    from streamvoxel_b200 import _lib
    names = _lib.header_symbols()
    assert len(names) >= 19
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(_lib._SIGNATURES), set(names) ^ set(_lib._SIGNATURES)


def test_library_answers_without_a_device(lib):
    assert lib.svx_version() == 1
    if not torch.cuda.is_available():
        assert lib.svx_device_supported() == 0
    assert isinstance(lib.svx_last_error(), bytes)


def test_invalid_arguments_are_rejected_before_any_launch(lib):
    from streamvoxel_b200 import _lib
    status = lib.svx_ease_select(None, None, None, None, None, 1, 256, 16, 16, 3, 256, None, None, 1, None, None,
                                 None, None)
    assert status == _lib.SVX_ERR_INVALID and b'4^3' in lib.svx_last_error()
    with pytest.raises(ValueError):
        _lib.check(status)


def test_ctypes_structs_match_the_c_layout():
    from streamvoxel_b200 import _lib, ops
    assert ctypes.sizeof(_lib.StepParams) == 32 == ops.STEP_DTYPE.itemsize
    assert _lib.EpilogueArgs.bias.offset == 8 and ctypes.sizeof(_lib.EpilogueArgs) == 8 + 5 * 8 + 8 * 4 + 5 * 8
    assert _lib.EpilogueArgs.ln_stats_in.offset == 80 and _lib.EpilogueArgs.ln_stats_out.offset == 112
    assert ctypes.sizeof(_lib.BlockWeights) == 18 * 8 and ctypes.sizeof(_lib.CrossWeights) == 10 * 8
    assert ctypes.sizeof(_lib.EngineWorkspace) == 10 * 8 and ctypes.sizeof(_lib.EngineWeights) == 20 * 8
    assert _lib.EngineConfig.layer_index.offset == 48


def test_host_schedule_matches_reference_fixtures():
    from streamvoxel_b200 import sampling
    g = np.load(os.path.join(GOLDEN, 'schedule.npz'))
    for i in range(int(g['count'])):
        total, steps, n_last = (int(v) for v in g[f's{i}_args'])
        assert sampling.low_entropy_last_quotas(total, steps, n_last) == g[f's{i}_quotas'].tolist()
        assert sampling.counts(total, steps) == g[f's{i}_counts'].tolist()
    assert [sampling.actual_time(f) for f in g['time_in']] == g['time_out'].tolist()


def test_weight_names_and_shapes_match_the_reference_state_dict():
    from streamvoxel_b200 import model as sm
    g = np.load(os.path.join(GOLDEN, 'dit_tiny.npz'))
    ref = {'backbone.' + k[3:]: tuple(g[k].shape) for k in g.files if k.startswith('sd.')}
    cfg = sm.ModelConfig(classes=5, voxel_shape=(16, 16, 16), d=48, heads=4, depth=3, mlp=192, layer_indices=())
    ours = sm.state_dict_shapes(cfg)
    for name, shape in ours.items():
        assert ref.get(name) == shape, name
    unused = {k for k in ref if k not in ours}
    assert all('time_' in k or 'rope' in k or 'patch_centers' in k for k in unused), unused


def test_synthetic_data_follows_the_benchmark_distribution():
    from streamvoxel_b200 import synth
    from streamvoxel_b200.stream.condition import ModelSpec
    spec = ModelSpec(height=256, tile=16, num_classes=256, biome_classes=16, biome_halo=4, y_origin=-64.)
    cells = synth.world(3, 2, 2)
    col = cells[(0, 0)]
    top = (col > 0).sum(0)
    assert top.min() >= 40 - 9 and top.max() <= 120 + 9
    assert set(np.unique(col[:30])) <= set(range(1, 256))
    item = synth.item(5, spec, k=4)
    assert item.l1_blocks.shape == (4, 256, 16, 16) and item.l2_blocks.shape == (80, 256, 16, 16)
    assert item.biomes.shape == (64, 12, 12) and item.biomes[:, :3].sum() == 0
    logits, truth = synth.ease_logits(0, 2, classes=8, voxels=1000)
    assert logits.shape == (2, 8, 1000) and truth.shape == (2, 1000)


def _lpt_makespan(costs, ctas):
    """Longest-processing-time assignment restated in Python: each unit, largest first, to the least-loaded CTA."""
    import heapq
    heap = [(0, c) for c in range(ctas)]
    for cost in sorted(costs, reverse=True):
        load, c = heapq.heappop(heap)
        heapq.heappush(heap, (load + cost, c))
    return max(load for load, _ in heap)


@pytest.mark.parametrize('lengths, heads, queries, ctas', [
    ([2368, 3392, 2368, 9536, 4416, 4416, 6464, 9536], 8, 1024, 148),   # the bench's eight slots
    ([0, 96, 97, 9600], 8, 1024, 148),
    ([577, 0, 577, 1280], 2, 384, 5),                                     # odd query tiles, fewer CTAs than units
    (None, 4, 256, 300),                                                  # more CTAs than units
])
def test_attention_plan_partitions_units_longest_first(lib, lengths, heads, queries, ctas):
    """svx_attention_plan assigns every (slot, head, query-pair) unit to exactly one CTA, with a makespan between
    the lower bound and that of the longest-processing-time rule."""
    from streamvoxel_b200 import ops
    slots = 4 if lengths is None else len(lengths)
    keys = 9600
    plan, grid = ops.attention_plan(lengths, slots, heads, queries, keys, ctas)
    pairs = (queries // 128 + 1) // 2
    units = slots * heads * pairs
    assert grid == min(ctas, units) and plan.numel() == grid + 1 + units
    offsets, ids = plan[:grid + 1].tolist(), plan[grid + 1:].tolist()
    assert offsets[0] == 0 and offsets[-1] == units and all(a <= b for a, b in zip(offsets, offsets[1:]))
    assert sorted(ids) == list(range(units))
    lens = [keys] * slots if lengths is None else lengths
    cost = [(4 * t + 8 if t else 1) for t in ((lens[u // (heads * pairs)] + 95) // 96 for u in range(units))]
    loads = [sum(cost[u] for u in ids[offsets[c]:offsets[c + 1]]) for c in range(grid)]
    assert max(max(cost), -(-sum(cost) // grid)) <= max(loads) <= _lpt_makespan(cost, grid)
    for c in range(grid):   # each CTA's units longest first
        own = [cost[u] for u in ids[offsets[c]:offsets[c + 1]]]
        assert own == sorted(own, reverse=True)


def test_attention_plan_rejects_bad_shapes_and_small_buffers(lib):
    from streamvoxel_b200 import _lib
    assert lib.svx_attention_plan_ints(2, 8, 1000, 148) == 0   # queries not a multiple of 128
    buf = (ctypes.c_int32 * 4)()
    assert lib.svx_attention_plan(None, 2, 8, 1024, 4096, 148, buf, 4) == _lib.SVX_ERR_INVALID


def test_attention_plan_balances_the_bench_lengths(lib):
    """For the bench's eight slots the boustrophedon order gives a makespan of 125 key tiles (+2 units) against an
    average of 96.4; the plan's makespan (key tiles + 2 per unit) stays within 9% of its average (the longest unit
    alone is 102)."""
    from streamvoxel_b200 import ops
    lengths = [2368, 3392, 2368, 9536, 4416, 4416, 6464, 9536]
    plan, grid = ops.attention_plan(lengths, 8, 8, 1024, 9600, 148)
    offsets, ids = plan[:grid + 1].tolist(), plan[grid + 1:].tolist()
    tiles = [(lengths[u // 32] + 95) // 96 + 2 for u in range(256)]
    loads = [sum(tiles[u] for u in ids[offsets[c]:offsets[c + 1]]) for c in range(grid)]
    assert max(loads) <= 1.09 * sum(loads) / grid


def test_attention_multi_plan_covers_both_problems(lib):
    """The joint plan of a cross-attention (bench lengths) and a self-attention assigns all 512 units once, problem
    0 first in the numbering, and balances better than the two launches' makespans added (108 + 26 unit costs)."""
    from streamvoxel_b200 import ops
    lengths = [2368, 3392, 2368, 9536, 4416, 4416, 6464, 9536]
    plan, grid = ops.attention_multi_plan([(lengths, 9600), (None, 1024)], 8, 8, 1024, 148)
    offsets, ids = plan[:grid + 1].tolist(), plan[grid + 1:].tolist()
    assert grid == 148 and sorted(ids) == list(range(512))
    tiles = [((lengths[u // 32] if u < 256 else 1024) + 95) // 96 + 2 for u in range(512)]
    loads = [sum(tiles[u] for u in ids[offsets[c]:offsets[c + 1]]) for c in range(grid)]
    assert max(loads) < 108 + 26 and sum(loads) / grid > 0.93 * max(loads)
    assert lib.svx_attention_multi_plan_ints(3, 8, 8, 1024, 148) == 0


def test_layernorm_fold_algebra_matches_layernorm_then_linear():
    """The host half of the LayerNorm fold: with W' = fold_layernorm(W, b, 1 + scale, shift), the epilogue formula
    r (x W'^T - mu u) + v equals LayerNorm -> modulate -> linear (float64, up to the bf16 rounding of W')."""
    from streamvoxel_b200.model import fold_layernorm
    g = torch.Generator().manual_seed(3)
    m, k, n = 64, 768, 96
    x = torch.randn((m, k), generator=g, dtype=torch.float64) * 0.7 + 0.3
    w = (torch.randn((n, k), generator=g) * 0.03).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
    ops_ = (1 + torch.randn(k, generator=g) * 0.2).to(torch.bfloat16)
    shift = (torch.randn(k, generator=g) * 0.2).to(torch.bfloat16)
    wf, u, v = fold_layernorm(w, b, ops_, shift)
    assert wf.dtype == torch.bfloat16 and u.dtype == v.dtype == torch.float32
    mu = x.mean(1, keepdim=True)
    r = 1 / torch.sqrt(x.var(1, unbiased=False, keepdim=True) + 1e-6)
    got = r * (x @ wf.double().t() - mu * u.double()) + v.double()
    want = ((x - mu) * r * ops_.double() + shift.double()) @ w.double().t() + b.double()
    torch.testing.assert_close(got, want, atol=1e-2, rtol=1e-2)   # W' rounded to bf16 (as h is, unfolded)
    exact = r * (x @ (w.double() * ops_.double()).t() - mu * (w.double() * ops_.double()).sum(1)) + v.double()
    torch.testing.assert_close(exact, want, atol=1e-7, rtol=1e-6)   # the identity itself (float64 rounding only)
    wf0, u0, v0 = fold_layernorm(w, b)   # LayerNorm without affine
    assert torch.equal(wf0, w) and torch.equal(v0, b.float())


def test_down_conv_as_gemm_layout():
    """The L2 down-conv of the condition encoder (`streaming_controlnet.py:148`, Conv3d 4^3 stride 4 over the
    patchified column) equals the GEMM the encoder runs: the [n H/16, 64 d] view of the patchified rows times
    `down_conv_weight` (float64, CPU)."""
    from streamvoxel_b200.model import down_conv_weight
    g = torch.Generator().manual_seed(5)
    n, h, d = 3, 8, 16                                   # columns, patch layers (y), channels; 4 x 4 patches per layer
    x = torch.randn((n * h * 16, d), generator=g, dtype=torch.float64)   # rows in patch order (y, z, x)
    w = (torch.randn((d, d, 4, 4, 4), generator=g) * 0.1).to(torch.bfloat16).double()
    grid = x.reshape(n, h, 4, 4, d).permute(0, 4, 1, 2, 3)
    want = torch.nn.functional.conv3d(grid, w, None, stride=4).flatten(2).transpose(1, 2).reshape(-1, d)
    got = x.view(n * h // 4, 64 * d) @ down_conv_weight(w).double().t()
    torch.testing.assert_close(got, want, atol=1e-12, rtol=1e-12)


def test_grouped_gemm_validates_before_any_launch(lib):
    """`svx_gemm_group` takes two gated residuals with row statistics and 256-row multiples, checked on the host
    before any CUDA call."""
    from streamvoxel_b200 import _lib
    fake = 1 << 20   # never dereferenced: the checks fail first
    good = _lib.EpilogueArgs(epilogue=_lib.EPI_GATE_RESIDUAL, bias=fake, gate=fake, residual=fake, ln_stats_out=fake)
    plain = _lib.EpilogueArgs(epilogue=_lib.EPI_RESIDUAL, bias=fake, residual=fake, ln_stats_out=fake)
    p = ctypes.c_void_p(fake)
    for a, b, m in ((good, plain, 256), (good, good, 384)):
        status = lib.svx_gemm_group(p, p, p, ctypes.byref(a), p, p, p, ctypes.byref(b), m, 768, 768, None)
        assert status == _lib.SVX_ERR_INVALID and b'gemm group' in lib.svx_last_error()


def test_row_statistics_merge_restated():
    """The kernels' chunk statistics and their merge, restated in numpy: per 32-column chunk (mean, M2); the row's mean
    and variance from shifted sums about the first chunk's mean (`row_norm` in gemm.cu) equal the two-pass values,
    also when the row's mean is far larger than its spread."""
    rng = np.random.default_rng(5)
    for offset in (0.0, 50.0):
        x = (rng.standard_normal((16, 768)) * 0.5 + offset).astype(np.float32)
        c = x.reshape(16, 24, 32).astype(np.float64)
        mean_c, m2_c = c.mean(-1), ((c - c.mean(-1, keepdims=True)) ** 2).sum(-1)
        d = mean_c - mean_c[:, :1]
        dm = d.sum(1) / 24
        mean = mean_c[:, 0] + dm
        var = (m2_c + 32 * d * d).sum(1) / 768 - dm * dm
        np.testing.assert_allclose(mean, x.astype(np.float64).mean(1), rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(var, x.astype(np.float64).var(1), rtol=1e-9)
