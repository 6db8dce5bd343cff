"""Per-kernel parity of libsvx on the GPU, through the C-ABI (streamvoxel_b200.ops), against the CPU oracle.

Tolerances: integer/index results (selection, marking, sampling given identical inputs) are exact; entropy within
1e-5 abs (the contract of the EASE scores); bf16 GEMM/attention outputs within 1e-2 abs + 1e-2 rel of an fp32
reference rounded at the same points (one bf16 ulp at the magnitudes used).
"""
import os

import numpy as np
import pytest
import torch

from oracle import sampler as osm

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')


@pytest.fixture(scope='module')
def ops():
    from streamvoxel_b200 import _lib, ops
    _lib.require_device()
    return ops


def _bf16(x):
    return x.bfloat16().float()


# ---------------------------------------------------------------------------------------------- EASE

@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_entropy_scores_match_oracle(ops, dtype):
    g = torch.Generator().manual_seed(0)
    logits = (torch.randn((3, 256, 64, 16, 16), generator=g) * 2).to(dtype)
    logits[:, 7] += 6.0
    got = ops.ease_scores(logits.cuda().contiguous()).cpu()
    want = np.stack([osm.entropy_scores(logits[i].float().numpy()) for i in range(3)])
    np.testing.assert_allclose(got.numpy(), want, atol=1e-5, rtol=0)


def test_marking_matches_oracle(ops):
    g = np.load(os.path.join(GOLDEN, 'scores.npz'))
    for i in range(int(g['count'])):
        logits = torch.from_numpy(g[f'e{i}_logits'])[None].contiguous()
        if logits[0, 0].numel() % 4:
            continue
        last, count = ops.ease_mark(logits.cuda(), (0,), float(g[f'e{i}_eps']))
        assert np.array_equal(last[0].cpu().numpy().astype(bool), g[f'e{i}_last']), i
        assert int(count[0]) == int(g[f'e{i}_last'].sum())


def _select_inputs(score, selectable, last, mask_id=256):
    tokens = np.where(selectable | last, mask_id, 0).astype(np.int16)
    return tokens


def test_selection_matches_reference_fixtures(ops):
    """The kernel fed the reference's scores selects exactly the reference's voxels (`block_quota_select`)."""
    g = np.load(os.path.join(GOLDEN, 'quota_select.npz'))
    for i in range(int(g['count'])):
        p = f'c{i}_'
        score, selectable, last = g[p + 'score'], g[p + 'selectable'], g[p + 'last']
        k, committed, frac = int(g[p + 'k']), int(g[p + 'committed']), float(g[p + 'frac'])
        order = g[p + 'order']
        pos = np.empty_like(order)
        pos[order] = np.arange(len(order))
        tokens = _select_inputs(score, selectable, last)
        params = ops.step_params([(k, 1, committed, frac, 0)], 'cuda')
        status = torch.zeros(1, dtype=torch.int32, device='cuda')
        chosen, index, count = ops.ease_select(
            torch.from_numpy(score)[None].cuda(), torch.from_numpy(tokens)[None].cuda(),
            torch.from_numpy(last.astype(np.uint8))[None].cuda(), torch.from_numpy(pos.astype(np.int32))[None].cuda(),
            params, 256, max(k, 1), status=status)
        want = g[p + 'chosen']
        assert np.array_equal(chosen[0].cpu().numpy().astype(bool), want), i
        assert int(count[0]) == k and int(status[0]) == 0
        assert np.array_equal(index[0, :k].cpu().numpy(), np.flatnonzero(want)), i


@pytest.mark.parametrize('seed', range(4))
def test_selection_full_size_batch_matches_oracle(ops, seed):
    """8 slots of full-size columns in one launch, including steps that need the global trim / top-up."""
    rng = np.random.default_rng(seed)
    shape, slots = (256, 16, 16), 8
    scores, tokens, lasts, poss, rows, wants = [], [], [], [], [], []
    for s in range(slots):
        tops = rng.integers(40, 256, (16, 16))
        last = np.arange(256)[:, None, None] >= tops[None]
        committed_mask = ~last & (rng.random(shape) < rng.random())
        selectable = ~last & ~committed_mask
        k = int(rng.integers(1, max(2, int(selectable.sum()))))
        committed = int(committed_mask.sum())
        frac = (committed + k) / int((~last).sum())
        if s % 3 == 1:   # break the invariant so the clamped quotas miss k and the fix-up runs
            frac = min(1.0, frac * 1.3)
        order = rng.permutation(1024)
        score = rng.standard_normal(shape).astype(np.float32)
        if s % 2:
            score = np.round(score * 2) / 2   # ties inside blocks
        n_total = osm.block_view(~last, 4).sum(1)
        pos = np.empty_like(order)
        pos[order] = np.arange(1024)
        want = osm.block_quota_select(score, selectable, k, 4, order, frac, n_total)
        scores.append(score); tokens.append(_select_inputs(score, selectable, last)); lasts.append(last)
        poss.append(pos); rows.append((k, 1, committed, frac, seed)); wants.append(want)
    params = ops.step_params(rows, 'cuda')
    cap = max(r[0] for r in rows)
    status = torch.zeros(slots, dtype=torch.int32, device='cuda')
    chosen, index, count = ops.ease_select(
        torch.from_numpy(np.stack(scores)).cuda(), torch.from_numpy(np.stack(tokens)).cuda(),
        torch.from_numpy(np.stack(lasts).astype(np.uint8)).cuda(), torch.from_numpy(np.stack(poss).astype(np.int32)).cuda(),
        params, 256, cap, status=status)
    chosen = chosen.cpu().numpy().astype(bool)
    for s in range(slots):
        assert np.array_equal(chosen[s], wants[s]), s
        assert int(count[s]) == rows[s][0]
    assert int(status.sum()) == 0


def test_softmax_rows_bitwise_equal_torch(ops):
    """The parity-mode softmax reproduces torch's CUDA `softmax(-1)` bit for bit (the multinomial's input)."""
    g = torch.Generator(device='cuda').manual_seed(3)
    for classes in (256, 6, 33, 1000, 1):
        x = torch.randn((4099, classes), device='cuda', generator=g) * 3
        assert torch.equal(ops.softmax_rows(x), x.softmax(-1)), classes


@pytest.mark.parametrize('classes', [256, 6])
def test_parity_sampling_equals_torch_multinomial(ops, classes):
    """Given the slot generator, the kernel's draw equals `torch.multinomial(softmax(x), 1, generator)`."""
    torch.manual_seed(0)
    voxels, k = 4096, 777
    logits = (torch.randn((1, classes, voxels), device='cuda') * 2).contiguous()
    idx = torch.sort(torch.randperm(voxels, device='cuda')[:k]).values.int()
    gen = torch.Generator(device='cuda').manual_seed(1234)
    clone = torch.Generator(device='cuda').set_state(gen.get_state())
    probs = logits[0][:, idx.long()].t().contiguous().float().softmax(-1)
    want = torch.multinomial(probs, 1, generator=clone).squeeze(-1)
    noise = torch.empty((k, classes), device='cuda').exponential_(generator=gen)
    assert torch.equal(gen.get_state(), clone.get_state())
    tokens = torch.full((1, voxels), classes, dtype=torch.int16, device='cuda')
    params = ops.step_params([(k, 1, 0, 0.0, 0)], 'cuda')
    values = ops.ease_sample(logits, idx[None].contiguous(), params, tokens, noise=noise[None].contiguous())
    assert torch.equal(values[0].long(), want)
    assert torch.equal(tokens[0, idx.long()].long(), want)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_native_sampling_equals_oracle_bit_for_bit(ops, dtype):
    """The native Gumbel-max draw (Philox + the atanh-series logs in single-rounded fp32) equals the oracle's
    restatement for every chosen voxel, at full size (2048 of 65536 voxels, V = 256) and with V = 6."""
    torch.manual_seed(1)
    for classes, voxels, k in ((256, 65536, 2048), (6, 1024, 300)):
        logits = (torch.randn((1, classes, voxels), device='cuda') * 2).to(dtype).contiguous()
        idx = torch.sort(torch.randperm(voxels, device='cuda')[:k]).values.int()
        tokens = torch.full((1, voxels), classes, dtype=torch.int16, device='cuda')
        seed, step = 0x1234567890ABCDEF, 7
        params = ops.step_params([(k, step, 0, 0.0, seed)], 'cuda')
        values = ops.ease_sample(logits, idx[None].contiguous(), params, tokens)[0].cpu().numpy()
        cols = logits[0].float().cpu().numpy()[:, idx.cpu().numpy()]
        want = osm.native_sample(cols, idx.cpu().numpy(), seed, step)
        assert np.array_equal(values, want), float((values == want).mean())
        assert np.array_equal(tokens[0, idx.long()].cpu().numpy(), want)


# ---------------------------------------------------------------------------------------------- forward ops

def _linear_ref(a, w, b):
    return _bf16(a.float() @ w.float().t() + b.float())


@pytest.mark.parametrize('m,n,k', [(256, 576, 192), (1024, 768, 768), (8192, 2304, 768), (2048, 768, 3072),
                                   (1024, 3072, 768), (384, 768, 256), (512, 1152, 256)])
def test_gemm_bias_matches_fp32(ops, m, n, k):
    torch.manual_seed(m + n + k)
    a = (torch.randn((m, k), device='cuda') * 0.5).bfloat16()
    w = (torch.randn((n, k), device='cuda') * 0.05).bfloat16()
    b = (torch.randn(n, device='cuda') * 0.1).bfloat16()
    got = ops.gemm(a, w, b).float()
    want = _linear_ref(a, w, b)
    torch.testing.assert_close(got, want, atol=1e-2, rtol=1e-2)
    assert (got - want).abs().mean() < 1e-3


def test_gemm_fused_epilogues(ops):
    from streamvoxel_b200 import _lib
    torch.manual_seed(0)
    m, n, k = 512, 768, 384
    a = (torch.randn((m, k), device='cuda') * 0.5).bfloat16()
    w = (torch.randn((n, k), device='cuda') * 0.05).bfloat16()
    b = (torch.randn(n, device='cuda') * 0.1).bfloat16()
    gate = (torch.randn(n, device='cuda') * 0.5).bfloat16()
    res = torch.randn((m, n), device='cuda').bfloat16()
    y = _linear_ref(a, w, b)
    got = ops.gemm(a, w, b, _lib.EPI_BIAS_GELU).float()
    torch.testing.assert_close(got, _bf16(torch.nn.functional.gelu(y)), atol=1e-2, rtol=1e-2)
    got = ops.gemm(a, w, b, _lib.EPI_GATE_RESIDUAL, gate=gate, residual=res.clone()).float()
    torch.testing.assert_close(got, _bf16(res.float() + _bf16(gate.float() * y)), atol=2e-2, rtol=1e-2)
    got = ops.gemm(a, w, b, _lib.EPI_RESIDUAL, residual=res.clone()).float()
    torch.testing.assert_close(got, _bf16(res.float() + y), atol=2e-2, rtol=1e-2)
    inplace = res.clone()
    ops.gemm(a, w, b, _lib.EPI_RESIDUAL, residual=inplace, out=inplace)
    torch.testing.assert_close(inplace.float(), _bf16(res.float() + y), atol=2e-2, rtol=1e-2)


def test_gemm_rope_epilogue_matches_oracle_rope(ops):
    from oracle import model as om
    from oracle.model import Precision
    from streamvoxel_b200 import _lib
    torch.manual_seed(2)
    heads, patches, slots = 2, 256, 2
    d = heads * 96
    m, k = slots * patches, 192
    a = (torch.randn((m, k), device='cuda') * 0.5).bfloat16()
    w = (torch.randn((3 * d, k), device='cuda') * 0.05).bfloat16()
    b = (torch.randn(3 * d, device='cuda') * 0.1).bfloat16()
    positions = om.patch_centers_xyz((64, 16, 16), 4) / 4
    phase = positions[:, :, None] * om.rope_frequencies(96)
    sin, cos = phase.sin().reshape(patches, 48).bfloat16().cuda(), phase.cos().reshape(patches, 48).bfloat16().cuda()
    got = ops.gemm(a, w, b, _lib.EPI_ROPE, rope=(sin, cos), rope_cols=2 * d, rows_per_slot=patches).float().cpu()
    y = _linear_ref(a, w, b).cpu().reshape(slots, patches, 3, heads, 96)
    p = Precision(True)
    want = []
    for part in range(3):
        t = y[:, :, part].transpose(1, 2)
        if part < 2:
            t = om.rope(t, positions[None].expand(slots, -1, -1), om.rope_frequencies(96), p)
        want.append(t.transpose(1, 2))
    want = torch.stack(want, 2).reshape(m, 3 * d)
    torch.testing.assert_close(got, want, atol=1e-2, rtol=1e-2)


def test_gemm_class_major_head_layout(ops):
    from streamvoxel_b200 import _lib
    torch.manual_seed(3)
    shape, classes, slots = (64, 16, 16), 32, 2
    patches = 16 * 4 * 4
    m, k = slots * patches, 192
    a = (torch.randn((m, k), device='cuda') * 0.5).bfloat16()
    w = (torch.randn((64 * classes, k), device='cuda') * 0.05).bfloat16()   # reference order n = o * V + v
    b = (torch.randn(64 * classes, device='cuda') * 0.1).bfloat16()
    # kernel order n' = v * 64 + o
    w2 = w.reshape(64, classes, k).transpose(0, 1).reshape(64 * classes, k).contiguous()
    b2 = b.reshape(64, classes).t().reshape(-1).contiguous()
    got = ops.gemm(a, w2, b2, _lib.EPI_CLASS_MAJOR, rows_per_slot=patches, classes=classes, geometry=shape).float()
    y = _linear_ref(a, w, b)
    want = y.reshape(slots, 16, 4, 4, 4, 4, 4, classes).permute(0, 7, 1, 4, 2, 5, 3, 6).reshape(slots, classes, *shape)
    torch.testing.assert_close(got, want, atol=1e-2, rtol=1e-2)


def test_attention_self_and_varlen_cross(ops):
    torch.manual_seed(4)
    slots, heads, n, d = 3, 2, 256, 192
    qkv = (torch.randn((slots * n, 3 * d), device='cuda')).bfloat16()
    got = ops.attention(qkv, qkv[:, d:], qkv[:, 2 * d:], slots, heads, n, n, q_row_stride=3 * d,
                        kv_slot_stride=n * 3 * d, kv_head_stride=96, kv_row_stride=3 * d).float()
    q, k_, v = qkv.float().reshape(slots, n, 3, heads, 96).unbind(2)
    want = torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), k_.transpose(1, 2), v.transpose(1, 2))
    want = want.transpose(1, 2).reshape(slots * n, d)
    torch.testing.assert_close(got, want, atol=1e-2, rtol=1e-2)
    cap = 1280
    kc = torch.randn((slots, heads, cap, 96), device='cuda').bfloat16()
    vc = torch.randn((slots, heads, cap, 96), device='cuda').bfloat16()
    lengths = torch.tensor([84, 1280, 577], dtype=torch.int32, device='cuda')
    qx = torch.randn((slots * n, d), device='cuda').bfloat16()
    got = ops.attention(qx, kc, vc, slots, heads, n, cap, q_row_stride=d, kv_slot_stride=heads * cap * 96,
                        kv_head_stride=cap * 96, kv_row_stride=96, lengths=lengths).float()
    for s in range(slots):
        L = int(lengths[s])
        qs = qx[s * n:(s + 1) * n].float().reshape(n, heads, 96).transpose(0, 1)
        want = torch.nn.functional.scaled_dot_product_attention(qs, kc[s, :, :L].float(), vc[s, :, :L].float())
        torch.testing.assert_close(got[s * n:(s + 1) * n], want.transpose(0, 1).reshape(n, d), atol=1e-2, rtol=1e-2)


def test_attention_plan_changes_only_the_schedule(ops):
    """A host-built work plan (LPT/MULTIFIT over the slots' key lengths), a stale plan built for other lengths and a
    plan for a small grid give bitwise the output of the default order: a plan moves units between CTAs, and each
    unit's arithmetic does not depend on its CTA."""
    torch.manual_seed(21)
    slots, heads, n, cap = 5, 8, 1024, 4096
    d = heads * 96
    kc = torch.randn((slots, heads, cap, 96), device='cuda').bfloat16()
    vc = torch.randn((slots, heads, cap, 96), device='cuda').bfloat16()
    host = [4096, 96, 0, 2500, 1000]
    lengths = torch.tensor(host, dtype=torch.int32, device='cuda')
    qx = (torch.randn((slots * n, d), device='cuda') * 1.5).bfloat16()
    run = lambda plan=None: ops.attention(qx, kc, vc, slots, heads, n, cap, q_row_stride=d,
                                          kv_slot_stride=heads * cap * 96, kv_head_stride=cap * 96, kv_row_stride=96,
                                          lengths=lengths, plan=plan)
    base = run()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for plan_lengths, ctas in ((host, sms), (None, sms), (host, 7)):
        got = run(ops.attention_plan(plan_lengths, slots, heads, n, cap, ctas, 'cuda'))
        assert torch.equal(got, base), (plan_lengths, ctas)
    for s in (0, 3):
        L = host[s]
        qs = qx[s * n:(s + 1) * n].float().reshape(n, heads, 96).transpose(0, 1)
        want = torch.nn.functional.scaled_dot_product_attention(qs, kc[s, :, :L].float(), vc[s, :, :L].float())
        torch.testing.assert_close(base[s * n:(s + 1) * n].float(), want.transpose(0, 1).reshape(n, d), atol=1e-2,
                                   rtol=1e-2)
    assert torch.count_nonzero(base[2 * n:3 * n]) == 0


def test_attention_multi_equals_separate_launches(ops):
    """The joint launch of a varlen cross-attention and a self-attention over the same slots (the engine's control
    layer) gives each problem bitwise the output of its own launch, with a joint plan and a stale one."""
    torch.manual_seed(22)
    slots, heads, n, cap = 3, 8, 1024, 2048
    d = heads * 96
    kc = torch.randn((slots, heads, cap, 96), device='cuda').bfloat16()
    vc = torch.randn((slots, heads, cap, 96), device='cuda').bfloat16()
    host = [2048, 0, 700]
    lengths = torch.tensor(host, dtype=torch.int32, device='cuda')
    qx = (torch.randn((slots * n, d), device='cuda') * 1.5).bfloat16()
    qkv = (torch.randn((slots * n, 3 * d), device='cuda') * 1.5).bfloat16()
    cross = dict(q=qx, k=kc, v=vc, keys=cap, q_row_stride=d, kv_slot_stride=heads * cap * 96, kv_head_stride=cap * 96,
                 kv_row_stride=96, lengths=lengths)
    self_ = dict(q=qkv, k=qkv[:, d:], v=qkv[:, 2 * d:], keys=n, q_row_stride=3 * d, kv_slot_stride=n * 3 * d,
                 kv_head_stride=96, kv_row_stride=3 * d)
    alone = [ops.attention(p['q'], p['k'], p['v'], slots, heads, n, p['keys'], q_row_stride=p['q_row_stride'],
                           kv_slot_stride=p['kv_slot_stride'], kv_head_stride=p['kv_head_stride'],
                           kv_row_stride=p['kv_row_stride'], lengths=p.get('lengths')) for p in (cross, self_)]
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for plan_lengths, ctas in ((host, sms), (None, sms), (host, 5)):
        plan = ops.attention_multi_plan([(plan_lengths, cap), (None, n)], slots, heads, n, ctas, 'cuda')
        outs = [torch.full((slots * n, d), 7.0, device='cuda').bfloat16() for _ in range(2)]
        ops.attention_multi([dict(cross, out=outs[0]), dict(self_, out=outs[1])], slots, heads, n, plan)
        assert torch.equal(outs[0], alone[0]) and torch.equal(outs[1], alone[1]), (plan_lengths, ctas)


def test_attention_odd_query_tiles_ties_and_empty_slots(ops):
    """384 queries (a CTA with one query tile), tied and zero key lengths, and logits large enough to raise the
    exponent base several times within a row."""
    torch.manual_seed(14)
    slots, heads, n, d = 4, 2, 384, 192
    qkv = (torch.randn((slots * n, 3 * d), device='cuda') * 2.5).bfloat16()
    got = ops.attention(qkv, qkv[:, d:], qkv[:, 2 * d:], slots, heads, n, n, q_row_stride=3 * d,
                        kv_slot_stride=n * 3 * d, kv_head_stride=96, kv_row_stride=3 * d).float()
    q, k_, v = qkv.float().reshape(slots, n, 3, heads, 96).unbind(2)
    want = torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), k_.transpose(1, 2), v.transpose(1, 2))
    torch.testing.assert_close(got, want.transpose(1, 2).reshape(slots * n, d), atol=2e-2, rtol=2e-2)
    cap = 1280
    kc = (torch.randn((slots, heads, cap, 96), device='cuda') * 2.0).bfloat16()
    vc = torch.randn((slots, heads, cap, 96), device='cuda').bfloat16()
    lengths = torch.tensor([577, 0, 577, 1280], dtype=torch.int32, device='cuda')
    qx = (torch.randn((slots * n, d), device='cuda') * 2.0).bfloat16()
    got = ops.attention(qx, kc, vc, slots, heads, n, cap, q_row_stride=d, kv_slot_stride=heads * cap * 96,
                        kv_head_stride=cap * 96, kv_row_stride=96, lengths=lengths).float()
    for s in range(slots):
        L = int(lengths[s])
        if L == 0:
            assert torch.count_nonzero(got[s * n:(s + 1) * n]) == 0
            continue
        qs = qx[s * n:(s + 1) * n].float().reshape(n, heads, 96).transpose(0, 1)
        want = torch.nn.functional.scaled_dot_product_attention(qs, kc[s, :, :L].float(), vc[s, :, :L].float())
        torch.testing.assert_close(got[s * n:(s + 1) * n], want.transpose(0, 1).reshape(n, d), atol=2e-2, rtol=2e-2)


def test_attention_key_length_edges(ops):
    """Cross-attention at the engine's key capacity (9600 = 100 key tiles of 96) with a single key, exactly one tile,
    one key into a second tile, one key short of the capacity and the whole capacity."""
    torch.manual_seed(21)
    heads, n, d, cap = 2, 256, 192, 9600
    lengths_list = [1, 96, 97, 9599, 9600]
    slots = len(lengths_list)
    kc = (torch.randn((slots, heads, cap, 96), device='cuda') * 1.5).bfloat16()
    vc = torch.randn((slots, heads, cap, 96), device='cuda').bfloat16()
    lengths = torch.tensor(lengths_list, dtype=torch.int32, device='cuda')
    qx = (torch.randn((slots * n, d), device='cuda') * 1.5).bfloat16()
    got = ops.attention(qx, kc, vc, slots, heads, n, cap, q_row_stride=d, kv_slot_stride=heads * cap * 96,
                        kv_head_stride=cap * 96, kv_row_stride=96, lengths=lengths).float()
    for s, L in enumerate(lengths_list):
        qs = qx[s * n:(s + 1) * n].float().reshape(n, heads, 96).transpose(0, 1)
        want = torch.nn.functional.scaled_dot_product_attention(qs, kc[s, :, :L].float(), vc[s, :, :L].float())
        torch.testing.assert_close(got[s * n:(s + 1) * n], want.transpose(0, 1).reshape(n, d), atol=2e-2, rtol=2e-2)
    # One key: every query's output is that key's value row, to within one bf16 ulp (measured: about one row in seven
    # comes out scaled by a factor within 2^-8 of 1, so some of its elements round to the neighbouring bf16 value).
    single = vc[0, :, 0].float()
    torch.testing.assert_close(got[:n].reshape(n, heads, 96), single[None].expand(n, heads, 96), atol=0,
                               rtol=2 ** -7 + 1e-6)


def test_layernorm_modulate(ops):
    torch.manual_seed(5)
    for d in (192, 768):
        x = torch.randn((1000, d), device='cuda').bfloat16()
        ops_ = (1 + torch.randn(d, device='cuda') * 0.1).bfloat16()
        shift = (torch.randn(d, device='cuda') * 0.1).bfloat16()
        got = ops.layernorm_modulate(x, 1e-6, ops_, shift).float()
        ln = torch.nn.functional.layer_norm(x.float(), (d,), eps=1e-6)
        torch.testing.assert_close(got, _bf16(ln * ops_.float() + shift.float()), atol=1e-2, rtol=1e-2)
        got = ops.layernorm_modulate(x, 1e-6).float()
        torch.testing.assert_close(got, _bf16(ln), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize('d', [192, 768])
def test_layernorm_affine_matches_torch(ops, d):
    """The condition encoder's LayerNorms on `svx_layernorm_affine`: l2_norm (fp32 affine, eps 1e-5) + GELU(erf), and
    + type/size embeddings then the no-affine context_norm (eps 1e-6), against torch fp32 rounded once to bf16; in
    place (out = x) as the encoder runs it."""
    F = torch.nn.functional
    torch.manual_seed(21)
    rows = 300
    x = (torch.randn((rows, d), device='cuda') * 0.7 + 0.1).bfloat16()
    w = torch.randn(d, device='cuda') * 0.5 + 1
    b = torch.randn(d, device='cuda') * 0.2
    pre = torch.randn(d, device='cuda') * 0.3
    got = ops.layernorm_affine(x, 1e-5, weight=w, bias=b, gelu=True).float()
    torch.testing.assert_close(got, _bf16(F.gelu(F.layer_norm(x.float(), (d,), w, b, 1e-5))), atol=1e-2, rtol=1e-2)
    got = ops.layernorm_affine(x, 1e-6, pre=pre).float()
    torch.testing.assert_close(got, _bf16(F.layer_norm(x.float() + pre, (d,), eps=1e-6)), atol=1e-2, rtol=1e-2)
    y = x.clone()
    ops.layernorm_affine(y, 1e-6, pre=pre, out=y)
    assert torch.equal(y.float(), got)


def test_patch_embed_matches_gather(ops):
    from oracle import model as om
    from oracle.model import Precision
    torch.manual_seed(6)
    classes, d, shape = 31, 192, (64, 16, 16)
    sd = {'t.weight': torch.randn((d, classes + 1, 4, 4, 4)) * 0.05, 't.bias': torch.randn(d) * 0.1}
    tokens = torch.randint(0, classes + 1, (2, *shape))
    p = Precision(True)
    want = om.patchify(sd, 't', tokens, classes, p)
    add = (torch.randn((256, d)) * 0.1).bfloat16()
    want = _bf16(want + add.float()[None])
    table = sd['t.weight'].permute(1, 2, 3, 4, 0).reshape(-1, d).bfloat16().contiguous().cuda()
    out_b, out_c = ops.patch_embed(tokens.to(torch.int16).cuda(), classes, table, sd['t.bias'].bfloat16().cuda(),
                                   add.cuda(), table, sd['t.bias'].bfloat16().cuda(), add.cuda())
    torch.testing.assert_close(out_b.float().cpu().reshape(2, 256, d), want, atol=1e-2, rtol=1e-2)
    assert torch.equal(out_b, out_c)


@pytest.mark.parametrize('seed', [0, 1, 2])
def test_eval_select_full_size_matches_oracle(ops, seed):
    """`svx_eval_select` on full-size columns (256 x 16 x 16, 1024 blocks, one slot per mode, tied scores and draws)
    equals the oracle's random / entropy / mixed / block / threshold selections voxel for voxel."""
    from oracle import eval_samplers as oes
    rng = np.random.default_rng(seed)
    shape, classes, slots = (256, 16, 16), 256, 5
    total = int(np.prod(shape))
    tokens = np.where(rng.random((slots, *shape)) < rng.uniform(0.2, 0.9, (slots, 1, 1, 1)),
                      classes, rng.integers(0, classes, (slots, *shape))).astype(np.int16)
    scores = (np.round(rng.standard_normal((slots, *shape)) * 4) / 4).astype(np.float32)   # many ties
    draw = (np.round(rng.random((slots, *shape)) * 512) / 512).astype(np.float32)
    orders = [rng.permutation(total // 64) for _ in range(slots)]
    rows, want = [], []
    for s in range(slots):
        mask = tokens[s] == classes
        m = int(mask.sum())
        mode = ['random', 'entropy', 'mixed', 'block', 'threshold'][s]
        q = int(rng.integers(1, m // 3))
        if mode == 'random':
            want.append(oes.top_mask(draw[s], mask, q)); rows.append((mode, q, 0, 0, 0., 3))
        elif mode == 'entropy':
            want.append(oes.top_mask(scores[s], mask, q)); rows.append((mode, q, 0, 0, 0., 3))
        elif mode == 'mixed':
            chosen, info = oes.mixed_select(scores[s], mask, draw[s], q, 2.5)
            want.append(chosen); rows.append((mode, q, info['candidate_count'], 0, 0., 3))
        elif mode == 'block':   # a prefix of block steps from an all-MASK column (quotas stay valid), then one step
            tokens[s] = classes
            mask = tokens[s] == classes
            for q_prev in (3000, 9000, 20000):
                step_scores = rng.standard_normal(shape).astype(np.float32)
                done, _ = oes.block_select(step_scores, mask, q_prev, 4, orders[s], total - int(mask.sum()))
                tokens[s][done] = rng.integers(0, classes, int(done.sum()))
                mask = tokens[s] == classes
            committed = total - int(mask.sum())
            q = 7777
            chosen, _ = oes.block_select(scores[s], mask, q, 4, orders[s], committed)
            want.append(chosen); rows.append((mode, q, 0, committed, 0., 3))
        else:
            p = np.float32(0.37)
            want.append(mask & (draw[s] < p)); rows.append((mode, 0, 0, 0, float(p), 3))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    pos = np.zeros((slots, total // 64), np.int32)
    for s in range(slots):
        pos[s, orders[s]] = np.arange(total // 64)
    chosen = torch.zeros((slots, *shape), dtype=torch.uint8, device='cuda')
    index = torch.zeros((slots, total), dtype=torch.int32, device='cuda')
    count = torch.zeros(slots, dtype=torch.int32, device='cuda')
    commit = torch.zeros((slots, *shape), dtype=torch.int32, device='cuda')
    status = torch.zeros(slots, dtype=torch.int32, device='cuda')
    ops.eval_select(dev(scores), dev(draw), dev(tokens), dev(pos), ops.eval_params(rows, 'cuda'), classes, chosen=chosen,
                    index=index, count=count, commit_step=commit, status=status)
    got = chosen.cpu().numpy().astype(bool)
    for s in range(slots):
        assert np.array_equal(got[s], want[s]), rows[s][0]
        n = int(want[s].sum())
        assert int(count[s]) == n and np.array_equal(index[s, :n].cpu().numpy(), np.flatnonzero(want[s]))
        assert (index[s, n:] == -1).all() and int(status[s]) == 0
        assert np.array_equal(commit[s].cpu().numpy() == 3, want[s])


def _chunk_stats(x):
    """(mean, M2) of every 32-column chunk of the rows of x, chunk-major [K/32, M, 2], in float64."""
    c = x.double().reshape(x.shape[0], -1, 32)
    mean = c.mean(-1)
    return torch.stack((mean, ((c - mean[..., None]) ** 2).sum(-1)), -1).transpose(0, 1)


def test_patch_embed_writes_row_statistics(ops):
    torch.manual_seed(16)
    classes, d = 31, 192
    table = (torch.randn(((classes + 1) * 64, d)) * 0.05).bfloat16().cuda()
    bias = (torch.randn(d) * 0.1 + 0.3).bfloat16().cuda()
    add = (torch.randn((256, d)) * 0.1).bfloat16().cuda()
    tokens = torch.randint(0, classes + 1, (2, 64, 16, 16)).to(torch.int16).cuda()
    stats_b = torch.zeros((d // 32, 512, 2), device='cuda')
    stats_c = torch.zeros_like(stats_b)
    out_b, out_c = ops.patch_embed(tokens, classes, table, bias, add, table, bias, add, stats_b=stats_b,
                                   stats_c=stats_c)
    want = _chunk_stats(out_b.float())
    torch.testing.assert_close(stats_b.double(), want, atol=1e-5, rtol=1e-5)
    assert torch.equal(stats_b, stats_c)


def _embed_sequential(tokens, table, bias, add, classes):
    """The embed in the kernel's arithmetic: fp32 sum over the 64 offsets in order o = 0..63, then bf16(bf16(bf16(sum)
    + bias) + add[p]), ids clamped to [0, classes]."""
    s, h, dz, w = tokens.shape
    t = tokens.long().clamp(0, classes).reshape(s, h // 4, 4, dz // 4, 4, w // 4, 4)
    rows = t.permute(0, 1, 3, 5, 2, 4, 6).reshape(-1, 64) * 64 + torch.arange(64)
    tab = table.float()
    acc = torch.zeros((len(rows), table.shape[1]))
    for o in range(64):
        acc = acc + tab[rows[:, o]]
    return _bf16(_bf16(_bf16(acc) + bias.float()) + add.float().repeat(s, 1))


@pytest.mark.parametrize('shape,tokens', [((3, 4, 8, 4), 'random'), ((1, 4, 4, 12), 'random'),
                                          ((3, 8, 8, 4), 'terrain'), ((2, 64, 16, 16), 'terrain'),
                                          ((2, 64, 16, 16), 'mask'), ((5, 4, 8, 4), 'out_of_range')])
def test_patch_embed_bit_exact_sequential_sum(ops, shape, tokens):
    """The embed (fp32 sum of 64 bf16 table rows with sm_100's mixed-precision adds) is bit-exact against the
    sequential fp32 sum: odd row counts (6, 3 and 10 rows), terrain-like columns (air above a height, a few ids below,
    MASK with probability r), all-MASK columns and out-of-vocabulary ids (clamped); the chunk statistics follow the same
    rows."""
    g = torch.Generator().manual_seed(sum(shape) + len(tokens))
    classes, d = 40, 128
    s, h, dz, w = shape
    if tokens == 'random':
        t = torch.randint(0, classes + 1, shape, generator=g)
    elif tokens == 'terrain':
        height = torch.randint(h // 4, 3 * h // 4, (s, 1, dz, w), generator=g)
        y = torch.arange(h)[None, :, None, None]
        t = torch.where(y < height, torch.randint(1, 5, shape, generator=g), 0)
        r = torch.rand((s, 1, 1, 1), generator=g)
        t = torch.where(torch.rand(shape, generator=g) < r, classes, t)
    elif tokens == 'mask':
        t = torch.full(shape, classes)
    else:
        t = torch.randint(-3, classes + 4, shape, generator=g)
    table = (torch.randn(((classes + 1) * 64, d), generator=g) * 0.05).bfloat16()
    bias = (torch.randn(d, generator=g) * 0.1).bfloat16()
    patches = (h // 4) * (dz // 4) * (w // 4)
    add = (torch.randn((patches, d), generator=g) * 0.1).bfloat16()
    want = _embed_sequential(t, table, bias, add, classes)
    rows = s * patches
    stats_b = torch.zeros((d // 32, rows, 2), device='cuda')
    out_b, out_c = ops.patch_embed(t.to(torch.int16).cuda(), classes, table.cuda(), bias.cuda(), add.cuda(),
                                   table.cuda(), bias.cuda(), add.cuda(), stats_b=stats_b)
    assert torch.equal(out_b.float().cpu(), want)
    assert torch.equal(out_b, out_c)
    torch.testing.assert_close(stats_b.double().cpu(), _chunk_stats(want), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize('m', [256, 2048, 8192])
def test_gemm_group_equals_two_launches(ops, m):
    """`svx_gemm_group` (two gated-residual GEMMs with row statistics in one launch, as the engine runs a control
    layer's cross projection with its backbone block's attention projection) equals the two launches bit for bit,
    outputs and statistics; a gate of ones gives the plain residual epilogue exactly."""
    from streamvoxel_b200 import _lib
    torch.manual_seed(23)
    d = 768
    a = [(torch.randn((m, d), device='cuda') * 0.5).bfloat16() for _ in range(2)]
    w = [(torch.randn((d, d), device='cuda') * 0.03).bfloat16() for _ in range(2)]
    b = [(torch.randn(d, device='cuda') * 0.1).bfloat16() for _ in range(2)]
    res = [torch.randn((m, d), device='cuda').bfloat16() for _ in range(2)]
    gate = (torch.randn(d, device='cuda') * 0.5).bfloat16()
    ones = torch.ones(d, device='cuda', dtype=torch.bfloat16)
    stats = [torch.zeros((d // 32, m, 2), device='cuda') for _ in range(4)]
    want0 = ops.gemm(a[0], w[0], b[0], _lib.EPI_GATE_RESIDUAL, gate=gate, residual=res[0], stats_out=stats[0])
    want1 = ops.gemm(a[1], w[1], b[1], _lib.EPI_RESIDUAL, residual=res[1], stats_out=stats[1])
    got0, got1 = ops.gemm_group([dict(a=a[0], w=w[0], bias=b[0], gate=gate, residual=res[0], stats_out=stats[2]),
                                 dict(a=a[1], w=w[1], bias=b[1], gate=ones, residual=res[1], stats_out=stats[3])])
    assert torch.equal(got0, want0) and torch.equal(got1, want1)
    assert torch.equal(stats[2], stats[0]) and torch.equal(stats[3], stats[1])


@pytest.mark.parametrize('epilogue', ['bias', 'gelu', 'rope', 'class_major'])
def test_gemm_layernorm_fold_matches_layernorm_then_linear(ops, epilogue):
    """A residual GEMM writes its output rows' chunk statistics; the next linear takes the raw rows with the LayerNorm
    + AdaLN modulate folded in (W' = W (1 + scale), r (acc - mu u) + v) and matches LayerNorm -> modulate -> linear
    in fp32 within 1e-2 abs + 1e-2 rel."""
    from streamvoxel_b200 import _lib
    from streamvoxel_b200.model import fold_layernorm
    torch.manual_seed(17)
    m, k = 1024, 768
    n = {'bias': 768, 'gelu': 3072, 'rope': 2304, 'class_major': 64 * 5}[epilogue]
    res = (torch.randn((m, k), device='cuda') * 0.8 + 0.2).bfloat16()
    a = (torch.randn((m, k), device='cuda') * 0.5).bfloat16()
    wr = (torch.randn((k, k), device='cuda') * 0.03).bfloat16()
    br = (torch.randn(k, device='cuda') * 0.1).bfloat16()
    x = res.clone()
    stats = torch.full((k // 32, m, 2), float('nan'), device='cuda')
    ops.gemm(a, wr, br, _lib.EPI_RESIDUAL, out=x, residual=x, stats_out=stats)
    torch.testing.assert_close(stats.double(), _chunk_stats(x.float()), atol=1e-5, rtol=1e-5)
    w = (torch.randn((n, k), device='cuda') * 0.03).bfloat16()
    b = (torch.randn(n, device='cuda') * 0.1).bfloat16()
    ops_ = (1 + torch.randn(k, device='cuda') * 0.2).bfloat16()
    shift = (torch.randn(k, device='cuda') * 0.2).bfloat16()
    wf, u, v = fold_layernorm(w, b, ops_, shift)
    h = torch.nn.functional.layer_norm(x.float(), (k,), eps=1e-6) * ops_.float() + shift.float()
    y = h @ w.float().t() + b.float()
    kwargs = {}
    if epilogue == 'gelu':
        kind, want = _lib.EPI_BIAS_GELU, torch.nn.functional.gelu(y)
    elif epilogue == 'rope':
        theta = torch.rand((1024, 48), device='cuda') * 6.2831853
        sin, cos = theta.sin().bfloat16(), theta.cos().bfloat16()
        kind, kwargs = _lib.EPI_ROPE, dict(rope=(sin, cos), rope_cols=2 * k, rows_per_slot=1024)
        want = None   # compared against the unfolded GEMM on the same LayerNorm output below
    elif epilogue == 'class_major':
        kind, kwargs = _lib.EPI_CLASS_MAJOR, dict(rows_per_slot=1024, classes=5, geometry=(256, 16, 16))
        want = None
    else:
        kind, want = _lib.EPI_BIAS, y
    got = ops.gemm(x, wf, b, kind, ln=(stats, u, v, 1e-6), **kwargs)
    if want is None:   # the same epilogue without the fold, on the bf16 LayerNorm output
        want = ops.gemm(h.bfloat16(), w, b, kind, **kwargs)
    if epilogue == 'rope':
        # RoPE rounds a*cos, b*sin and their difference to bf16: a one-ulp difference of its inputs (the fold rounds W',
        # the unfolded path rounds h) flips a product's rounding now and then, up to one ulp of the product (0.03 at
        # magnitude 4) where the difference cancels. Allowed: 0.1% of the elements outside the bound, none past 0.0625.
        diff = (got.float() - want.float()).abs()
        outside = diff > 1e-2 + 1e-2 * want.float().abs()
        assert outside.float().mean().item() <= 1e-3 and diff.max().item() <= 0.0625
    else:
        torch.testing.assert_close(got.float(), want.float(), atol=1e-2, rtol=1e-2)
