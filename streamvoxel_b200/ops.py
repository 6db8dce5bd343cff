"""Torch-tensor wrappers over the libsvx entry points (device tensors in, device tensors out, current stream).

Each wrapper validates dtypes/shapes on the host and calls exactly one C-ABI function; there is no CPU path.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from streamvoxel_b200 import _lib
from streamvoxel_b200._lib import check, ptr, stream_ptr

STEP_DTYPE = np.dtype([('k', '<i4'), ('step', '<i4'), ('committed', '<i8'), ('frac', '<f8'), ('seed', '<u8')])
assert STEP_DTYPE.itemsize == ctypes.sizeof(_lib.StepParams)


def _dtype_code(t):
    if t.dtype == torch.bfloat16:
        return _lib.BF16
    if t.dtype == torch.float32:
        return _lib.F32
    raise ValueError(f'logits must be bf16 or fp32, got {t.dtype}')


def step_params(rows, device=None, out=None):
    """Pack per-slot step scalars [(k, step, committed, frac, seed)] into an `svx_step_params` array.

    Returns a uint8 tensor on `device` (or copies into `out`, a pinned/device uint8 tensor of the right size)."""
    arr = np.zeros(len(rows), STEP_DTYPE)
    for i, (k, step, committed, frac, seed) in enumerate(rows):
        arr[i] = (int(k), int(step), int(committed), float(frac), int(seed) & 0xFFFFFFFFFFFFFFFF)
    host = torch.from_numpy(arr.view(np.uint8).copy())
    if out is not None:
        out.copy_(host, non_blocking=False)
        return out
    return host.to(device)


def _slots_view(logits):
    """[S, C, ...] contiguous -> (S, C, voxels, slot stride)."""
    if not logits.is_contiguous():
        raise ValueError('logits must be contiguous [slots, classes, Y, Z, X]')
    s, c = logits.shape[0], logits.shape[1]
    voxels = logits[0, 0].numel()
    return s, c, voxels, c * voxels


def ease_scores(logits, status=None, out=None):
    """Negative entropy per voxel of class-major logits [S, C, Y, Z, X] -> fp32 [S, Y, Z, X]."""
    s, c, voxels, stride = _slots_view(logits)
    scores = out if out is not None else torch.empty((s, *logits.shape[2:]), device=logits.device, dtype=torch.float32)
    check(_lib.load().svx_ease_scores(ptr(logits), _dtype_code(logits), s, c, voxels, stride, ptr(scores), ptr(status),
                                      stream_ptr()), 'svx_ease_scores')
    return scores


def ease_mark(logits, air_ids, last_eps, last=None, last_count=None):
    """Marking forward: per-column top run of voxels with P(air) > 1 - eps. Returns (last uint8, last_count int32).
    air_ids: a sequence of ids, or an int32 device tensor of them (no host-to-device copy per call)."""
    s, c, voxels, stride = _slots_view(logits)
    height, depth, width = logits.shape[2:]
    dev = logits.device
    if last is None:
        last = torch.empty((s, height, depth, width), device=dev, dtype=torch.uint8)
    if last_count is None:
        last_count = torch.empty(s, device=dev, dtype=torch.int32)
    if isinstance(air_ids, torch.Tensor) and air_ids.is_cuda:
        air = air_ids
        assert air.dtype == torch.int32 and air.is_contiguous()
    else:
        air = torch.as_tensor(list(air_ids), dtype=torch.int32, device=dev)
    check(_lib.load().svx_ease_mark(ptr(logits), _dtype_code(logits), s, c, height, depth, width, stride, ptr(air),
                                    len(air), float(last_eps), ptr(last), ptr(last_count), stream_ptr()),
          'svx_ease_mark')
    return last, last_count


def select_workspace(slots, voxels, device):
    n = _lib.load().svx_ease_select_workspace_bytes(slots, voxels)
    return torch.empty(n, dtype=torch.uint8, device=device)


def ease_select(scores, tokens, last, pos, params, mask_id, index_capacity, *, chosen=None, index=None, count=None,
                status=None, workspace=None, block=4):
    """Block-quota selection. Returns (chosen uint8 [S,Y,Z,X], index int32 [S, capacity], count int32 [S])."""
    s, height, depth, width = tokens.shape
    dev = tokens.device
    assert tokens.dtype == torch.int16 and last.dtype == torch.uint8 and scores.dtype == torch.float32
    assert pos.dtype == torch.int32 and params.dtype == torch.uint8
    if chosen is None:
        chosen = torch.empty((s, height, depth, width), device=dev, dtype=torch.uint8)
    if index is None:
        index = torch.empty((s, index_capacity), device=dev, dtype=torch.int32)
    if count is None:
        count = torch.empty(s, device=dev, dtype=torch.int32)
    if workspace is None:
        workspace = select_workspace(s, height * depth * width, dev)
    check(_lib.load().svx_ease_select(ptr(scores), ptr(tokens), ptr(last), ptr(pos), ptr(params), s, height, depth,
                                      width, block, mask_id, ptr(chosen), ptr(index), index_capacity, ptr(count),
                                      ptr(status), ptr(workspace), stream_ptr()), 'svx_ease_select')
    return chosen, index, count


EVAL_MODES = dict(random=0, entropy=1, mixed=2, block=3, threshold=4)


def eval_params(rows, device):
    """Pack per-slot evaluation-step scalars [(mode, k, candidates, committed, threshold, step)] (`svx_eval_params`)
    into a device uint8 tensor."""
    arr = (_lib.EvalParams * len(rows))(*[_lib.EvalParams(EVAL_MODES[m] if isinstance(m, str) else int(m), int(k),
                                                          int(c), int(done), float(th), int(st))
                                          for m, k, c, done, th, st in rows])
    host = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
    return host.to(device)


def eval_select(scores, draw, tokens, pos, params, mask_id, *, chosen, index, count, commit_step=None,
                quota_range=None, status=None):
    """Selections of the evaluation decoders (random / entropy / mixed / block / threshold) over the masked voxels
    of each slot: fills chosen [S, Y, Z, X] uint8, index [S, capacity] (ascending, -1 padded), count [S] and, when
    given, commit_step [S, Y, Z, X] int32 and quota_range [S, 2] int32."""
    s, height, depth, width = tokens.shape
    check(_lib.load().svx_eval_select(ptr(scores), ptr(draw), ptr(tokens), ptr(pos), ptr(params), s, height, depth,
                                      width, mask_id, ptr(chosen), ptr(index), index.shape[1], ptr(count),
                                      ptr(commit_step), ptr(quota_range), ptr(status), stream_ptr()),
          'svx_eval_select')
    return chosen, index, count


def ease_sample(logits, index, params, tokens, noise=None, values=None, status=None):
    """Categorical draw for the chosen voxels; writes tokens in place. noise [S, capacity, C] fp32 or None (native)."""
    s, c, voxels, stride = _slots_view(logits)
    capacity = index.shape[1]
    if values is None:
        values = torch.empty((s, capacity), device=logits.device, dtype=torch.int16)
    noise_stride = 0
    if noise is not None:
        assert noise.dtype == torch.float32 and noise.is_contiguous() and noise.shape[-1] == c
        noise_stride = noise[0].numel() if noise.dim() == 3 else 0
    check(_lib.load().svx_ease_sample(ptr(logits), _dtype_code(logits), s, c, voxels, stride, ptr(index), ptr(params),
                                      ptr(noise), noise_stride, capacity, ptr(tokens), ptr(values), ptr(status),
                                      stream_ptr()), 'svx_ease_sample')
    return values


def softmax_rows(x):
    out = torch.empty_like(x)
    check(_lib.load().svx_softmax_rows(ptr(x), x.shape[0], x.shape[1], ptr(out), stream_ptr()), 'svx_softmax_rows')
    return out


def ease_finish(tokens, last, finish, air_token):
    s = tokens.shape[0]
    check(_lib.load().svx_ease_finish(ptr(tokens), ptr(last), ptr(finish), s, tokens[0].numel(), int(air_token),
                                      stream_ptr()), 'svx_ease_finish')


def patch_embed(tokens, classes, table_b, bias_b, add_b, table_c=None, bias_c=None, add_c=None, out_b=None,
                out_c=None, stats_b=None, stats_c=None):
    """Patch-4 token embed of both branches; stats_b / stats_c (optional fp32 [d/32, rows, 2]) receive each output
    row's 32-column chunk statistics (mean, M2), chunk-major, for the LayerNorm fold of the next linear."""
    s, height, depth, width = tokens.shape
    d = table_b.shape[1]
    patches = (height // 4) * (depth // 4) * (width // 4)
    if out_b is None:
        out_b = torch.empty((s * patches, d), device=tokens.device, dtype=torch.bfloat16)
    if table_c is not None and out_c is None:
        out_c = torch.empty((s * patches, d), device=tokens.device, dtype=torch.bfloat16)
    check(_lib.load().svx_patch_embed(ptr(tokens), s, height, depth, width, 4, classes, d, ptr(table_b), ptr(bias_b),
                                      ptr(add_b), ptr(out_b), ptr(table_c), ptr(bias_c), ptr(add_c), ptr(out_c),
                                      ptr(stats_b), ptr(stats_c), stream_ptr()), 'svx_patch_embed')
    return out_b, out_c


def layernorm_modulate(x, eps=1e-6, one_plus_scale=None, shift=None, out=None):
    rows, d = x.shape
    if out is None:
        out = torch.empty_like(x)
    check(_lib.load().svx_layernorm_modulate(ptr(x), rows, d, float(eps), ptr(one_plus_scale), ptr(shift), ptr(out),
                                             stream_ptr()), 'svx_layernorm_modulate')
    return out


def layernorm_affine(x, eps, pre=None, weight=None, bias=None, gelu=False, out=None):
    """bf16(g(LN(x + pre) * weight + bias)) in fp32 (the condition encoder's LayerNorms; g = GELU(erf) with gelu).
    x [rows, d] bf16; pre, weight, bias [d] fp32 or None."""
    rows, d = x.shape
    if out is None:
        out = torch.empty_like(x)
    check(_lib.load().svx_layernorm_affine(ptr(x), rows, d, float(eps), ptr(pre), ptr(weight), ptr(bias), int(gelu),
                                           ptr(out), stream_ptr()), 'svx_layernorm_affine')
    return out


def gemm(a, w, bias, epilogue=_lib.EPI_BIAS, out=None, gate=None, residual=None, rope=None, rope_cols=0,
         rows_per_slot=0, head_dim=96, classes=0, geometry=(0, 0, 0), ln=None, stats_out=None):
    """out = epilogue(a @ w.T + bias) on the tcgen05 GEMM. a [M,K], w [N,K], bias [N] bf16.
    ln = (stats [K/32, M, 2] fp32, u [N], v [N] fp32, eps): the LayerNorm folded in, out = epilogue(r (acc - mu u) + v)
    with w the modulated weights; stats_out: fp32 [N/32, M, 2] chunk statistics of the bf16 output rows."""
    m, k = a.shape
    n = w.shape[0]
    for t in (a, w, bias):
        assert t.dtype == torch.bfloat16 and t.is_contiguous()
    if out is None:
        if epilogue == _lib.EPI_CLASS_MAJOR:
            out = torch.empty((m // rows_per_slot, classes, *geometry), device=a.device, dtype=torch.bfloat16)
        else:
            out = torch.empty((m, n), device=a.device, dtype=torch.bfloat16)
    args = _lib.EpilogueArgs(epilogue=epilogue, bias=bias.data_ptr(), gate=ptr(gate).value, residual=ptr(residual).value,
                             rope_sin=ptr(rope[0] if rope else None).value, rope_cos=ptr(rope[1] if rope else None).value,
                             rope_cols=rope_cols, rows_per_slot=rows_per_slot, head_dim=head_dim, classes=classes,
                             height=geometry[0], depth=geometry[1], width=geometry[2], patch=4)
    if ln is not None:
        stats, u, v, eps = ln
        assert stats.dtype == u.dtype == v.dtype == torch.float32
        args.ln_stats_in, args.ln_u, args.ln_v, args.ln_eps = ptr(stats).value, ptr(u).value, ptr(v).value, eps
    if stats_out is not None:
        assert stats_out.dtype == torch.float32
        args.ln_stats_out = ptr(stats_out).value
    check(_lib.load().svx_gemm(ptr(a), ptr(w), ptr(out), m, n, k, ctypes.byref(args), stream_ptr()), 'svx_gemm')
    return out


def gemm_group(problems):
    """Two gated-residual GEMMs with row statistics in one launch (`svx_gemm_group`): problems = two dicts with a, w,
    bias, gate, residual, stats_out (and optional out); out_i = bf16(res_i + bf16(gate_i bf16(a_i w_i^T + bias_i))).
    Returns the two outputs."""
    outs, args = [], []
    for p in problems:
        m, k = p['a'].shape
        n = p['w'].shape[0]
        for t in (p['a'], p['w'], p['bias'], p['gate'], p['residual']):
            assert t.dtype == torch.bfloat16 and t.is_contiguous()
        assert p['stats_out'].dtype == torch.float32
        out = p.get('out')
        if out is None:
            out = torch.empty((m, n), device=p['a'].device, dtype=torch.bfloat16)
        outs.append(out)
        args.append(_lib.EpilogueArgs(epilogue=_lib.EPI_GATE_RESIDUAL, bias=p['bias'].data_ptr(),
                                      gate=p['gate'].data_ptr(), residual=p['residual'].data_ptr(),
                                      ln_stats_out=p['stats_out'].data_ptr(), patch=4))
    (m, k), n = problems[0]['a'].shape, problems[0]['w'].shape[0]
    assert problems[1]['a'].shape == (m, k) and problems[1]['w'].shape == (n, k)
    check(_lib.load().svx_gemm_group(ptr(problems[0]['a']), ptr(problems[0]['w']), ptr(outs[0]), ctypes.byref(args[0]),
                                     ptr(problems[1]['a']), ptr(problems[1]['w']), ptr(outs[1]), ctypes.byref(args[1]),
                                     m, n, k, stream_ptr()), 'svx_gemm_group')
    return outs


def attention_plan(lengths, slots, heads, queries, keys, ctas, device=None):
    """Work-unit plan of `svx_attention_plan` for host key lengths (sequence or None) on `ctas` CTAs. Returns the
    int32 plan (on `device`, or a host tensor) and the CTA count the launch must use."""
    lib = _lib.load()
    size = lib.svx_attention_plan_ints(slots, heads, queries, ctas)
    if size <= 0:
        raise ValueError('attention_plan: bad shape')
    plan = torch.empty(size, dtype=torch.int32)
    host = None if lengths is None else torch.as_tensor(list(lengths), dtype=torch.int32)
    check(lib.svx_attention_plan(ptr(host), slots, heads, queries, keys, ctas, ptr(plan), size),
          'svx_attention_plan')
    units = slots * heads * ((queries // 128 + 1) // 2)
    return (plan if device is None else plan.to(device)), min(ctas, units)


def attention_multi_plan(problems, slots, heads, queries, ctas, device=None):
    """Joint work plan of `svx_attention_multi_plan` for one or two problems, each given as (host key lengths or
    None, keys). Returns the int32 plan (on `device`, or a host tensor) and the CTA count the launch must use."""
    lib = _lib.load()
    count = len(problems)
    size = lib.svx_attention_multi_plan_ints(count, slots, heads, queries, ctas)
    if size <= 0:
        raise ValueError('attention_multi_plan: bad shape')
    hosts = [None if lengths is None else torch.as_tensor(list(lengths), dtype=torch.int32)
             for lengths, _ in problems]
    lens = (ctypes.c_void_p * count)(*[None if h is None else h.data_ptr() for h in hosts])
    keys = (ctypes.c_int * count)(*[int(k) for _, k in problems])
    plan = torch.empty(size, dtype=torch.int32)
    check(lib.svx_attention_multi_plan(lens, keys, count, slots, heads, queries, ctas, ptr(plan), size),
          'svx_attention_multi_plan')
    units = count * slots * heads * ((queries // 128 + 1) // 2)
    return (plan if device is None else plan.to(device)), min(ctas, units)


def attention_multi(problems, slots, heads, queries, plan):
    """One launch over one or two attention problems (dicts of `attention`'s arguments: q, k, v, keys, the four
    strides, lengths, out), with a plan from `attention_multi_plan`. Returns the outputs."""
    raw = _lib.raw_ptr
    table, ctas = plan
    structs = []
    for pr in problems:
        structs.append(_lib.AttentionProblem(raw(pr['q']), raw(pr['k']), raw(pr['v']), pr['q_row_stride'],
                                             pr['kv_slot_stride'], pr['kv_head_stride'], pr['kv_row_stride'],
                                             ptr(pr.get('lengths')), pr['keys'], ptr(pr['out'])))
    arr = (_lib.AttentionProblem * len(structs))(*structs)
    check(_lib.load().svx_attention_multi(arr, len(structs), slots, heads, queries, ptr(table), ctas, stream_ptr()),
          'svx_attention_multi')
    return [pr['out'] for pr in problems]


def attention(q, k, v, slots, heads, queries, keys, *, q_row_stride, kv_slot_stride, kv_head_stride, kv_row_stride,
              lengths=None, out=None, plan=None):
    """Non-causal head_dim-96 attention over per-slot key lengths; out [slots*queries, heads*96] bf16.
    `plan`: an `attention_plan` result (device plan, CTA count) or None."""
    if out is None:
        out = torch.empty((slots * queries, heads * 96), device=q.device, dtype=torch.bfloat16)
    raw = _lib.raw_ptr
    table, ctas = plan if plan is not None else (None, 0)
    check(_lib.load().svx_attention(raw(q), q_row_stride, raw(k), raw(v), kv_slot_stride, kv_head_stride,
                                    kv_row_stride, ptr(lengths), slots, heads, queries, keys, ptr(out), ptr(table),
                                    ctas, stream_ptr()),
          'svx_attention')
    return out
