"""Run one hot kernel at the config-2 step shapes, for a focused profiler capture.

    python -m streamvoxel_b200.profile_case <case> [--launches N]

Cases: attention_cross, attention_joint (cross + self in one launch), attention_self, gemm_fc1, gemm_fc1_fold (the
LayerNorm folded in, as the engine runs fc1), gemm_qkv, gemm_dxd, gemm_head, ease_scores, ease_mark, ease_select,
ease_sample, patch_embed (both branches; tokens uniform over the 257 ids, the gather's worst case). Inputs are seeded
random tensors with the bench's shapes (8 slots, d=768, 8 heads x 96, V=256, 65536 voxels, packed keys of k = 0..7
L1 tiles); every case's working set is larger than the 126 MB L2 except the GEMMs' and the selection. Prints the mean launch time measured with CUDA events.
"""
from __future__ import annotations

import argparse

import numpy as np
import torch

from streamvoxel_b200 import _lib, ops

SLOTS, PATCHES, D, HEADS, V, MLP, VOXELS = 8, 1024, 768, 8, 256, 3072, 65536
CAPACITY = 9600


def cases():
    g = torch.Generator(device='cuda').manual_seed(0)
    bf = dict(device='cuda', dtype=torch.bfloat16)
    rows = SLOTS * PATCHES
    rnd = lambda *shape, s=1.0: (torch.randn(shape, device='cuda', generator=g) * s).to(torch.bfloat16)
    h = rnd(rows, D)
    qkv = rnd(rows, 3 * D)
    out = torch.empty((rows, D), **bf)
    mlp = torch.empty((rows, MLP), **bf)
    k = rnd(SLOTS, HEADS, CAPACITY, 96)
    v = rnd(SLOTS, HEADS, CAPACITY, 96)
    lengths = torch.tensor([1344 + 1024 * i for i in range(SLOTS)], dtype=torch.int32, device='cuda')
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    plan = ops.attention_plan(lengths.tolist(), SLOTS, HEADS, PATCHES, CAPACITY, sms, 'cuda')
    joint_plan = ops.attention_multi_plan([(lengths.tolist(), CAPACITY), (None, PATCHES)], SLOTS, HEADS, PATCHES, sms,
                                          'cuda')
    qx = rnd(rows, D)
    cross = dict(q=qx, k=k, v=v, keys=CAPACITY, q_row_stride=D, kv_slot_stride=HEADS * CAPACITY * 96,
                 kv_head_stride=CAPACITY * 96, kv_row_stride=96, lengths=lengths, out=torch.empty((rows, D), **bf))
    w = {n: rnd(*shape, s=0.02) for n, shape in
         (('qkv', (3 * D, D)), ('fc1', (MLP, D)), ('dxd', (D, D)), ('head', (64 * V, D)))}
    b = {n: rnd(t.shape[0], s=0.02) for n, t in w.items()}
    gate = rnd(D, s=0.1)
    from streamvoxel_b200.model import fold_layernorm
    fc1_fold = fold_layernorm(w['fc1'], b['fc1'], (1 + rnd(D, s=0.1).float()).bfloat16(), rnd(D, s=0.1))
    hc = h.double().reshape(rows, D // 32, 32)
    h_stats = torch.stack((hc.mean(-1), ((hc - hc.mean(-1, keepdim=True)) ** 2).sum(-1)), -1).transpose(0, 1)
    h_stats = h_stats.float().contiguous()
    logits = rnd(SLOTS, V, 256, 16, 16, s=2.0)
    sin = rnd(PATCHES, 48)
    cos = rnd(PATCHES, 48)
    scores = torch.empty((SLOTS, 256, 16, 16), device='cuda', dtype=torch.float32)
    tokens = torch.full((SLOTS, 256, 16, 16), V, dtype=torch.int16, device='cuda')
    last = torch.zeros((SLOTS, 256, 16, 16), dtype=torch.uint8, device='cuda')
    rng = np.random.default_rng(0)
    pos = torch.from_numpy(np.stack([rng.permutation(1024) for _ in range(SLOTS)]).astype(np.int32)).cuda()
    table = rnd((V + 1) * 64, D, s=0.02)
    table_bias = rnd(D, s=0.02)
    y_add = rnd(PATCHES, D, s=0.02)
    embed_tokens = torch.randint(0, V + 1, (SLOTS, 256, 16, 16), device='cuda', dtype=torch.int16, generator=g)
    embed_out = (torch.empty((rows, D), **bf), torch.empty((rows, D), **bf))
    last_count = torch.empty(SLOTS, dtype=torch.int32, device='cuda')
    params = ops.step_params([(2048, 5, 2048 * 4, 2048 * 5 / VOXELS, i) for i in range(SLOTS)], 'cuda')
    ops.ease_scores(logits, out=scores)
    chosen, index, count = ops.ease_select(scores, tokens, last, pos, params, V, VOXELS)
    return {
        'attention_cross': (lambda: ops.attention(qkv, k, v, SLOTS, HEADS, PATCHES, CAPACITY, q_row_stride=3 * D,
                                                  kv_slot_stride=HEADS * CAPACITY * 96, kv_head_stride=CAPACITY * 96,
                                                  kv_row_stride=96, lengths=lengths, out=out, plan=plan),
                            4.0 * HEADS * PATCHES * 96 * float(lengths.sum())),
        'attention_joint': (lambda: ops.attention_multi(
            [cross, dict(q=qkv, k=qkv[:, D:], v=qkv[:, 2 * D:], keys=PATCHES, q_row_stride=3 * D,
                         kv_slot_stride=PATCHES * 3 * D, kv_head_stride=96, kv_row_stride=3 * D, out=out)],
            SLOTS, HEADS, PATCHES, joint_plan),
            4.0 * HEADS * PATCHES * 96 * float(lengths.sum()) + 4.0 * SLOTS * HEADS * PATCHES * PATCHES * 96),
        'attention_self': (lambda: ops.attention(qkv, qkv[:, D:], qkv[:, 2 * D:], SLOTS, HEADS, PATCHES, PATCHES,
                                                 q_row_stride=3 * D, kv_slot_stride=PATCHES * 3 * D, kv_head_stride=96,
                                                 kv_row_stride=3 * D, out=out),
                           4.0 * SLOTS * HEADS * PATCHES * PATCHES * 96),
        'gemm_fc1': (lambda: ops.gemm(h, w['fc1'], b['fc1'], _lib.EPI_BIAS_GELU, out=mlp), 2.0 * rows * D * MLP),
        # fc1 as the engine runs it: the LayerNorm + modulate folded in (raw rows h, their chunk statistics)
        'gemm_fc1_fold': (lambda: ops.gemm(h, fc1_fold[0], b['fc1'], _lib.EPI_BIAS_GELU, out=mlp,
                                           ln=(h_stats, *fc1_fold[1:], 1e-6)), 2.0 * rows * D * MLP),
        'gemm_qkv': (lambda: ops.gemm(h, w['qkv'], b['qkv'], _lib.EPI_ROPE, out=qkv, rope=(sin, cos),
                                      rope_cols=2 * D, rows_per_slot=PATCHES), 2.0 * rows * D * 3 * D),
        'gemm_dxd': (lambda: ops.gemm(h, w['dxd'], b['dxd'], _lib.EPI_GATE_RESIDUAL, out=out, gate=gate,
                                      residual=out), 2.0 * rows * D * D),
        'gemm_head': (lambda: ops.gemm(h, w['head'], b['head'], _lib.EPI_CLASS_MAJOR, out=logits,
                                       rows_per_slot=PATCHES, classes=V, geometry=(256, 16, 16)),
                      2.0 * rows * D * 64 * V),
        'ease_scores': (lambda: ops.ease_scores(logits, out=scores), float(logits.numel() * 2 + scores.numel() * 4)),
        'ease_mark': (lambda: ops.ease_mark(logits, (0,), 1e-3, last=last, last_count=last_count),
                      float(logits.numel() * 2 + 2 * last.numel())),
        'patch_embed': (lambda: ops.patch_embed(embed_tokens, V, table, table_bias, y_add, table, table_bias, y_add,
                                                out_b=embed_out[0], out_c=embed_out[1]),
                        float(embed_tokens.numel() * 2 + 2 * rows * D * 2)),
        'ease_select': (lambda: ops.ease_select(scores, tokens, last, pos, params, V, VOXELS, chosen=chosen,
                                                index=index, count=count), float(SLOTS * VOXELS * 8)),
        'ease_sample': (lambda: ops.ease_sample(logits, index, params, tokens.clone()),
                        float(SLOTS * 2048 * V * 2)),
    }


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument('case')
    parser.add_argument('--launches', type=int, default=3)
    args = parser.parse_args()
    _lib.require_device()
    table = cases()
    fn, work = table[args.case]
    fn()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.launches):
        fn()
    stop.record()
    stop.synchronize()
    seconds = start.elapsed_time(stop) * 1e-3 / args.launches
    unit = 'GB/s' if args.case.startswith(('ease', 'patch')) else 'TFLOP/s'
    rate = work / seconds / (1e9 if unit == 'GB/s' else 1e12)
    print(f'{args.case}: {seconds * 1e6:.1f} us per launch, {rate:.1f} {unit} (work {work:.4g})')


if __name__ == '__main__':
    main()
