"""Time-free DiT + compact ControlNet forward restated functionally (TEST INFRASTRUCTURE ONLY).

Runs on the CPU from a reference-named state dict (`backbone.blocks.0.attn.qkv.weight`, ...). Two precisions:

* `bf16=False`: plain fp32, the reference's own CPU numerics (`streamvoxel/train/runtime.py:15-16` turns
  autocast off on the CPU). Pinned against the reference at 1e-5 by the golden fixtures.
* `bf16=True`: fp32 arithmetic with the rounding points of CUDA bf16 autocast, the reference's GPU forward: every
  linear / conv rounds its inputs, weights and output to bf16; LayerNorm runs in fp32; element-wise ops on bf16
  operands round their result to bf16; RoPE sin/cos are rounded to bf16 after fp32 phases.

Citations are `path:line` in zzf1955/StreamVoxel.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


class Precision:
    def __init__(self, bf16):
        self.bf16 = bool(bf16)

    def r(self, x):
        """Round to bf16 (a bf16-valued op output) or pass through in fp32."""
        return x.bfloat16().float() if self.bf16 else x

    def linear(self, x, w, b=None):
        """`nn.Linear` under autocast: bf16 operands, fp32 accumulation, bf16 output."""
        r = self.r
        return r(F.linear(r(x), r(w), None if b is None else r(b)))

    def layer_norm(self, x, eps, weight=None, bias=None):
        """LayerNorm runs in fp32 under autocast (fp32 output)."""
        return F.layer_norm(x, x.shape[-1:], weight, bias, eps)

    def modulate(self, x, shift, scale):
        """`streamvoxel/models/unconditional_md4_timefree.py:12-13`: (1+scale) is a bf16 op; the fp32 x promotes."""
        return x * self.r(1 + scale)[:, None] + shift[:, None]

    def gelu(self, x):
        return self.r(F.gelu(x))

    def silu(self, x):
        return self.r(F.silu(x))

    def add(self, a, b):
        return self.r(a + b)

    def mul(self, a, b):
        return self.r(a * b)

    def sdpa(self, q, k, v):
        """`F.scaled_dot_product_attention` (non-causal, scale 1/sqrt(D)). Under CUDA autocast SDPA runs a flash-style
        bf16 kernel: fp32 scores and row sums, the unnormalised probabilities rounded to bf16 for the P.V product,
        the output normalised in fp32 and rounded to bf16. The bf16 emulation follows those rounding points."""
        if not self.bf16:
            return F.scaled_dot_product_attention(q, k, v)
        s = (q @ k.transpose(-1, -2)) * (1.0 / q.shape[-1] ** 0.5)
        p = torch.exp(s - s.amax(-1, keepdim=True))
        return self.r((self.r(p) @ v) / p.sum(-1, keepdim=True))


# ------------------------------------------------------------------------------------------------- RoPE

def rope_frequencies(head_dim, base=10000.):
    """`streamvoxel/models/unconditional_md4_timefree.py:16-22`."""
    axis = head_dim // 3
    return base ** (-torch.arange(0, axis, 2).float() / axis)


def rope(x, positions, frequencies, p):
    """`AxialRoPE.forward` `unconditional_md4_timefree.py:24-30`. x [B,H,N,D]; positions [B,N,3] (x, y, z)."""
    phase = positions.float()[..., None] * frequencies
    sin, cos = p.r(phase.sin()[:, None]), p.r(phase.cos()[:, None])
    axis = x.shape[-1] // 3
    pairs = x.reshape(*x.shape[:-1], 3, axis // 2, 2)
    a, b = pairs.unbind(-1)
    first = p.r(p.r(a * cos) - p.r(b * sin))
    second = p.r(p.r(a * sin) + p.r(b * cos))
    return torch.stack((first, second), -1).flatten(-3)


# ------------------------------------------------------------------------------------------------- blocks

def patch_centers_xyz(voxel_shape, patch):
    """`unconditional_md4_timefree.py:84-86`: patch centres in (x, y, z) voxels, patch grid in YZX order."""
    grid = torch.stack(torch.meshgrid(*(torch.arange(v // patch).float() for v in voxel_shape), indexing='ij'), -1)
    return grid.reshape(-1, 3)[:, [2, 0, 1]] * patch + patch / 2


def ada_vectors(sd, prefix, count, p, time_key='backbone.constant_time'):
    """`ada(constant_time)` of a time-free block (`unconditional_md4_timefree.py:58,120-121`): SiLU then linear.

    The backbone and the control copy each carry their own `constant_time` (`compact_controlnet.py:122-123`)."""
    time = sd[time_key][None].float()
    out = p.linear(F.silu(time), sd[prefix + '.1.weight'], sd[prefix + '.1.bias'])
    return out.chunk(count, -1)


def block(sd, prefix, time_key, x, positions, heads, p):
    """`UnconditionalBlock.forward` `unconditional_md4_timefree.py:60-63` + `RotaryAttention` `:41-47`."""
    s1, c1, g1, s2, c2, g2 = ada_vectors(sd, prefix + '.ada', 6, p, time_key)
    bsz, n, d = x.shape
    h = p.modulate(p.layer_norm(x, 1e-6), s1, c1)
    qkv = p.linear(h, sd[prefix + '.attn.qkv.weight'], sd[prefix + '.attn.qkv.bias'])
    q, k, v = qkv.reshape(bsz, n, 3, heads, d // heads).unbind(2)
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    freq = rope_frequencies(d // heads)
    q, k = rope(q, positions, freq, p), rope(k, positions, freq, p)
    attn = p.sdpa(q, k, v).transpose(1, 2).reshape(bsz, n, d)
    attn = p.linear(attn, sd[prefix + '.attn.proj.weight'], sd[prefix + '.attn.proj.bias'])
    x = p.add(x, p.mul(g1[:, None], attn))
    h = p.modulate(p.layer_norm(x, 1e-6), s2, c2)
    m = p.gelu(p.linear(h, sd[prefix + '.mlp.0.weight'], sd[prefix + '.mlp.0.bias']))
    m = p.linear(m, sd[prefix + '.mlp.2.weight'], sd[prefix + '.mlp.2.bias'])
    return p.add(x, p.mul(g2[:, None], m))


def patchify(sd, prefix, tokens, classes, p):
    """One-hot Conv3d patchify (`unconditional_md4_timefree.py:144-150`): bf16 conv, then the bias in bf16.

    Computed as the gather `bias + sum_o W[:, t_o, o]` (`streamvoxel/stream/fast_ops.py:58-75`)."""
    w = sd[prefix + '.weight']  # [d, C+1, P, P, P]
    d, _, patch = w.shape[0], w.shape[1], w.shape[2]
    bsz, height, depth, width = tokens.shape
    cells = tokens.long().reshape(bsz, height // patch, patch, depth // patch, patch, width // patch, patch)
    cells = cells.permute(0, 1, 3, 5, 2, 4, 6).reshape(-1, patch ** 3)
    table = p.r(w.permute(1, 2, 3, 4, 0).reshape(-1, d).float())
    index = cells * patch ** 3 + torch.arange(patch ** 3)
    out = p.r(table[index].sum(1))
    out = p.r(out + p.r(sd[prefix + '.bias'].float()))
    return out.reshape(bsz, -1, d)


def y_embed(sd, prefix, y, p):
    """`y_embed` MLP `unconditional_md4_timefree.py:88`: Linear(1,d) -> SiLU -> Linear(d,d)."""
    h = p.silu(p.linear(y, sd[prefix + '.0.weight'], sd[prefix + '.0.bias']))
    return p.linear(h, sd[prefix + '.2.weight'], sd[prefix + '.2.bias'])


def head(sd, x, voxel_shape, classes, patch, p):
    """Final AdaLN + class head + voxel layout (`compact_controlnet.py:151-159`)."""
    shift, gain = ada_vectors(sd, 'backbone.final_ada', 2, p)
    patches = p.linear(p.modulate(p.layer_norm(x, 1e-6), shift, gain), sd['backbone.class_head.weight'],
                       sd['backbone.class_head.bias'])
    gy, gz, gx = (v // patch for v in voxel_shape)
    n = x.shape[0]
    return patches.reshape(n, gy, gz, gx, patch, patch, patch, classes).permute(0, 7, 1, 4, 2, 5, 3, 6).reshape(
        n, classes, *voxel_shape)


def _geometry(voxel_shape, patch, origin_xyz, y_range):
    centers_local = patch_centers_xyz(voxel_shape, patch)
    centers = centers_local[None] + origin_xyz[:, None]
    sa_positions = centers_local[None].expand(len(origin_xyz), -1, -1) / patch
    y = 2 * (centers[..., 1:2] - y_range[0]) / (y_range[1] - y_range[0]) - 1
    return centers, sa_positions, y


def unconditional_forward(sd, tokens, cfg, bf16=False):
    """`UnconditionalMD4DiT.forward` (time-free) `unconditional_md4_timefree.py:152-177`. Logits [B,C,Y,Z,X]."""
    p = Precision(bf16)
    shape, patch, classes = cfg['voxel_shape'], cfg['patch_size'], cfg['num_classes']
    origin = torch.tensor([0., float(cfg['y_range'][0]), 0.])[None].expand(len(tokens), -1)
    _, positions, y = _geometry(shape, patch, origin, cfg['y_range'])
    x = p.add(patchify(sd, 'backbone.target_patch', tokens, classes, p), y_embed(sd, 'backbone.y_embed', y, p))
    for i in range(cfg['depth']):
        x = block(sd, f'backbone.blocks.{i}', 'backbone.constant_time', x, positions, cfg['num_heads'], p)
    return head(sd, x, shape, classes, patch, p)


def cross_attention(sd, prefix, value, positions, kv, heads, p):
    """`RotaryCrossAttention.forward` `streaming_controlnet.py:37-61` over already encoded per-sample K/V.

    kv = (k, v) [B,H,L,D] with RoPE applied to k (prefix keys then local keys)."""
    bsz, n, d = value.shape
    q = p.linear(p.layer_norm(value, 1e-6), sd[prefix + '.query.weight'], sd[prefix + '.query.bias'])
    q = rope(q.reshape(bsz, n, heads, d // heads).transpose(1, 2), positions, rope_frequencies(d // heads), p)
    out = p.sdpa(q, kv[0], kv[1]).transpose(1, 2).reshape(bsz, n, d)
    return p.linear(out, sd[prefix + '.proj.weight'], sd[prefix + '.proj.bias'])


def control_forward(sd, tokens, kv_layers, cfg, bf16=False):
    """`CompactStreamingControlNet.forward` `compact_controlnet.py:100-159` (time-free backbone, scale 1).

    kv_layers[j] = (k, v) [B,H,L,D]: the encoded prefix + local keys of each control layer j."""
    p = Precision(bf16)
    shape, patch, classes, heads = cfg['voxel_shape'], cfg['patch_size'], cfg['num_classes'], cfg['num_heads']
    origin = torch.tensor([0., float(cfg['y_range'][0]), 0.])[None].expand(len(tokens), -1)
    centers, sa_positions, y = _geometry(shape, patch, origin, cfg['y_range'])
    positions = (centers - origin[0][None, None]) / 4
    b = p.add(patchify(sd, 'backbone.target_patch', tokens, classes, p), y_embed(sd, 'backbone.y_embed', y, p))
    c = p.add(patchify(sd, 'control.target_patch', tokens, classes, p), y_embed(sd, 'control.y_embed', y, p))
    layer_map = {i: j for j, i in enumerate(cfg['layer_indices'])}
    for i in range(cfg['depth']):
        b_next = block(sd, f'backbone.blocks.{i}', 'backbone.constant_time', b, sa_positions, heads, p)
        j = layer_map.get(i)
        if j is None:
            b = b_next
            continue
        c = block(sd, f'control.blocks.{j}', 'control.constant_time', c, sa_positions, heads, p)
        c = p.add(c, cross_attention(sd, f'cross.{j}', c, positions, kv_layers[j], heads, p))
        b = p.add(b_next, p.linear(c, sd[f'zero.{j}.weight'], sd[f'zero.{j}.bias']))
    return head(sd, b, shape, classes, patch, p)


# ------------------------------------------------------------------------------------------ condition encode

def _centers(shape, size):
    """`streamvoxel/stream/condition.py:201-204`."""
    grid = np.stack(np.meshgrid(*(np.arange(s) for s in shape), indexing='ij'), -1)
    return (grid[..., [2, 0, 1]] * size + size / 2).reshape(-1, 3).astype(np.float32)


def build_group(l1_xz, l2_xz, height, tile):
    """Positions of `build_group` `streamvoxel/stream/condition.py:207-223` (the item's own frame)."""
    offsets = lambda xz: np.stack((xz[:, 0], np.zeros(len(xz)), xz[:, 1]), -1).astype(np.float32)
    pos1 = (_centers((height // 4, tile // 4, tile // 4), 4)[None] + offsets(np.asarray(l1_xz).reshape(-1, 2))[:, None]) / 4
    pos2 = ((_centers((height // 16, 1, 1), 16)[None] + offsets(np.asarray(l2_xz).reshape(-1, 2))[:, None]) / 4).reshape(-1, 3)
    bio = (_centers((height // 4, 12, 12), 4) + np.asarray([-tile, 0, -tile], np.float32)) / 4
    return torch.from_numpy(pos1), torch.from_numpy(pos2), torch.from_numpy(bio)


def conv3d(x, w, b, stride, p):
    """Conv3d under autocast: bf16 conv without bias, then the bias added as a separate bf16 op."""
    return p.r(p.r(F.conv3d(p.r(x), p.r(w), None, stride=stride)) + p.r(b)[:, None, None, None])


def encode_columns(sd, tokens, level, classes, p):
    """`StreamingControlNet._encode_columns` `streaming_controlnet.py:142-158` for L1 (level 0) and L2 (level 1).

    The type/size embeddings are fp32 parameters, so their sum promotes to fp32 (no bf16 rounding)."""
    d = sd['type_embed.weight'].shape[1]
    if not len(tokens):
        count = (tokens.shape[1] // (16 if level else 4)) * (1 if level else 16)
        return torch.zeros((0, count, d))
    conv = 'l1_patch' if level == 0 else 'l2_patch'
    x = patchify(sd, conv, tokens, classes, p)  # [n, patches, d] in YZX patch order
    if level:
        n, _, d = x.shape
        x = F.gelu(p.layer_norm(x, 1e-5, sd['l2_norm.weight'], sd['l2_norm.bias']))
        h, t = tokens.shape[1] // 4, tokens.shape[2] // 4
        grid = x.reshape(n, h, t, t, d).permute(0, 4, 1, 2, 3)
        x = conv3d(grid, sd['l2_down.weight'], sd['l2_down.bias'], 4, p).flatten(2).transpose(1, 2)
    return x + sd['type_embed.weight'][level] + sd['size_embed.weight'][level]


def biome_condition(sd, biomes, bio_positions, height, halo, bpatch, p):
    """`StreamingControlNet._biome_condition` `streaming_controlnet.py:196-219` (halo 4 or 16, patch 1/2/4)."""
    if halo == 16 and bpatch == 1:
        values = sd['biome_embed.weight'][biomes.reshape(-1)][None]
        positions = bio_positions[None]
    else:
        labels = biomes.reshape(1, height // 4, 12, 12)
        positions = bio_positions.reshape(1, height // 4, 12, 12, 3)
        if halo == 4:
            labels, positions = labels[:, :, 3:9, 3:9], positions[:, :, 3:9, 3:9]
        values = sd['biome_embed.weight'][labels].permute(0, 4, 1, 2, 3)
        if bpatch > 1:
            pad = (-labels.shape[-1]) % bpatch
            mask = torch.ones((1, 1, height // 4, labels.shape[-2], labels.shape[-1]))
            fraction = F.avg_pool3d(F.pad(mask, (0, pad, 0, pad)), bpatch, bpatch)
            down = conv3d(F.pad(values, (0, pad, 0, pad)), sd['biome_down.weight'], sd['biome_down.bias'], bpatch, p)
            values = down / fraction
            coords = positions.permute(0, 4, 1, 2, 3)
            coords = F.avg_pool3d(F.pad(coords, (0, pad, 0, pad)), bpatch, bpatch) / fraction
            positions = coords.flatten(2).transpose(1, 2)
        else:
            positions = positions.reshape(1, -1, 3)
        values = values.flatten(2).transpose(1, 2)
    size = sd['biome_size8'] if bpatch == 2 else sd['size_embed.weight'][int(bpatch == 4)]
    values = values + sd['type_embed.weight'][2] + size
    return p.layer_norm(values, 1e-6), positions


def encode_kv(sd, l1_blocks, l1_xz, l2_blocks, l2_xz, biomes, cfg, bf16=False):
    """Packed per-layer cross K/V of one item: `encode_item` `streamvoxel/stream/engine.py:75-84` followed by
    `prefix_kv` (`streaming_controlnet.py:171-176`) and `local_kv` (`streamvoxel/stream/fast_ops.py:90-95`),
    prefix keys first (`fast_ops.py:228-239`). Returns [(k, v)] per control layer, each [1,H,L,D]."""
    prefix_kv, (local_kv, _, _) = encode_condition(sd, l1_blocks, l1_xz, l2_blocks, l2_xz, biomes, cfg, bf16)
    return [(torch.cat((pk, lk), 2), torch.cat((pv, lv), 2)) for (pk, pv), (lk, lv) in zip(prefix_kv, local_kv)]


def encode_condition(sd, l1_blocks, l1_xz, l2_blocks, l2_xz, biomes, cfg, bf16=False):
    """The pieces `engine.unpadded_logits` hands the model (`streamvoxel/stream/engine.py:75-102`): per control layer
    the prefix (k, v) [1,H,P,D] (keys rotated), and (local K/V per layer, the local condition tokens [1,L,d], their
    key positions [1,L,3])."""
    p = Precision(bf16)
    height, tile, classes, heads = cfg['voxel_shape'][0], cfg['voxel_shape'][1], cfg['num_classes'], cfg['num_heads']
    pos1, pos2, bio_pos = build_group(l1_xz, l2_xz, height, tile)
    l2 = encode_columns(sd, torch.as_tensor(l2_blocks).long(), 1, classes, p).flatten(0, 1)
    prefix = p.layer_norm(l2, 1e-6)
    l1 = p.layer_norm(encode_columns(sd, torch.as_tensor(l1_blocks).long(), 0, classes, p), 1e-6)
    bio, bio_positions = biome_condition(sd, torch.as_tensor(biomes).long(), bio_pos, height, cfg['biome_halo'],
                                         cfg['biome_patch'], p)
    local = torch.cat((l1.flatten(0, 1)[None], bio), 1)
    local_positions = torch.cat((pos1.reshape(1, -1, 3), bio_positions), 1)
    d = l2.shape[-1] if len(l2) else local.shape[-1]
    layers, locals_ = [], []
    for j in range(len(cfg['layer_indices'])):
        w, bias = sd[f'cross.{j}.key_value.weight'], sd[f'cross.{j}.key_value.bias']
        freq = rope_frequencies(d // heads)

        def kv(value, positions):
            k, v = p.linear(value, w, bias).reshape(value.shape[0], value.shape[1], 2, heads, d // heads).unbind(2)
            return rope(k.transpose(1, 2), positions, freq, p), v.transpose(1, 2)
        layers.append(kv(prefix[None], pos2[None]))
        locals_.append(kv(local, local_positions))
    return layers, (locals_, local, local_positions)
