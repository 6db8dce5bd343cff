"""Model configuration, seeded weights, device weight preparation and the per-window condition encoder.

The network is the reference's live model: a time-free AdaLN DiT backbone (`streamvoxel/models/
unconditional_md4_timefree.py`) plus a CompactStreamingControlNet with full width (`streamvoxel/models/
compact_controlnet.py`). Weights use the reference's state-dict names, so a reference checkpoint's state dict loads
unchanged. Everything a time-free model holds constant is precomputed here once, on the device, with the same torch
operations and bf16 autocast rounding the reference applies every forward:

* AdaLN vectors `ada(constant_time)` per block and the final `final_ada` (`timefree.py:58,120-121,171`);
* the per-position y-embedding `y_embed(y)` (`timefree.py:166-168`) and both RoPE sin/cos tables (`:24-30`);
* the patch-embed gather tables `GatherPatch.table` (`streamvoxel/stream/fast_ops.py:61-67`);
* the class head reordered so its output columns are class-major (n = v*64 + o).

The per-step forward then runs entirely in libsvx (`svx_engine_forward`).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

import numpy as np
import torch
import torch.nn.functional as F

from streamvoxel_b200 import _lib, ops
from streamvoxel_b200._lib import check


@dataclass(frozen=True)
class ModelConfig:
    classes: int = 256                  # V; the mask token id is V
    voxel_shape: tuple = (256, 16, 16)  # Y, Z, X
    patch: int = 4
    d: int = 768
    heads: int = 8                      # head_dim 96 (= d / heads), the only width the axial RoPE allows at d=768
    depth: int = 12
    mlp: int = 3072
    layer_indices: tuple = tuple(range(12))  # backbone layer fed by each control layer
    biome_halo: int = 4
    biome_patch: int = 4
    biome_classes: int = 16
    y_range: tuple = (-64., 192.)

    @property
    def patches(self):
        y, z, x = self.voxel_shape
        return (y // 4) * (z // 4) * (x // 4)

    @property
    def head_dim(self):
        return self.d // self.heads

    def condition_widths(self):
        """`streamvoxel/stream/engine.py:60-72`: tokens of one L1 tile, one L2 tile and the biome window."""
        height, tile = self.voxel_shape[0], self.voxel_shape[1]
        l1 = (height // 4) * (tile // 4) * (tile // 4)
        l2 = (height // 16) * (tile // 16) * (tile // 16)
        if self.biome_halo == 16 and self.biome_patch == 1:
            biome = (height // 4) * 12 * 12
        else:
            side = 6 if self.biome_halo == 4 else 12
            side += (-side) % self.biome_patch
            biome = (height // 4 // self.biome_patch) * (side // self.biome_patch) ** 2
        return l1, l2, biome


def dit_b4_control():
    """DiT-B/4 (d=768, 8 heads x 96, MLP 3072, 12 layers, V=256) + 12-layer ControlNet."""
    return ModelConfig()


def dit_l4_control():
    """the DiT-L/4-class backbone + a ControlNet of the same depth. d = 1024 cannot carry the axial
    RoPE (head_dim must be a multiple of 6: 1024 has no factor 3), so the nearest buildable width with the same
    96-wide heads: d = 1152, 12 heads x 96, MLP 4608, 24 layers, 24 control layers."""
    return ModelConfig(d=1152, heads=12, depth=24, mlp=4608, layer_indices=tuple(range(24)))


def dit_b4_unconditional():
    """the time-free DiT-B/4 alone (no ControlNet)."""
    return ModelConfig(layer_indices=())


def small_test_config(**overrides):
    """A small model with the same kernels (head_dim 96) for parity tests: d=192, 2 heads, 3 layers, V=32."""
    base = ModelConfig(classes=32, voxel_shape=(64, 16, 16), d=192, heads=2, depth=3, mlp=768, layer_indices=(0, 2),
                       biome_classes=16)
    return replace(base, **overrides)


def state_dict_shapes(cfg):
    """Every parameter the live path reads, with the reference's names and shapes (no buffers, no time MLP)."""
    d, v, m = cfg.d, cfg.classes, cfg.mlp
    shapes = {}

    def backbone_like(prefix, blocks):
        shapes[f'{prefix}.target_patch.weight'] = (d, v + 1, 4, 4, 4)
        shapes[f'{prefix}.target_patch.bias'] = (d,)
        shapes[f'{prefix}.y_embed.0.weight'] = (d, 1)
        shapes[f'{prefix}.y_embed.0.bias'] = (d,)
        shapes[f'{prefix}.y_embed.2.weight'] = (d, d)
        shapes[f'{prefix}.y_embed.2.bias'] = (d,)
        shapes[f'{prefix}.constant_time'] = (d,)
        for i in blocks:
            b = f'{prefix}.blocks.{i}'
            shapes.update({f'{b}.attn.qkv.weight': (3 * d, d), f'{b}.attn.qkv.bias': (3 * d,),
                           f'{b}.attn.proj.weight': (d, d), f'{b}.attn.proj.bias': (d,),
                           f'{b}.mlp.0.weight': (m, d), f'{b}.mlp.0.bias': (m,),
                           f'{b}.mlp.2.weight': (d, m), f'{b}.mlp.2.bias': (d,),
                           f'{b}.ada.1.weight': (6 * d, d), f'{b}.ada.1.bias': (6 * d,)})

    backbone_like('backbone', range(cfg.depth))
    shapes['backbone.final_ada.1.weight'] = (2 * d, d)
    shapes['backbone.final_ada.1.bias'] = (2 * d,)
    shapes['backbone.class_head.weight'] = (64 * v, d)
    shapes['backbone.class_head.bias'] = (64 * v,)
    if not cfg.layer_indices:
        return shapes
    backbone_like('control', range(len(cfg.layer_indices)))
    for j in range(len(cfg.layer_indices)):
        shapes.update({f'cross.{j}.query.weight': (d, d), f'cross.{j}.query.bias': (d,),
                       f'cross.{j}.key_value.weight': (2 * d, d), f'cross.{j}.key_value.bias': (2 * d,),
                       f'cross.{j}.proj.weight': (d, d), f'cross.{j}.proj.bias': (d,),
                       f'zero.{j}.weight': (d, d), f'zero.{j}.bias': (d,)})
    for name in ('l1_patch', 'l2_patch'):
        shapes[f'{name}.weight'] = (d, v + 1, 4, 4, 4)
        shapes[f'{name}.bias'] = (d,)
    shapes.update({'l2_norm.weight': (d,), 'l2_norm.bias': (d,), 'l2_down.weight': (d, d, 4, 4, 4),
                   'l2_down.bias': (d,), 'biome_embed.weight': (cfg.biome_classes, d),
                   'type_embed.weight': (3, d), 'size_embed.weight': (2, d)})
    if cfg.biome_patch > 1:
        p = cfg.biome_patch
        shapes['biome_down.weight'] = (d, d, p, p, p)
        shapes['biome_down.bias'] = (d,)
    if cfg.biome_patch == 2:
        shapes['biome_size8'] = (d,)
    return shapes


def synthetic_state_dict(cfg, seed=0, std=0.02):
    """Seeded random weights with the reference's names: every parameter re-drawn N(0, std^2) (the reference's own
    init zeroes the head and AdaLN outputs, which makes every logit 0). fp32 on the CPU."""
    g = torch.Generator().manual_seed(seed)
    sd = {}
    for name, shape in state_dict_shapes(cfg).items():
        sd[name] = torch.empty(shape).normal_(0.0, std, generator=g)
    return sd


def to_device(array, device, dtype=None):
    """A host array on `device` without blocking the host: staged in pinned memory and copied asynchronously on the
    current stream (a copy from pageable memory would first wait for all work already queued on that stream)."""
    host = torch.from_numpy(np.ascontiguousarray(array)) if isinstance(array, np.ndarray) else torch.as_tensor(array)
    if dtype is not None:
        host = host.to(dtype)
    return host.pin_memory().to(device, non_blocking=True)


def _bf16(t, device):
    return t.detach().to(device=device, dtype=torch.float32).to(torch.bfloat16).contiguous()


def patch_centers_xyz(voxel_shape, patch):
    """`unconditional_md4_timefree.py:84-86`: patch centres (x, y, z) in voxels, patch grid in YZX order."""
    grid = torch.stack(torch.meshgrid(*(torch.arange(v // patch).float() for v in voxel_shape), indexing='ij'), -1)
    return grid.reshape(-1, 3)[:, [2, 0, 1]] * patch + patch / 2


def rope_frequencies(head_dim, base=10000.):
    """`unconditional_md4_timefree.py:19-22`."""
    axis = head_dim // 3
    return base ** (-torch.arange(0, axis, 2).float() / axis)


def rope_tables(positions, head_dim):
    """sin/cos of `AxialRoPE.forward` (`timefree.py:26-27`): fp32 phases, rounded to bf16; [N, 3*16] axis-major."""
    phase = positions.float()[..., None] * rope_frequencies(head_dim).to(positions.device)
    n = positions.shape[0]
    return (phase.sin().to(torch.bfloat16).reshape(n, -1).contiguous(),
            phase.cos().to(torch.bfloat16).reshape(n, -1).contiguous())


def fold_layernorm(weight, bias, one_plus_scale=None, shift=None):
    """The LayerNorm + AdaLN modulate before a linear, folded into it (`svx_epilogue_args` ln_*): the linear then
    takes the raw residual stream x and computes r (x W'^T - mu u) + v, with mu, r the row's LayerNorm statistics.
    W' = bf16(W (1 + scale)) (exact fp32 product of two bf16 values, rounded once), u = sum_k W'[n, k],
    v = b + W shift (float64 sums, fp32). Without scale/shift (LayerNorm without affine) W' = W and v = b."""
    w = weight.float()
    folded = weight if one_plus_scale is None else (w * one_plus_scale.float()[None, :]).to(torch.bfloat16)
    u = folded.double().sum(1)
    v = bias.double() + (w.double() @ shift.double() if shift is not None else 0.)
    return folded.contiguous(), u.float().contiguous(), v.float().contiguous()


def down_conv_weight(weight):
    """The 4^3 stride-4 Conv3d weight [d_out, d_in, 4, 4, 4] as the [d_out, 64 d_in] bf16 weight of the GEMM that
    replaces it: an output token's 64 patches are consecutive patchified rows (patch order y, z, x over a 16-wide
    column, 16 patches per y layer), so A is the [tokens, 64 d_in] view with k = (ky * 16 + kz * 4 + kx) * d_in + c."""
    return weight.permute(0, 2, 3, 4, 1).reshape(weight.shape[0], -1).to(torch.bfloat16).contiguous()


class PreparedModel:
    """Device-resident bf16 weights and precomputed constants of one model (one per GPU)."""

    def __init__(self, cfg, state_dict, device):
        if cfg.patch != 4 or cfg.head_dim != 96:
            raise ValueError('the kernels implement patch 4 and head_dim 96')
        self.cfg = cfg
        self.device = torch.device(device)
        dev = self.device
        sd = {k: v.detach().to(dev, torch.float32) for k, v in state_dict.items()}
        self.sd = sd
        origin = torch.tensor([0., float(cfg.y_range[0]), 0.], device=dev)
        self.origin = origin
        local = patch_centers_xyz(cfg.voxel_shape, 4).to(dev)
        centers = local + origin
        y = 2 * (centers[:, 1:2] - cfg.y_range[0]) / (cfg.y_range[1] - cfg.y_range[0]) - 1
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
            self.backbone = [self._block(f'backbone.blocks.{i}', 'backbone.constant_time') for i in range(cfg.depth)]
            self.control = [self._block(f'control.blocks.{j}', 'control.constant_time')
                            for j in range(len(cfg.layer_indices))]
            shift, gain = self._ada('backbone.final_ada', 'backbone.constant_time', 2)
            self.final_shift, self.final_ops = shift, (1 + gain).contiguous()
            self.yadd_b = self._y_embed('backbone.y_embed', y)
            self.yadd_c = self._y_embed('control.y_embed', y) if cfg.layer_indices else self.yadd_b
        # Self-attention positions are the local patch centres / 4; cross-attention queries use the group-relative
        # centres (`compact_controlnet.py:104-108`), identical here because every slot shares the group origin.
        self.rope_sin, self.rope_cos = rope_tables(local / 4, 96)
        self.cross_sin, self.cross_cos = rope_tables((centers - origin) / 4, 96)
        self.table_b, self.bias_b = self._table('backbone.target_patch')
        self.table_c, self.bias_c = (self._table('control.target_patch') if cfg.layer_indices
                                     else (self.table_b, self.bias_b))
        v = cfg.classes
        head_w = sd['backbone.class_head.weight'].reshape(64, v, cfg.d).transpose(0, 1).reshape(64 * v, cfg.d)
        self.head_w = head_w.to(torch.bfloat16).contiguous()
        self.head_b = sd['backbone.class_head.bias'].reshape(64, v).t().reshape(-1).to(torch.bfloat16).contiguous()
        self.head_fold = fold_layernorm(self.head_w, self.head_b, self.final_ops, self.final_shift)
        self.cross = []
        for j in range(len(cfg.layer_indices)):
            self.cross.append({n: _bf16(sd[f'cross.{j}.{n}'], dev) for n in
                               ('query.weight', 'query.bias', 'proj.weight', 'proj.bias')} |
                              {'zero.weight': _bf16(sd[f'zero.{j}.weight'], dev),
                               'zero.bias': _bf16(sd[f'zero.{j}.bias'], dev)})
            self.cross[j]['query_fold'] = fold_layernorm(self.cross[j]['query.weight'], self.cross[j]['query.bias'])
        self.zero_yadd = torch.zeros((cfg.patches, cfg.d), device=dev, dtype=torch.bfloat16)
        if cfg.layer_indices:
            self.table_l1, self.bias_l1 = self._table('l1_patch')
            self.table_l2, self.bias_l2 = self._table('l2_patch')
            # the column encoder's constants: l2_norm's fp32 affine, the 4^3 down-conv as a [d, 64 d] GEMM weight in
            # (ky, kz, kx, d_in) order, its bias (bf16, added to the bf16 conv output), and each level's type + size
            # embeddings summed in fp32 (added before context_norm)
            self.l2_norm_w = sd['l2_norm.weight'].contiguous()
            self.l2_norm_b = sd['l2_norm.bias'].contiguous()
            self.l2_down_w = down_conv_weight(sd['l2_down.weight'])
            self.l2_down_b = sd['l2_down.bias'].to(torch.bfloat16)
            self.level_embed = [(sd['type_embed.weight'][i] + sd['size_embed.weight'][i]).contiguous() for i in (0, 1)]
            self.zero_bias = torch.zeros(cfg.d, device=dev, dtype=torch.bfloat16)
            self._down_bias_rows = self.l2_down_b[None].expand(256, cfg.d).contiguous()
        self.kv_weight = [_bf16(sd[f'cross.{j}.key_value.weight'], dev) for j in range(len(cfg.layer_indices))]
        self.kv_bias = [_bf16(sd[f'cross.{j}.key_value.bias'], dev) for j in range(len(cfg.layer_indices))]

    # -- constants
    def _ada(self, prefix, time_key, count):
        time = self.sd[time_key][None]
        out = F.linear(F.silu(time), self.sd[prefix + '.1.weight'], self.sd[prefix + '.1.bias'])[0]
        return [c.contiguous() for c in out.chunk(count)]

    def _block(self, prefix, time_key):
        s1, c1, g1, s2, c2, g2 = self._ada(prefix + '.ada', time_key, 6)
        w = {n: _bf16(self.sd[f'{prefix}.{n}'], self.device) for n in
             ('attn.qkv.weight', 'attn.qkv.bias', 'attn.proj.weight', 'attn.proj.bias', 'mlp.0.weight', 'mlp.0.bias',
              'mlp.2.weight', 'mlp.2.bias')}
        w.update(shift1=s1, ops1=(1 + c1).contiguous(), gate1=g1, shift2=s2, ops2=(1 + c2).contiguous(), gate2=g2)
        w['qkv_fold'] = fold_layernorm(w['attn.qkv.weight'], w['attn.qkv.bias'], w['ops1'], w['shift1'])
        w['fc1_fold'] = fold_layernorm(w['mlp.0.weight'], w['mlp.0.bias'], w['ops2'], w['shift2'])
        return w

    def _y_embed(self, prefix, y):
        h = F.silu(F.linear(y, self.sd[prefix + '.0.weight'], self.sd[prefix + '.0.bias']))
        return F.linear(h, self.sd[prefix + '.2.weight'], self.sd[prefix + '.2.bias']).contiguous()

    def _table(self, prefix):
        w = self.sd[prefix + '.weight']
        table = w.permute(1, 2, 3, 4, 0).reshape(-1, w.shape[0]).to(torch.bfloat16).contiguous()
        return table, self.sd[prefix + '.bias'].to(torch.bfloat16).contiguous()

    # -- per-window condition encoder (runs once per window, on the caller's stream)
    @torch.no_grad()
    def encode_item(self, l1_blocks, l1_xz, l2_blocks, l2_xz, biomes, l2_keys=None, cache=None):
        """Packed per-layer cross K/V of one window: `FastSlotForward.encode` (`streamvoxel/stream/fast_ops.py:228-239`)
        = `encode_item` (`streamvoxel/stream/engine.py:75-84`) -> `encode_group` / `prefix_kv` / `local_condition`
        (`streamvoxel/models/streaming_controlnet.py:160-219`) -> `local_kv` (`fast_ops.py:90-95`).
        Returns [(k, v)] per control layer, each [heads, L, 96] bf16 (RoPE on k), prefix keys first.
        With `l2_keys` (one hashable key per L2 column) and a `cache` (an `L2TokenCache`), each L2 column's encoded
        tokens (LayerNorm of its 16 down-sampled tokens, bf16) are computed once and reused: they depend on the
        column alone, its position enters through the RoPE of the keys only."""
        cfg, dev, sd = self.cfg, self.device, self.sd
        height, tile = cfg.voxel_shape[0], cfg.voxel_shape[1]
        pos1, pos2, bio_pos = _group_positions(l1_xz, l2_xz, height, tile, dev)
        with torch.autocast('cuda', dtype=torch.bfloat16):
            if l2_keys and cache is not None:
                prefix = cache.tokens(l2_keys, l2_blocks, self._l2_prefix)
            else:
                prefix = self._l2_prefix(np.asarray(l2_blocks))
            l1 = self._encode_columns(np.asarray(l1_blocks), 0)
            bio, bio_positions = self._biome(to_device(np.asarray(biomes, np.int64), dev), bio_pos)
            local = torch.cat((l1.flatten(0, 1), bio.to(torch.bfloat16)), 0)
            local_positions = torch.cat((pos1.reshape(-1, 3), bio_positions), 0)
        # Every layer's key_value linear over all condition tokens at once (prefix rows, then local rows).
        return self.key_values(torch.cat((prefix, local), 0), torch.cat((pos2, local_positions.float()), 0))

    @torch.no_grad()
    def key_values(self, tokens, positions):
        """Per control layer (k, v), each [heads, n, 96] bf16, of n encoded condition tokens [n, d] at key positions
        [n, 3]: `RotaryCrossAttention.encode_kv` (`streaming_controlnet.py:31-35`) = the key_value linear on the bf16
        input autocast would cast, then the axial RoPE of the keys. One tcgen05 GEMM per layer with the bias and the
        RoPE fused in its epilogue (the same bf16 rounding points as `F.linear` then `AxialRoPE`), tables built once."""
        cfg, dev = self.cfg, self.device
        n = len(tokens)
        rows = -(-n // 256) * 256
        padded = torch.zeros((rows, cfg.d), device=dev, dtype=torch.bfloat16)
        padded[:n] = tokens.to(device=dev, dtype=torch.bfloat16)
        if not hasattr(self, '_key_freq'):
            self._key_freq = rope_frequencies(96).to(dev)
        phase = (positions.to(dev).float()[..., None] * self._key_freq).reshape(n, 48)
        sin = torch.zeros((rows, 48), device=dev, dtype=torch.bfloat16)
        cos = torch.zeros((rows, 48), device=dev, dtype=torch.bfloat16)
        sin[:n], cos[:n] = phase.sin().to(torch.bfloat16), phase.cos().to(torch.bfloat16)
        layers = []
        for j in range(len(cfg.layer_indices)):
            out = ops.gemm(padded, self.kv_weight[j], self.kv_bias[j], _lib.EPI_ROPE, rope=(sin, cos),
                           rope_cols=cfg.d, rows_per_slot=rows)
            kv = out[:n].view(n, 2, cfg.heads, 96)
            layers.append((kv[:, 0].transpose(0, 1), kv[:, 1].transpose(0, 1)))
        return layers

    def _l2_prefix(self, blocks):
        """Encoded prefix tokens of L2 columns [n, H, T, T] -> [n * H / 16, d] bf16 (the cast the key_value linear
        makes)."""
        return self._encode_columns(blocks, 1).flatten(0, 1)

    def _encode_columns(self, tokens, level):
        """`_encode_columns` (`streaming_controlnet.py:142-158`) and `context_norm` (`:167-168`) on libsvx kernels:
        the one-hot conv patchify (the gather kernel); for L2 `l2_norm` + GELU (`svx_layernorm_affine`, fp32) and the
        4^3 stride-4 down-conv as one GEMM: the 64 patches under an output token are 64 consecutive rows of the
        patchified column (patch order y, z, x with 4 x 4 patches per y), so A is the [n H/16, 64 d] view and W the
        conv weight in (ky, kz, kx, d_in) order; the conv's bias is added to its bf16 output in bf16 (the separate
        bias add of the conv under autocast) by the residual epilogue over rows of the bias. Then the type + size
        embeddings and the no-affine LayerNorm (`svx_layernorm_affine` with `pre`; the two fp32 embeddings summed
        once, not added one after the other). Returns [n, count, d] bf16."""
        cfg, dev = self.cfg, self.device
        height, tile = cfg.voxel_shape[0], cfg.voxel_shape[1]
        count = (height // 16) if level else cfg.patches
        if len(tokens) == 0:
            return torch.zeros((0, count, cfg.d), device=dev, dtype=torch.bfloat16)
        t = to_device(np.asarray(tokens, np.int16), dev)
        table, bias = (self.table_l1, self.bias_l1) if level == 0 else (self.table_l2, self.bias_l2)
        n = len(t)
        if not level:
            x, _ = ops.patch_embed(t, cfg.classes, table, bias, self.zero_yadd)
            return ops.layernorm_affine(x, 1e-6, pre=self.level_embed[0]).view(n, count, cfg.d)
        if tile != 16:
            raise ValueError('the L2 down-conv takes 16-wide columns (one output token per 4 patch layers)')
        rows = n * count
        padded = -(-rows // 256) * 256
        grid = torch.zeros((padded * 64, cfg.d), device=dev, dtype=torch.bfloat16)
        x, _ = ops.patch_embed(t, cfg.classes, table, bias, self.zero_yadd, out_b=grid[:rows * 64])
        ops.layernorm_affine(x, 1e-5, weight=self.l2_norm_w, bias=self.l2_norm_b, gelu=True, out=x)
        if len(self._down_bias_rows) < padded:
            self._down_bias_rows = self.l2_down_b[None].expand(padded, cfg.d).contiguous()
        down = ops.gemm(grid.view(padded, 64 * cfg.d), self.l2_down_w, self.zero_bias, _lib.EPI_RESIDUAL,
                        residual=self._down_bias_rows[:padded])
        return ops.layernorm_affine(down[:rows], 1e-6, pre=self.level_embed[1]).view(n, count, cfg.d)

    def _biome(self, biomes, bio_positions):
        """`_biome_condition` (`streaming_controlnet.py:196-219`) on libsvx kernels: the biome embedding rows gathered
        (bf16, the cast autocast makes for the down-conv), the p^3 stride-p down-conv as one GEMM over the gathered
        rows with its bf16 bias add in the residual epilogue, then the type + size embeddings and the no-affine
        LayerNorm (`svx_layernorm_affine` with `pre`). The division by the window fraction of a padded block
        (1, 1/2 or 1/4 for p = 4: always a power of two) is applied to the gathered rows and to the bias rows, which is
        exact and commutes with every bf16 rounding, so the result equals bf16(bf16(conv) + bias) / fraction. The
        pooled key positions depend only on the window geometry and are computed once. Returns (values [T, d] bf16,
        positions [T, 3])."""
        cfg, dev = self.cfg, self.device
        height = cfg.voxel_shape[0]
        if not hasattr(self, '_biome_plan'):
            self._biome_plan = self._plan_biome(bio_positions)
        index, scale, positions, bias_rows, tokens = self._biome_plan
        labels = biomes.reshape(-1)
        if cfg.biome_halo != 16 or cfg.biome_patch != 1:
            labels = biomes.reshape(height // 4, 12, 12)
            if cfg.biome_halo == 4:
                labels = labels[:, 3:9, 3:9]
            labels = labels.reshape(-1)
        # padded grid cells point at the zero row appended to the table
        padded = torch.cat((labels, labels.new_full((1,), cfg.biome_classes)))
        rows = self._biome_table[padded[index]]                     # [T or rows, p^3, d] bf16
        if cfg.biome_patch == 1:
            x = rows.reshape(tokens, cfg.d)
        else:
            p3 = cfg.biome_patch ** 3
            a = (rows * scale[:, None, None]).reshape(-1, p3 * cfg.d).contiguous()
            x = ops.gemm(a, self._biome_down_w, self.zero_bias, _lib.EPI_RESIDUAL, residual=bias_rows)[:tokens]
        return ops.layernorm_affine(x.contiguous(), 1e-6, pre=self._biome_pre), positions

    def _plan_biome(self, bio_positions):
        """Constants of the biome branch (window geometry only): the gather index of every down-conv input row, the
        1/fraction scale per output token, the pooled key positions and the bias rows (bias / fraction, bf16)."""
        cfg, dev, sd = self.cfg, self.device, self.sd
        height, p = cfg.voxel_shape[0], cfg.biome_patch
        table = torch.cat((sd['biome_embed.weight'], torch.zeros((1, cfg.d), device=dev)), 0)
        self._biome_table = table.to(torch.bfloat16)
        size = sd['biome_size8'] if p == 2 else sd['size_embed.weight'][int(p == 4)]
        self._biome_pre = (sd['type_embed.weight'][2] + size).contiguous()
        if cfg.biome_halo == 16 and p == 1:
            n = bio_positions.reshape(-1, 3).shape[0]
            return torch.arange(n, device=dev), None, bio_positions.reshape(-1, 3), None, n
        side = 6 if cfg.biome_halo == 4 else 12
        positions = bio_positions.reshape(height // 4, 12, 12, 3)
        if cfg.biome_halo == 4:
            positions = positions[:, 3:9, 3:9]
        if p == 1:
            n = height // 4 * side * side
            return torch.arange(n, device=dev), None, positions.reshape(-1, 3), None, n
        pad = (-side) % p
        grid = side + pad
        cells = torch.arange(height // 4 * side * side, device=dev).reshape(height // 4, side, side)
        cells = F.pad(cells, (0, pad, 0, pad), value=height // 4 * side * side)   # the zero row
        gy, gz = height // 4 // p, grid // p
        blocks = cells.reshape(gy, p, gz, p, gz, p).permute(0, 2, 4, 1, 3, 5).reshape(gy * gz * gz, p ** 3)
        valid = F.pad(torch.ones((1, 1, height // 4, side, side), device=dev), (0, pad, 0, pad))
        fraction = F.avg_pool3d(valid, p, p).reshape(-1)
        coords = F.avg_pool3d(F.pad(positions.permute(3, 0, 1, 2)[None], (0, pad, 0, pad)), p, p)[0]
        pooled = (coords / fraction.reshape(gy, gz, gz)[None]).reshape(3, -1).t().contiguous()
        tokens = len(blocks)
        rows = -(-tokens // 256) * 256
        index = torch.full((rows, p ** 3), height // 4 * side * side, device=dev, dtype=torch.long)
        index[:tokens] = blocks
        scale = torch.ones(rows, device=dev)
        scale[:tokens] = 1.0 / fraction
        self._biome_down_w = down_conv_weight(sd['biome_down.weight'])
        bias = sd['biome_down.bias'].to(torch.bfloat16).float()
        bias_rows = (bias[None] * scale[:, None]).to(torch.bfloat16).contiguous()
        return index, scale.to(torch.bfloat16), pooled, bias_rows, tokens


class L2TokenCache:
    """Encoded L2 tokens per committed column (LRU, at most `capacity` columns; 24 KB each at d = 768)."""

    def __init__(self, capacity=32768):
        from collections import OrderedDict
        self.capacity, self.entries = int(capacity), OrderedDict()
        self.hits = self.misses = 0

    def tokens(self, keys, blocks, encode):
        missing = [i for i, key in enumerate(keys) if key not in self.entries]
        self.hits += len(keys) - len(missing)
        self.misses += len(missing)
        if missing:
            try:   # an array or a lazy column stack copies only the columns asked for
                picked = np.asarray(blocks[missing])
            except TypeError:   # a list of tiles
                picked = np.asarray(blocks)[missing]
            fresh = encode(picked)
            per = len(fresh) // len(missing)
            for n, i in enumerate(missing):
                self.entries[keys[i]] = fresh[n * per:(n + 1) * per]
        rows = []
        for key in keys:
            self.entries.move_to_end(key)
            rows.append(self.entries[key])
        while len(self.entries) > self.capacity:
            self.entries.popitem(last=False)
        return torch.cat(rows, 0)


def _rope(x, positions, freq):
    """`AxialRoPE.forward` on [H, N, D] bf16 (`timefree.py:24-30`): bf16 element-wise ops, fp32 phases."""
    phase = positions.float()[..., None] * freq
    sin, cos = phase.sin()[None].to(x.dtype), phase.cos()[None].to(x.dtype)
    pairs = x.reshape(*x.shape[:-1], 3, x.shape[-1] // 6, 2)
    a, b = pairs.unbind(-1)
    return torch.stack((a * cos - b * sin, a * sin + b * cos), -1).flatten(-3)


def _centers(shape, size):
    """`streamvoxel/stream/condition.py:201-204`."""
    grid = np.stack(np.meshgrid(*(np.arange(s) for s in shape), indexing='ij'), -1)
    return (grid[..., [2, 0, 1]] * size + size / 2).reshape(-1, 3).astype(np.float32)


def _group_positions(l1_xz, l2_xz, height, tile, device):
    """Key positions of `build_group` (`streamvoxel/stream/condition.py:207-223`) in the target's frame."""
    offsets = lambda xz: np.stack((xz[:, 0], np.zeros(len(xz)), xz[:, 1]), -1).astype(np.float32)
    l1_xz, l2_xz = np.asarray(l1_xz).reshape(-1, 2), np.asarray(l2_xz).reshape(-1, 2)
    pos1 = (_centers((height // 4, tile // 4, tile // 4), 4)[None] + offsets(l1_xz)[:, None]) / 4
    pos2 = ((_centers((height // 16, 1, 1), 16)[None] + offsets(l2_xz)[:, None]) / 4).reshape(-1, 3)
    bio = (_centers((height // 4, 12, 12), 4) + np.asarray([-tile, 0, -tile], np.float32)) / 4
    return to_device(pos1, device), to_device(pos2, device), to_device(bio, device)


class Engine:
    """Owner of one `svx_engine` handle: packed K/V buffers, per-slot key lengths and the activation workspace."""

    def __init__(self, model, slots, key_capacity):
        cfg, dev = model.cfg, model.device
        self.model, self.cfg, self.slots = model, cfg, int(slots)
        self.key_capacity = int(key_capacity)
        rows = self.slots * cfg.patches
        bf = dict(device=dev, dtype=torch.bfloat16)
        n_control = len(cfg.layer_indices)
        self.kv = [(torch.zeros((self.slots, cfg.heads, self.key_capacity, 96), **bf),
                    torch.zeros((self.slots, cfg.heads, self.key_capacity, 96), **bf)) for _ in range(n_control)]
        self.lengths = torch.zeros(self.slots, dtype=torch.int32, device=dev)
        self.host_lengths = (ctypes.c_int32 * self.slots)()
        self.pending_lengths = {}
        self.ws = {n: torch.zeros((rows, w), **bf) for n, w in
                   (('xb', cfg.d), ('xc', cfg.d), ('h', cfg.d), ('qkv', 3 * cfg.d), ('attn', cfg.d), ('mlp', cfg.mlp),
                    ('qx', cfg.d), ('ax', cfg.d))}
        # row statistics of the residual streams for the folded LayerNorms: chunk-major [d/32][n*patches] (mean, M2)
        self.stats = {n: torch.zeros((cfg.d // 32, rows, 2), device=dev, dtype=torch.float32) for n in ('b', 'c')}
        p = lambda t: t.data_ptr()

        def block(w):
            (qkv_w, qkv_u, qkv_v), (fc1_w, fc1_u, fc1_v) = w['qkv_fold'], w['fc1_fold']
            return _lib.BlockWeights(p(qkv_w), p(w['attn.qkv.bias']), p(w['attn.proj.weight']),
                                     p(w['attn.proj.bias']), p(fc1_w), p(w['mlp.0.bias']),
                                     p(w['mlp.2.weight']), p(w['mlp.2.bias']), p(w['shift1']), p(w['ops1']),
                                     p(w['gate1']), p(w['shift2']), p(w['ops2']), p(w['gate2']),
                                     p(qkv_u), p(qkv_v), p(fc1_u), p(fc1_v))
        self._backbone = (_lib.BlockWeights * cfg.depth)(*[block(w) for w in model.backbone])
        self._control = (_lib.BlockWeights * max(1, n_control))(*[block(w) for w in model.control])
        self._cross = (_lib.CrossWeights * max(1, n_control))(*[
            _lib.CrossWeights(p(c['query.weight']), p(c['query.bias']), p(c['proj.weight']), p(c['proj.bias']),
                              p(c['zero.weight']), p(c['zero.bias']), p(k), p(v), p(c['query_fold'][1]),
                              p(c['query_fold'][2]))
            for c, (k, v) in zip(model.cross, self.kv)])
        self._layer_index = (ctypes.c_int32 * max(1, n_control))(*cfg.layer_indices)
        y, z, x = cfg.voxel_shape
        self._config = _lib.EngineConfig(self.slots, y, z, x, 4, cfg.classes, cfg.d, cfg.heads, cfg.mlp, cfg.depth,
                                         self.key_capacity, n_control, self._layer_index)
        self._weights = _lib.EngineWeights(
            p(model.table_b), p(model.bias_b), p(model.yadd_b), p(model.table_c), p(model.bias_c), p(model.yadd_c),
            self._backbone, self._control, self._cross, p(model.final_shift), p(model.final_ops),
            p(model.head_fold[0]), p(model.head_b), p(model.rope_sin), p(model.rope_cos), p(model.cross_sin),
            p(model.cross_cos), p(self.lengths), p(model.head_fold[1]), p(model.head_fold[2]))
        self._workspace = _lib.EngineWorkspace(*[p(self.ws[n]) for n in
                                                 ('xb', 'xc', 'h', 'qkv', 'attn', 'mlp', 'qx', 'ax')],
                                               p(self.stats['b']), p(self.stats['c']))
        handle = ctypes.c_void_p()
        check(_lib.load().svx_engine_create(ctypes.byref(self._config), ctypes.byref(self._weights),
                                            ctypes.byref(self._workspace), ctypes.byref(handle)), 'svx_engine_create')
        self.handle = handle

    def write_slot(self, index, layers, defer=False):
        """Copy one window's packed K/V into slot `index` (`FastSlotForward._write`, `fast_ops.py:241-250`). With
        `defer`, the slot's key length (and the attention work plans built from the lengths) is applied later by
        `apply_lengths`, on the stream that runs the forward."""
        length = layers[0][0].shape[1]
        if length > self.key_capacity:
            raise ValueError('Condition exceeds the captured capacity')
        # Rows past the length are left as they are: the attention kernel loads only the tiles that hold the slot's
        # keys and gives the keys past its length in the last tile a zero weight, so stale (finite) rows there never
        # reach an output.
        for (sk, sv), (k, v) in zip(self.kv, layers):
            sk[index, :, :length].copy_(k)
            sv[index, :, :length].copy_(v)
        self.pending_lengths[index] = length
        if not defer:
            self.apply_lengths()

    def apply_lengths(self):
        """Set the pending slot key lengths on the current stream and rebuild the attention plans (their copy to the
        device waits for the work queued on this stream, so run it where no step is in flight)."""
        if not self.pending_lengths:
            return
        for index, length in self.pending_lengths.items():
            self.lengths[index] = length
            self.host_lengths[index] = length
        self.pending_lengths = {}
        check(_lib.load().svx_engine_set_lengths(self.handle, self.host_lengths, _lib.stream_ptr(None)),
              'svx_engine_set_lengths')

    def forward(self, n, tokens, logits, stream=None):
        """Logits of the first n slots into `logits` [>= n, V, Y, Z, X] bf16 from int16 tokens."""
        assert tokens.dtype == torch.int16 and tokens.is_contiguous() and logits.dtype == torch.bfloat16
        check(_lib.load().svx_engine_forward(self.handle, int(n), _lib.ptr(tokens), _lib.ptr(logits),
                                             _lib.stream_ptr(stream)), 'svx_engine_forward')
        return logits

    def launches(self, n):
        return _lib.load().svx_engine_launches(self.handle, int(n))

    def close(self):
        if getattr(self, 'handle', None):
            _lib.load().svx_engine_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
