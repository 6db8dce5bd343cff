"""Drop-ins for the model forwards the reference calls (`streamvoxel/models`), on the libsvx engine.

* `prepare(model)`: a reference model object -- a `CompactStreamingControlNet` (`compact_controlnet.py:10-159`, the
  class the live worker loads) or a bare time-free `UnconditionalMD4DiT` (`unconditional_md4_timefree.py:66-177`) --
  becomes (`ModelConfig`, state dict) read from its attributes and `state_dict()`, so
  `FastSlotForward(model, spec, ...)` takes the module exactly as `Worker.run_loop` passes it
  (`streamvoxel/stream/worker.py:272`).
* `ControlNetForward(model)(tokens, *, timestep, origin_xyz, group_origin_xyz, prefix_kv, local, local_positions)`:
  `CompactStreamingControlNet.forward` (`compact_controlnet.py:100-159`) for one batch of conditions: the prefix K/V
  (keys already rotated, `RotaryCrossAttention.encode_kv`), the local condition tokens and their key positions, as
  `engine.unpadded_logits` hands them over (`streamvoxel/stream/engine.py:87-102`).
* `DiTForward(model)(tokens, *, timestep, origin_xyz=None)`: `UnconditionalMD4DiT.forward` (`timefree.py:152-177`).

Both forwards return bf16 logits [B, V, Y, Z, X] (the dtype the reference's class head returns under CUDA autocast)
and raise `ValueError` for inputs the reference rejects or the engine does not implement. The timestep is checked
for shape and otherwise ignored: the time-free model's AdaLN vectors are constants.
"""
from __future__ import annotations

import torch

from streamvoxel_b200 import _lib
from streamvoxel_b200.model import Engine, ModelConfig, PreparedModel, state_dict_shapes

KEY_BLOCK = 128


def _is_controlnet(model):
    return hasattr(model, 'backbone') and hasattr(model, 'cross') and hasattr(model, 'control')


def model_config(model):
    """The `ModelConfig` of a reference model object (attributes of `UnconditionalMD4DiT.__init__`,
    `timefree.py:67-78`, and of the ControlNet, `streaming_controlnet.py:64-128`, `compact_controlnet.py:89-98`)."""
    control = _is_controlnet(model)
    bb = model.backbone if control else model
    if not getattr(bb, 'time_free', False) or not hasattr(bb, 'constant_time'):
        raise ValueError('the engine runs the time-free AdaLN backbone (unconditional_md4_timefree, time_free=True)')
    if int(bb.patch_size) != 4:
        raise ValueError('the engine implements patch size 4')
    d, heads = int(bb.hidden_dim), int(bb.num_heads)
    mlp = int(d * bb.mlp_ratio)
    fields = dict(classes=int(bb.num_classes), voxel_shape=tuple(int(v) for v in bb.voxel_shape), patch=4, d=d,
                  heads=heads, depth=int(bb.depth), mlp=mlp, y_range=tuple(float(v) for v in bb.y_range))
    if not control:
        return ModelConfig(layer_indices=(), **fields)
    if int(model.control.hidden_dim) != d or mlp != int(model.control.hidden_dim * model.control.mlp_ratio):
        raise ValueError('the engine runs a control branch of the backbone width (control_hidden_dim = hidden_dim)')
    if int(getattr(model, 'struct_classes', 0)):
        raise ValueError('structure tokens (struct_classes > 0) are not on the live path')
    indices = getattr(model, 'layer_indices', None)
    indices = tuple(range(int(bb.depth))) if indices is None else tuple(int(i) for i in indices)
    return ModelConfig(layer_indices=indices, biome_halo=int(model.biome_halo), biome_patch=int(model.biome_patch),
                       biome_classes=int(model.biome_embed.num_embeddings), **fields)


def prepare(model):
    """(`ModelConfig`, state dict with the reference's names) of a reference model object. A bare DiT's parameters
    are named under `backbone.`, as in the ControlNet. Raises `ValueError` when a parameter the path reads is missing
    or has another shape."""
    cfg = model_config(model)
    raw = model.state_dict()
    if not _is_controlnet(model):
        raw = {'backbone.' + k: v for k, v in raw.items()}
    state = {}
    for name, shape in state_dict_shapes(cfg).items():
        if name not in raw:
            raise ValueError(f'the model has no parameter {name}')
        if tuple(raw[name].shape) != tuple(shape):
            raise ValueError(f'{name} has shape {tuple(raw[name].shape)}, expected {tuple(shape)}')
        state[name] = raw[name].detach()
    return cfg, state


def prepared_model(model, device):
    """A `PreparedModel` on `device` from a `PreparedModel`, a (`ModelConfig`, state dict) pair or a reference model
    object."""
    if isinstance(model, PreparedModel):
        return model
    if isinstance(model, tuple) and len(model) == 2 and isinstance(model[0], ModelConfig):
        cfg, state = model
    else:
        cfg, state = prepare(model)
    return PreparedModel(cfg, state, device)


def _check_origin(cfg, origin_xyz, batch):
    """The engine precomputes the y-embedding for patch centres at the origin (0, y_range[0], 0), the origin the live
    path always uses (`streamvoxel/stream/engine.py:98`, `ModelSpec.y_origin`); x and z of an origin cancel."""
    if origin_xyz is None:
        return
    origin = torch.as_tensor(origin_xyz, dtype=torch.float32).cpu()
    if tuple(origin.shape) != (batch, 3):
        raise ValueError('Expected per-sample XYZ origin')
    if not bool((origin[:, 1] == float(cfg.y_range[0])).all()):
        raise ValueError(f'the engine takes origins at y = {cfg.y_range[0]} (the model y_range start)')


class DiTForward:
    """`UnconditionalMD4DiT.forward(tokens, *, timestep, origin_xyz=None)` of the time-free backbone on libsvx."""

    def __init__(self, model, device='cuda'):
        self.device = torch.device(device)
        _lib.require_device(self.device)
        self.model = prepared_model(model, self.device)
        self.cfg = self.model.cfg
        if self.cfg.layer_indices:
            raise ValueError('DiTForward runs the backbone alone (use ControlNetForward for a ControlNet)')
        self.engine, self.logits = None, None

    def _engine(self, batch):
        if self.engine is None or self.engine.slots < batch:
            self.engine = Engine(self.model, batch, 0)
            self.logits = torch.empty((batch, self.cfg.classes, *self.cfg.voxel_shape), dtype=torch.bfloat16,
                                      device=self.device)
        return self.engine

    @torch.no_grad()
    def __call__(self, tokens, *, timestep, origin_xyz=None):
        cfg = self.cfg
        if tokens.ndim != 4 or tuple(tokens.shape[1:]) != tuple(cfg.voxel_shape):
            raise ValueError('Invalid target shape')
        if tuple(torch.as_tensor(timestep).shape) != (len(tokens),):
            raise ValueError('Invalid time shape')
        _check_origin(cfg, origin_xyz, len(tokens))
        batch = len(tokens)
        engine = self._engine(batch)
        t = tokens.to(device=self.device, dtype=torch.int16).contiguous()
        engine.forward(batch, t, self.logits)
        return self.logits[:batch].clone()


class ControlNetForward:
    """`CompactStreamingControlNet.forward` (scale 1) on libsvx for one batch of per-sample conditions.

    prefix_kv[j] = (k, v), each [B, H, P, 96] (keys rotated), per control layer; local [B, L, d] encoded local
    condition tokens with key positions local_positions [B, L, 3]; the local keys and values are projected here
    (`RotaryCrossAttention.forward`, `streaming_controlnet.py:37-61`, the 4-d prefix branch) and packed after the
    prefix into the engine's per-slot key buffers."""

    def __init__(self, model, device='cuda'):
        self.device = torch.device(device)
        _lib.require_device(self.device)
        self.model = prepared_model(model, self.device)
        self.cfg = self.model.cfg
        if not self.cfg.layer_indices:
            raise ValueError('ControlNetForward needs a model with control layers (use DiTForward for the backbone)')
        self.engine, self.logits = None, None

    def _engine(self, batch, keys):
        capacity = keys + (-keys) % KEY_BLOCK
        if self.engine is None or self.engine.slots < batch or self.engine.key_capacity < capacity:
            slots = batch if self.engine is None else max(batch, self.engine.slots)
            capacity = capacity if self.engine is None else max(capacity, self.engine.key_capacity)
            self.engine = Engine(self.model, slots, capacity)
            self.logits = torch.empty((slots, self.cfg.classes, *self.cfg.voxel_shape), dtype=torch.bfloat16,
                                      device=self.device)
        return self.engine

    @torch.no_grad()
    def __call__(self, tokens, *, timestep, origin_xyz, group_origin_xyz, prefix_kv, local, local_positions,
                 scale=1.):
        cfg = self.cfg
        if float(scale) != 1.0:
            raise ValueError('the engine runs the ControlNet at scale 1 (the live path)')
        if tokens.ndim != 4 or tuple(tokens.shape[1:]) != tuple(cfg.voxel_shape):
            raise ValueError('Invalid target shape')
        batch = len(tokens)
        if tuple(torch.as_tensor(timestep).shape) != (batch,):
            raise ValueError('Invalid time shape')
        _check_origin(cfg, origin_xyz, batch)
        origin = torch.as_tensor(origin_xyz, dtype=torch.float32).cpu()
        group = torch.as_tensor(group_origin_xyz, dtype=torch.float32).cpu()
        group = group[None].expand(batch, 3) if group.ndim == 1 else group
        if tuple(group.shape) != (batch, 3) or not torch.equal(group, origin):
            raise ValueError('the engine takes the group origin equal to each sample origin (cross-attention query '
                             'positions are the local patch centres)')
        if len(prefix_kv) != len(cfg.layer_indices):
            raise ValueError(f'prefix_kv must hold one (k, v) per control layer ({len(cfg.layer_indices)})')
        prefix = prefix_kv[0][0].shape[2]
        for k, v in prefix_kv:
            if tuple(k.shape) != (batch, cfg.heads, prefix, 96) or tuple(v.shape) != tuple(k.shape):
                raise ValueError('Slot prefix K/V must be [batch, heads, keys, dim]')
        if local.ndim != 3 or len(local) != batch or local.shape[2] != cfg.d:
            raise ValueError('local must be [batch, keys, width]')
        if tuple(local_positions.shape) != (batch, local.shape[1], 3):
            raise ValueError('local_positions must be [batch, keys, 3]')
        count = local.shape[1]
        engine = self._engine(batch, prefix + count)
        projected = self.model.key_values(local.reshape(batch * count, cfg.d),
                                          local_positions.reshape(batch * count, 3))
        for slot in range(batch):
            rows = slice(slot * count, (slot + 1) * count)
            layers = []
            for (pk, pv), (lk, lv) in zip(prefix_kv, projected):
                layers.append((torch.cat((pk[slot].to(self.device, torch.bfloat16), lk[:, rows]), 1),
                               torch.cat((pv[slot].to(self.device, torch.bfloat16), lv[:, rows]), 1)))
            engine.write_slot(slot, layers)
        t = tokens.to(device=self.device, dtype=torch.int16).contiguous()
        engine.forward(batch, t, self.logits)
        return self.logits[:batch].clone()
