"""An object with the attribute surface of the reference's model classes (TEST INFRASTRUCTURE ONLY).

`streamvoxel_b200.modules.prepare` reads a `CompactStreamingControlNet` / time-free `UnconditionalMD4DiT` through the
attributes below and `state_dict()`; the reference package is not importable on the GPU box, so the GPU tests hand
the drop-ins this stand-in, and `tests/test_modules_host.py` checks on the CPU that the real reference objects give
the same configuration and parameter names.
"""
from __future__ import annotations


class _Attrs:
    def __init__(self, **kwargs):
        self.__dict__.update(kwargs)


def reference_like(cfg, state_dict):
    """A ControlNet-shaped object (a bare DiT when `cfg.layer_indices` is empty) holding `state_dict`."""
    bb = _Attrs(num_classes=cfg.classes, voxel_shape=tuple(cfg.voxel_shape), patch_size=4, hidden_dim=cfg.d,
                depth=cfg.depth, num_heads=cfg.heads, mlp_ratio=cfg.mlp / cfg.d, y_range=tuple(cfg.y_range),
                time_free=True, constant_time=state_dict['backbone.constant_time'])
    if not cfg.layer_indices:
        bb.state_dict = lambda: {k[len('backbone.'):]: v for k, v in state_dict.items() if k.startswith('backbone.')}
        return bb
    control = _Attrs(hidden_dim=cfg.d, mlp_ratio=cfg.mlp / cfg.d, depth=len(cfg.layer_indices))
    model = _Attrs(backbone=bb, control=control, cross=[None] * len(cfg.layer_indices),
                   layer_indices=tuple(cfg.layer_indices), biome_halo=cfg.biome_halo, biome_patch=cfg.biome_patch,
                   biome_embed=_Attrs(num_embeddings=cfg.biome_classes), struct_classes=0)
    model.state_dict = lambda: dict(state_dict)
    return model
