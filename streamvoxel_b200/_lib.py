"""ctypes binding of libsvx.so (include/svx.h). The product path has no fallback: if the library is missing or the
device is not sm_100, calls raise.

Status codes map to the reference's exceptions: SVX_ERR_INVALID -> ValueError (shape / capacity, as
`streamvoxel/stream/fast_ops.py:233,244`), anything else -> RuntimeError.
"""
from __future__ import annotations

import ctypes
import os
import re

PACKAGE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(PACKAGE, 'libsvx.so')
HEADER = os.path.join(os.path.dirname(PACKAGE), 'include', 'svx.h')

SVX_OK, SVX_ERR_INVALID, SVX_ERR_CUDA, SVX_ERR_UNSUPPORTED = 0, 1, 2, 3
STATUS_QUOTA_MISSED, STATUS_NAN_LOGITS, STATUS_WAIT_TIMEOUT = 0x1, 0x2, 0x4
F32, BF16 = 0, 1
EPI_BIAS, EPI_BIAS_GELU, EPI_GATE_RESIDUAL, EPI_RESIDUAL, EPI_ROPE, EPI_CLASS_MAJOR = range(6)

c_ptr = ctypes.c_void_p
c_int = ctypes.c_int
c_i64 = ctypes.c_int64


class StepParams(ctypes.Structure):
    """`svx_step_params`."""
    _fields_ = [('k', ctypes.c_int32), ('step', ctypes.c_int32), ('committed', ctypes.c_int64),
                ('frac', ctypes.c_double), ('seed', ctypes.c_uint64)]


class EpilogueArgs(ctypes.Structure):
    """`svx_epilogue_args`."""
    _fields_ = [('epilogue', c_int), ('bias', c_ptr), ('gate', c_ptr), ('residual', c_ptr), ('rope_sin', c_ptr),
                ('rope_cos', c_ptr), ('rope_cols', c_int), ('rows_per_slot', c_int), ('head_dim', c_int),
                ('classes', c_int), ('height', c_int), ('depth', c_int), ('width', c_int), ('patch', c_int),
                ('ln_stats_in', c_ptr), ('ln_u', c_ptr), ('ln_v', c_ptr), ('ln_eps', ctypes.c_float),
                ('ln_stats_out', c_ptr)]


class BlockWeights(ctypes.Structure):
    _fields_ = [(n, c_ptr) for n in ('qkv_w', 'qkv_b', 'proj_w', 'proj_b', 'fc1_w', 'fc1_b', 'fc2_w', 'fc2_b',
                                     'shift1', 'one_plus_scale1', 'gate1', 'shift2', 'one_plus_scale2', 'gate2',
                                     'qkv_u', 'qkv_v', 'fc1_u', 'fc1_v')]


class CrossWeights(ctypes.Structure):
    _fields_ = [(n, c_ptr) for n in ('query_w', 'query_b', 'proj_w', 'proj_b', 'zero_w', 'zero_b', 'k', 'v',
                                     'query_u', 'query_v')]


class EngineConfig(ctypes.Structure):
    _fields_ = [(n, c_int) for n in ('slots', 'height', 'depth', 'width', 'patch', 'classes', 'd', 'heads', 'mlp',
                                     'depth_layers', 'key_capacity', 'n_control')] + \
               [('layer_index', ctypes.POINTER(ctypes.c_int32))]


class EngineWeights(ctypes.Structure):
    _fields_ = [(n, c_ptr) for n in ('table_b', 'bias_b', 'yadd_b', 'table_c', 'bias_c', 'yadd_c')] + \
               [('backbone', ctypes.POINTER(BlockWeights)), ('control', ctypes.POINTER(BlockWeights)),
                ('cross', ctypes.POINTER(CrossWeights))] + \
               [(n, c_ptr) for n in ('final_shift', 'final_one_plus_scale', 'head_w', 'head_b', 'rope_sin', 'rope_cos',
                                     'cross_sin', 'cross_cos', 'lengths', 'head_u', 'head_v')]


class EvalParams(ctypes.Structure):
    _fields_ = [('mode', ctypes.c_int32), ('k', ctypes.c_int32), ('candidates', ctypes.c_int32),
                ('committed', ctypes.c_int32), ('threshold', ctypes.c_float), ('step', ctypes.c_int32)]


class AttentionProblem(ctypes.Structure):
    _fields_ = [('q', c_ptr), ('k', c_ptr), ('v', c_ptr), ('q_row_stride', c_i64), ('kv_slot_stride', c_i64),
                ('kv_head_stride', c_i64), ('kv_row_stride', c_i64), ('lengths', c_ptr), ('keys', c_int),
                ('out', c_ptr)]


class EngineWorkspace(ctypes.Structure):
    _fields_ = [(n, c_ptr) for n in ('xb', 'xc', 'h', 'qkv', 'attn', 'mlp', 'qx', 'ax', 'stats_b', 'stats_c')]


_SIGNATURES = {
    'svx_last_error': (ctypes.c_char_p, []),
    'svx_version': (c_int, []),
    'svx_device_supported': (c_int, []),
    'svx_wait_timeouts': (ctypes.c_uint32, []),
    'svx_ease_scores': (c_int, [c_ptr, c_int, c_int, c_int, c_int, c_i64, c_ptr, c_ptr, c_ptr]),
    'svx_ease_mark': (c_int, [c_ptr, c_int, c_int, c_int, c_int, c_int, c_int, c_i64, c_ptr, c_int, ctypes.c_double,
                              c_ptr, c_ptr, c_ptr]),
    'svx_ease_select_workspace_bytes': (ctypes.c_size_t, [c_int, c_int]),
    'svx_ease_select': (c_int, [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_int, c_int, c_int, c_int, c_int, c_int, c_ptr,
                                c_ptr, c_int, c_ptr, c_ptr, c_ptr, c_ptr]),
    'svx_ease_select_noalloc': (c_int, [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_int, c_int, c_int, c_int, c_int, c_int,
                                        c_ptr, c_ptr, c_int, c_ptr, c_ptr, c_ptr]),
    'svx_ease_sample': (c_int, [c_ptr, c_int, c_int, c_int, c_int, c_i64, c_ptr, c_ptr, c_ptr, c_i64, c_int, c_ptr,
                                c_ptr, c_ptr, c_ptr]),
    'svx_softmax_rows': (c_int, [c_ptr, c_int, c_int, c_ptr, c_ptr]),
    'svx_eval_select': (c_int, [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_int, c_int, c_int, c_int, c_int, c_ptr, c_ptr,
                                c_int, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    'svx_ease_finish': (c_int, [c_ptr, c_ptr, c_ptr, c_int, c_int, c_int, c_ptr]),
    'svx_patch_embed': (c_int, [c_ptr, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_ptr, c_ptr, c_ptr, c_ptr,
                                c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    'svx_layernorm_modulate': (c_int, [c_ptr, c_int, c_int, ctypes.c_float, c_ptr, c_ptr, c_ptr, c_ptr]),
    'svx_layernorm_affine': (c_int, [c_ptr, c_int, c_int, ctypes.c_float, c_ptr, c_ptr, c_ptr, c_int, c_ptr, c_ptr]),
    'svx_gemm': (c_int, [c_ptr, c_ptr, c_ptr, c_int, c_int, c_int, ctypes.POINTER(EpilogueArgs), c_ptr]),
    'svx_gemm_group': (c_int, [c_ptr, c_ptr, c_ptr, ctypes.POINTER(EpilogueArgs), c_ptr, c_ptr, c_ptr,
                               ctypes.POINTER(EpilogueArgs), c_int, c_int, c_int, c_ptr]),
    'svx_attention': (c_int, [c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_i64, c_i64, c_ptr, c_int, c_int, c_int, c_int,
                              c_ptr, c_ptr, c_int, c_ptr]),
    'svx_attention_plan_ints': (c_int, [c_int, c_int, c_int, c_int]),
    'svx_attention_plan': (c_int, [c_ptr, c_int, c_int, c_int, c_int, c_int, c_ptr, c_int]),
    'svx_attention_multi': (c_int, [ctypes.POINTER(AttentionProblem), c_int, c_int, c_int, c_int, c_ptr, c_int,
                                    c_ptr]),
    'svx_attention_multi_plan_ints': (c_int, [c_int, c_int, c_int, c_int, c_int]),
    'svx_attention_multi_plan': (c_int, [ctypes.POINTER(c_ptr), ctypes.POINTER(c_int), c_int, c_int, c_int, c_int,
                                         c_int, c_ptr, c_int]),
    'svx_engine_create': (c_int, [ctypes.POINTER(EngineConfig), ctypes.POINTER(EngineWeights),
                                  ctypes.POINTER(EngineWorkspace), ctypes.POINTER(c_ptr)]),
    'svx_engine_forward': (c_int, [c_ptr, c_int, c_ptr, c_ptr, c_ptr]),
    'svx_engine_set_lengths': (c_int, [c_ptr, c_ptr, c_ptr]),
    'svx_engine_launches': (c_int, [c_ptr, c_int]),
    'svx_engine_destroy': (None, [c_ptr]),
}

_LIB = None


def header_symbols():
    """Every function the C header declares (`SVX_API <type> svx_name(`)."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r'SVX_API\s+[\w\s\*]+?\b(svx_\w+)\s*\(', text)))


def load():
    """Load libsvx.so (built in-tree by `python -m streamvoxel_b200.build`). Raises if it is missing."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIBRARY):
            raise RuntimeError(f'{LIBRARY} is missing: run `python -m streamvoxel_b200.build` (nvcc, sm_100a)')
        lib = ctypes.CDLL(LIBRARY)
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _LIB = lib
    return _LIB


def check(status, what=''):
    if status == SVX_OK:
        return
    text = load().svx_last_error().decode(errors='replace')
    if status == SVX_ERR_INVALID:
        raise ValueError(f'{what}: {text}' if what else text)
    raise RuntimeError(f'{what}: {text}' if what else text)


def require_device(device=None):
    """Raise unless the current CUDA device is an sm_100 part the kernels were built for."""
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError('streamvoxel_b200 needs a CUDA device (B200, sm_100a); no CPU fallback exists')
    if device is not None:
        device = torch.device(device)
        if device.type != 'cuda':
            raise RuntimeError(f'streamvoxel_b200 runs on CUDA devices only, got {device}')
        if device.index is not None:
            torch.cuda.set_device(device)
    if not load().svx_device_supported():
        raise RuntimeError('streamvoxel_b200 kernels are built for sm_100a (B200) only')


def ptr(tensor):
    """Raw device pointer of a contiguous tensor (None -> NULL). Non-contiguous views would be read with the wrong
    strides by the kernels, so they are rejected."""
    if tensor is None:
        return ctypes.c_void_p(0)
    if not tensor.is_contiguous():
        raise ValueError('libsvx operands must be contiguous tensors')
    return ctypes.c_void_p(tensor.data_ptr())


def raw_ptr(tensor):
    """Device pointer of a strided view whose strides the callee takes as explicit arguments."""
    return ctypes.c_void_p(0 if tensor is None else tensor.data_ptr())


def stream_ptr(stream=None):
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return ctypes.c_void_p(s.cuda_stream)
