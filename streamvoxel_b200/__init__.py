"""StreamVoxel's per-step column-generation hot path on B200 (sm_100a).

Python surface mirroring the reference (zzf1955/StreamVoxel): `stream.fast_ops` (FastSlotForward,
FastLowEntropyLastSlot, SelectGraphs, consume_batch), `sampling` (quota schedule), `model` (weights + forward).
Every hot-path operation runs in libsvx.so (include/svx.h); there is no CPU fallback.
"""
__version__ = '0.1.0'
