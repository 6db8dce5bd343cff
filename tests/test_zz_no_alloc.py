"""svx_ease_select_noalloc, the selection entry point for hosts that cannot allocate device memory, against
svx_ease_select given a workspace the caller allocated.

Who needs it: a host that leaves every byte of device memory to another framework's allocator, or that must not
allocate while it runs, has no workspace to pass; the no-allocation entry point keeps its scratch in a fixed array
inside the library. This file is collected last so a run that stops at the first failure has run every other test.
Both calls go through the C ABI with ctypes. Selection is index work, so the outputs must be equal (the tolerance of
the other selection tests); calls in a row with different inputs, slot counts and column sizes show that the shared
scratch left by one call does not leak into the next.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(seed, slots, shape=(256, 16, 16)):
    rng = np.random.default_rng(seed)
    total, blocks = int(np.prod(shape)), int(np.prod(shape)) // 64
    scores, tokens, lasts, poss, rows = [], [], [], [], []
    for s in range(slots):
        tops = rng.integers(shape[0] // 4, shape[0], shape[1:])
        last = np.arange(shape[0])[:, None, None] >= tops[None]
        committed_mask = ~last & (rng.random(shape) < rng.random())
        selectable = ~last & ~committed_mask
        k = int(rng.integers(1, max(2, int(selectable.sum()))))
        committed = int(committed_mask.sum())
        frac = (committed + k) / int((~last).sum())
        score = rng.standard_normal(shape).astype(np.float32)
        if s % 2:
            score = np.round(score * 2) / 2
        pos = np.empty(blocks, np.int64)
        pos[rng.permutation(blocks)] = np.arange(blocks)
        scores.append(score)
        tokens.append(np.where(selectable | last, 256, 0).astype(np.int16))
        lasts.append(last.astype(np.uint8))
        poss.append(pos.astype(np.int32))
        rows.append((k, 1, committed, frac, seed))
    dev = lambda a: torch.from_numpy(np.stack(a)).cuda().contiguous()
    return dict(scores=dev(scores), tokens=dev(tokens), last=dev(lasts), pos=dev(poss), rows=rows, slots=slots,
                shape=shape, total=total)


def _outputs(case):
    s, total = case['slots'], case['total']
    return dict(chosen=torch.zeros((s, *case['shape']), dtype=torch.uint8, device='cuda'),
                index=torch.zeros((s, total), dtype=torch.int32, device='cuda'),
                count=torch.zeros(s, dtype=torch.int32, device='cuda'),
                status=torch.zeros(s, dtype=torch.int32, device='cuda'))


def _call(lib, case, out, workspace=None):
    from streamvoxel_b200 import ops
    params = ops.step_params(case['rows'], 'cuda')
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    y, z, x = case['shape']
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = (p(case['scores']), p(case['tokens']), p(case['last']), p(case['pos']), p(params), case['slots'], y, z, x,
              4, 256, p(out['chosen']), p(out['index']), case['total'], p(out['count']), p(out['status']))
    if workspace is None:
        status = lib.svx_ease_select_noalloc(*common, stream)
    else:
        status = lib.svx_ease_select(*common, p(workspace), stream)
    torch.cuda.synchronize()
    return status


def test_no_alloc_selection_equals_workspace_selection_in_a_row():
    from streamvoxel_b200 import _lib, ops
    _lib.require_device()
    lib = _lib.load()
    # Calls in a row on the shared scratch: other inputs and fewer slots; then a smaller column (256 blocks, so the
    # per-slot counters sit where the first calls left block quotas); then the largest call the scratch takes (64 slots
    # of 1024 blocks).
    for seed, slots, shape in ((11, 8, (256, 16, 16)), (12, 5, (256, 16, 16)), (13, 6, (64, 16, 16)),
                               (14, 64, (256, 16, 16))):
        case = _case(seed, slots, shape)
        want = _outputs(case)
        workspace = ops.select_workspace(slots, case['total'], 'cuda')
        assert _call(lib, case, want, workspace) == _lib.SVX_OK
        got = _outputs(case)
        assert _call(lib, case, got) == _lib.SVX_OK, lib.svx_last_error()
        for name in ('chosen', 'index', 'count', 'status'):
            assert torch.equal(got[name], want[name]), (seed, name)
        assert [int(c) for c in got['count']] == [r[0] for r in case['rows']]


def test_no_alloc_selection_rejects_sizes_beyond_its_scratch():
    from streamvoxel_b200 import _lib
    _lib.require_device()
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    status = lib.svx_ease_select_noalloc(null, null, null, null, null, 65, 256, 16, 16, 4, 256, null, null, 1, null,
                                         null, null)
    assert status == _lib.SVX_ERR_INVALID and b'64 slots' in lib.svx_last_error()
    status = lib.svx_ease_select_noalloc(null, null, null, null, null, 1, 512, 16, 16, 4, 256, null, null, 1, null,
                                         null, null)
    assert status == _lib.SVX_ERR_INVALID and b'1024' in lib.svx_last_error()
    # 2^42 blocks: a 32-bit product would wrap to 0 and pass; the count is formed in 64 bits and rejected
    status = lib.svx_ease_select_noalloc(null, null, null, null, null, 1, 1 << 20, 1 << 20, 1 << 8, 4, 256, null, null,
                                         1, null, null, null)
    assert status == _lib.SVX_ERR_INVALID and b'1024' in lib.svx_last_error()
