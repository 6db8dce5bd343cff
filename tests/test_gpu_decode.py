"""The config-1 driver (one column decoded from all-MASK by the time-free model on our engine and the shipped sampler)
and the evaluation decoders on the same kernels."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_decode_low_entropy_last_completes_and_is_deterministic():
    from streamvoxel_b200 import model as sm
    from streamvoxel_b200.decode import UnconditionalForward, decode_low_entropy_last
    from streamvoxel_b200.sampling import low_entropy_last_quotas
    cfg = sm.small_test_config(layer_indices=())
    forward = UnconditionalForward(cfg, sm.synthetic_state_dict(cfg, seed=1, std=0.05))
    spec = dict(air_ids=(0,), air_token=0, last_eps=1e-4, block_size=4, steps=16)
    runs = [decode_low_entropy_last(forward, spec, 7, 'cuda', cfg.voxel_shape, cfg.classes) for _ in range(2)]
    (result, info), (again, _) = runs
    assert info['complete'] and info['nfe'] == 1 + len(low_entropy_last_quotas(
        int(np.prod(cfg.voxel_shape)), 16, info['last_count'], 'quartercos'))
    tokens, steps = result['compact'], result['commit_step']
    assert tokens.min() >= 0 and tokens.max() < cfg.classes          # every voxel decoded, no mask id left
    assert steps.min() >= 1 and steps.max() == info['nfe']            # every voxel has a commit step
    assert np.array_equal(tokens, again['compact']) and np.array_equal(steps, again['commit_step'])


def test_decode_low_entropy_last_equals_reference_slot():
    """Config-1 parity: `decode_low_entropy_last` (`streamvoxel/eval/samplers.py:118-134`) on the small time-free model
    equals the reference slot driven over the same forwards (each step's logits from our engine, the block order and
    the multinomial draws from CUDA generators on the same seeds, the selection given the kernel's scores): tokens,
    commit steps, nfe and last_count."""
    from reference_slot import ReferenceSlot
    from streamvoxel_b200 import model as sm, ops
    from streamvoxel_b200.decode import UnconditionalForward, decode_low_entropy_last
    cfg = sm.small_test_config(layer_indices=())
    forward = UnconditionalForward(cfg, sm.synthetic_state_dict(cfg, seed=4, std=0.05))
    shape, classes, seed = cfg.voxel_shape, cfg.classes, 21
    spec = dict(air_ids=(0,), air_token=0, last_eps=1e-4, block_size=4, steps=12)
    recorded = []

    def recording(tokens, t):
        out = forward(tokens, t)
        recorded.append(out[0].clone())
        return out

    result, info = decode_low_entropy_last(recording, spec, seed, 'cuda', shape, classes)
    blocks = int(np.prod(shape)) // 64
    order = torch.randperm(blocks, device='cuda', generator=torch.Generator(device='cuda').manual_seed(seed + 9173))
    ref = ReferenceSlot(shape, classes, last_eps=spec['last_eps'])
    ref.arm(seed, spec['steps'], (), order.cpu().numpy())
    tokens = np.full(shape, classes, np.int64)
    record = None
    for logits in recorded:
        assert record is None
        scores = ops.ease_scores(logits[None].contiguous())[0].cpu().numpy()
        record, _ = ref.consume(logits, tokens, scores)
    assert record is not None and info['nfe'] == record['nfe'] == len(recorded)
    assert info['last_count'] == record['last_count']
    assert np.array_equal(result['compact'], tokens)
    assert np.array_equal(result['commit_step'], record['step_map'])


@pytest.mark.slow
def test_decode_low_entropy_last_full_size():
    """BASELINE config 1 at full size: the time-free DiT-B/4 (d = 768, 8 x 96 heads, 12 layers, V = 256) decodes one
    all-MASK column, cap 32, seed 0, on one B200; reports NFE and wall time."""
    from streamvoxel_b200 import model as sm
    from streamvoxel_b200.decode import UnconditionalForward, decode_low_entropy_last
    from streamvoxel_b200.sampling import low_entropy_last_quotas
    cfg = sm.dit_b4_unconditional()
    forward = UnconditionalForward(cfg, sm.synthetic_state_dict(cfg, seed=0))
    spec = dict(air_ids=(0,), air_token=0, last_eps=1e-4, block_size=4, steps=32)
    decode_low_entropy_last(forward, spec, 1, 'cuda', cfg.voxel_shape, cfg.classes)   # warm-up
    result, info = decode_low_entropy_last(forward, spec, 0, 'cuda', cfg.voxel_shape, cfg.classes)
    print(f"config 1: nfe {info['nfe']}, last_count {info['last_count']}, {info['seconds'] * 1e3:.1f} ms per column")
    assert info['nfe'] == 1 + len(low_entropy_last_quotas(65536, 32, info['last_count'], 'quartercos'))
    assert result['compact'].max() < cfg.classes and result['commit_step'].min() >= 1


def _eval_fixture_module():
    import importlib.util
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden', 'make_golden.py')
    spec = importlib.util.spec_from_file_location('make_golden', path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_eval_decoders_match_oracle_given_the_same_draws():
    """`decode` (random, entropy, mixed, block, native_quarter; every schedule family) on libsvx equals the oracle
    decoder, pinned to the reference by `tests/test_oracle_golden.py`, fed the same CUDA generator stream (draws,
    multinomial noise, block order) and the kernel's entropy scores: tokens, commit steps and per-step events."""
    from oracle import eval_samplers as oes
    from streamvoxel_b200 import _lib, ops
    from streamvoxel_b200.decode import decode
    _lib.require_device()
    mg = _eval_fixture_module()
    shape, classes = (16, 8, 8), 6

    def forward(tokens, t):
        return mg.eval_logits(tokens[0].cpu(), classes)[None].cuda()

    for i, spec in enumerate(mg.EVAL_SPECS):
        seed = 100 + 17 * i
        result, meta = decode(forward, dict(spec), seed, 'cuda', shape=shape, classes=classes, trace=True)
        g = torch.Generator(device='cuda').manual_seed(seed)
        draw = lambda: torch.rand(shape, device='cuda', generator=g).cpu().numpy()
        noise = lambda k, c: torch.empty((1, k, c), device='cuda').exponential_(generator=g)[0].cpu().numpy()
        order = None
        if spec['selection'] == 'block':
            bg = torch.Generator(device='cuda').manual_seed(seed + 9173)
            order = torch.randperm(16, device='cuda', generator=bg).cpu().numpy()
        score_fn = lambda logits: ops.ease_scores(torch.from_numpy(logits)[None].cuda())[0].cpu().numpy()
        tokens, commit, events = oes.decode(lambda tok, t: mg.eval_logits(torch.from_numpy(tok), classes).numpy(),
                                            dict(spec), draw, noise, order=order, shape=shape, classes=classes,
                                            score_fn=score_fn)
        assert np.array_equal(result['compact'], tokens), spec
        assert np.array_equal(result['commit_step'], commit), spec
        assert meta['events'] == events, spec
        assert meta['complete'] == (meta['remaining'] == 0)
