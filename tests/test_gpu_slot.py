"""The drop-in sampler surface on the GPU against the reference's windows: `FastLowEntropyLastSlot` through
`consume_batch` + `SelectGraphs` (`streamvoxel/stream/fast_ops.py:481-642`) and the whole-step graph `SlotBatch`
in both draws, each compared commit for commit with the reference slot (`streamvoxel/stream/slot.py:117-176`).

Bar (the reference's own, `tests/stream/test_live_fast_ops.py:95`): commits (positions and values) of every step,
tokens, `step_map`, `values`, `nfe`, `actual` and `last_count` bit-equal.
"""
import os

import numpy as np
import pytest
import torch

from oracle import sampler as osm

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')


def _fixture_module():
    import importlib.util
    path = os.path.join(GOLDEN, 'make_golden.py')
    spec = importlib.util.spec_from_file_location('make_golden', path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


class _Outputs:
    """The part of an engine `SelectGraphs` reads: static outputs per bucket, token rows, the device."""

    def __init__(self, logits, tokens):
        self.device = logits.device
        self.outputs = {len(logits): logits}
        self.graphs = {len(logits): None}
        self.tokens = tokens


def _record_equal(got, want):
    for key in ('nfe', 'actual', 'last_count'):
        assert got[key] == want[key], key
    assert np.array_equal(np.asarray(got['step_map']), np.asarray(want['step_map']))
    assert np.array_equal(np.asarray(got['values']), np.asarray(want['values']))


@pytest.mark.parametrize('batched', [False, True])
def test_fast_slot_windows_equal_reference_fixtures(batched):
    """The reference's three recorded windows (seeds 3, 11, 12345; V = 6; `test_live_fast_ops.py:70-91`), replayed
    with the reference's block order and multinomial noise, through `consume_batch` + `SelectGraphs` (batched) or
    per-slot `consume`: every commit, the tokens and the window records equal the reference's."""
    from streamvoxel_b200.stream.fast_ops import FastLowEntropyLastSlot, SelectGraphs, consume_batch
    mg = _fixture_module()
    g = np.load(os.path.join(GOLDEN, 'slot_windows.npz'))
    shape, classes, n = (16, 8, 8), 6, int(g['count'])
    logits = torch.zeros((n, classes, *shape), dtype=torch.float32, device='cuda')
    tokens = torch.full((n, *shape), classes, dtype=torch.int16, device='cuda')
    slots = [FastLowEntropyLastSlot(shape, classes, air_ids=(0,), air_token=0, last_eps=1e-3, block_size=4,
                                    device='cuda', sampling='parity') for _ in range(n)]
    graphs = SelectGraphs(_Outputs(logits, tokens), slots) if batched else None
    steps = [0] * n
    for i, slot in enumerate(slots):
        seed, cap, _ = (int(v) for v in g[f'w{i}_args'])
        slot.arm(seed, cap, (i, 0), order=g[f'w{i}_order'])
        slot.noise_source = (lambda k, c, i=i: torch.from_numpy(g[f'w{i}_s{steps[i]}_noise']).cuda())
    records = {}
    while len(records) < n:
        for i in range(n):
            ground = int(g[f'w{i}_args'][2])
            logits[i].copy_(mg._fixture_logits(steps[i] + 31 * i, ground))
        if batched:
            results = consume_batch(slots, logits, tokens, n, graphs)
        else:
            results = {i: slots[i].consume(logits[i], tokens[i]) for i in range(n) if not slots[i].idle}
        for i, (record, commit) in results.items():
            if commit is not None:
                assert np.array_equal(commit['positions'], g[f'w{i}_s{steps[i]}_positions']), (i, steps[i])
                assert np.array_equal(commit['values'], g[f'w{i}_s{steps[i]}_values']), (i, steps[i])
                assert commit['step'] == slots[i].nfe
            if record is not None:
                records[i] = record
            steps[i] += 1
        assert max(steps) < 64
    for i in range(n):
        assert steps[i] == int(g[f'w{i}_steps'])
        assert np.array_equal(tokens[i].cpu().numpy(), g[f'w{i}_tokens'])
        nfe, actual, last_count = (int(v) for v in g[f'w{i}_record'])
        _record_equal(records[i], dict(nfe=nfe, actual=actual, last_count=last_count,
                                       step_map=g[f'w{i}_step_map'], values=g[f'w{i}_values']))


def _config3_logits(generator, slots, boost_index, classes=256, voxels=65536):
    """N(0, 2) per logit (sigma = sqrt 2), +6 on the ground-truth id of a seeded 70% of voxels
    (`boost_index`: flat indexes into [slots, classes, voxels]); fp32 class-major [slots, classes, Y, Z, X]."""
    logits = torch.randn((slots, classes, voxels), generator=generator, device='cuda') * (2 ** 0.5)
    logits.view(-1)[boost_index] += 6.0
    return logits.view(slots, classes, 256, 16, 16)


def _boost_index(slots, classes=256, voxels=65536, fraction=0.7, seed=5):
    from streamvoxel_b200 import synth
    from streamvoxel_b200.stream.condition import ModelSpec
    spec = ModelSpec(height=256, tile=16, num_classes=classes, biome_classes=16, biome_halo=4, y_origin=-64.)
    rng = np.random.default_rng(seed)
    index = []
    for s in range(slots):
        _, truth = synth.target_tokens(seed * 100 + s, spec)
        pick = np.flatnonzero(rng.random(voxels) < fraction)
        index.append((s * classes + truth.reshape(-1)[pick].astype(np.int64)) * voxels + pick)
    return torch.from_numpy(np.concatenate(index)).cuda()


def test_fast_slot_full_size_config3_windows_equal_reference_slot():
    """BASELINE config 3 at full size: 8 slots of [256, 16, 16] x V = 256 fp32 logits (N(0, 2), +6 on the ground-truth
    id of 70% of voxels, fresh logits every forward), whole cap-32 windows through `consume_batch` + `SelectGraphs`
    on the slots' own CUDA generators, against the reference slot on the same logits, generator seeds and block
    orders (its draws are the reference's `torch.multinomial` calls, its selection the oracle's on the kernel's
    scores). Also pins the kernel's scores to `entropy_scores` within 1e-5 on the first solid step."""
    from streamvoxel_b200.stream.fast_ops import FastLowEntropyLastSlot, SelectGraphs, consume_batch
    from reference_slot import ReferenceSlot
    slots_n, classes, shape = 8, 256, (256, 16, 16)
    logits = torch.zeros((slots_n, classes, *shape), dtype=torch.float32, device='cuda')
    tokens = torch.full((slots_n, *shape), classes, dtype=torch.int16, device='cuda')
    slots = [FastLowEntropyLastSlot(shape, classes, air_ids=(0,), air_token=0, last_eps=1e-4, block_size=4,
                                    device='cuda', sampling='parity') for _ in range(slots_n)]
    graphs = SelectGraphs(_Outputs(logits, tokens), slots)
    refs = [ReferenceSlot(shape, classes, last_eps=1e-4) for _ in range(slots_n)]
    ref_tokens = [np.full(shape, classes, np.int64) for _ in range(slots_n)]
    for i in range(slots_n):
        slots[i].arm(1000 + i, 32, (i, 0))
        refs[i].arm(1000 + i, 32, (i, 0), slots[i].order.cpu().numpy())
    boost = _boost_index(slots_n)
    generator = torch.Generator(device='cuda').manual_seed(77)
    records, step, checked = {}, 0, False
    while len(records) < slots_n:
        logits.copy_(_config3_logits(generator, slots_n, boost))
        results = consume_batch(slots, logits, tokens, slots_n, graphs)
        for i, (record, commit) in results.items():
            scores = slots[i].scores[0].cpu().numpy()
            if commit is not None and not checked:
                want = osm.entropy_scores(logits[i].cpu().numpy())
                np.testing.assert_allclose(scores, want, atol=1e-5, rtol=0)
                checked = True
            ref_record, ref_commit = refs[i].consume(logits[i], ref_tokens[i], scores)
            assert (commit is None) == (ref_commit is None), (i, step)
            if commit is not None:
                assert np.array_equal(commit['positions'], ref_commit['positions']), (i, step)
                assert np.array_equal(commit['values'], ref_commit['values']), (i, step)
                assert commit['step'] == ref_commit['step']
            assert (record is None) == (ref_record is None), (i, step)
            if record is not None:
                _record_equal(record, ref_record)
                records[i] = record
        step += 1
        assert step <= 40
    for i in range(slots_n):
        assert np.array_equal(tokens[i].cpu().numpy(), ref_tokens[i])


def _edge_air_boost(shape, seed=9):
    """Per-slot masks of voxels whose air logit is raised far above the rest (p(air) > 1 - 1e-6), chosen so the
    marking defers: every voxel (no solid step, the window ends at its marking); the upper half of every column;
    all but 8 voxels (one solid step of 8, most 4^3 blocks with no legal voxel); nothing, although a third of the voxels
    are air-certain (each column's top voxel is not, and the deferred run must reach the top)."""
    y, z, x = shape
    rng = np.random.default_rng(seed)
    everything = np.ones(shape, bool)
    upper = np.zeros(shape, bool)
    upper[y // 2:] = True
    but_eight = np.ones(shape, bool)
    but_eight[:5, 0, 0] = False
    but_eight[:3, 3, 4] = False
    scattered = rng.random(shape) < 0.35
    scattered[-1] = False
    return [everything, upper, but_eight, scattered]


def test_fast_slot_edge_windows_equal_reference_slot():
    """Windows whose marking defers all, half, all but 8, or none of the voxels (fresh N(0, 1) logits every forward
    plus the air boost of `_edge_air_boost`), through `consume_batch` + `SelectGraphs` on the slots' own generators,
    against the reference slot on the same logits, seeds and block orders: every commit, the tokens and the records
    bit-equal, including the window that ends at its marking and the steps whose quota lies in a few blocks."""
    from streamvoxel_b200.stream.fast_ops import FastLowEntropyLastSlot, SelectGraphs, consume_batch
    from reference_slot import ReferenceSlot
    shape, classes, cap = (32, 8, 8), 6, 8
    boosts = [torch.from_numpy(b).cuda() for b in _edge_air_boost(shape)]
    slots_n = len(boosts)
    logits = torch.zeros((slots_n, classes, *shape), dtype=torch.float32, device='cuda')
    tokens = torch.full((slots_n, *shape), classes, dtype=torch.int16, device='cuda')
    slots = [FastLowEntropyLastSlot(shape, classes, air_ids=(0,), air_token=0, last_eps=1e-4, block_size=4,
                                    device='cuda', sampling='parity') for _ in range(slots_n)]
    graphs = SelectGraphs(_Outputs(logits, tokens), slots)
    refs = [ReferenceSlot(shape, classes, last_eps=1e-4) for _ in range(slots_n)]
    ref_tokens = [np.full(shape, classes, np.int64) for _ in range(slots_n)]
    for i in range(slots_n):
        slots[i].arm(2000 + i, cap, (i, 0))
        refs[i].arm(2000 + i, cap, (i, 0), slots[i].order.cpu().numpy())
    generator = torch.Generator(device='cuda').manual_seed(13)
    records, step = {}, 0
    while len(records) < slots_n:
        logits.copy_(torch.randn(logits.shape, generator=generator, device='cuda'))
        for i in range(slots_n):
            logits[i, 0].masked_fill_(boosts[i], 20.0)
        results = consume_batch(slots, logits, tokens, slots_n, graphs)
        for i, (record, commit) in results.items():
            scores = slots[i].scores[0].cpu().numpy()
            ref_record, ref_commit = refs[i].consume(logits[i], ref_tokens[i], scores)
            assert (commit is None) == (ref_commit is None), (i, step)
            if commit is not None:
                assert np.array_equal(commit['positions'], ref_commit['positions']), (i, step)
                assert np.array_equal(commit['values'], ref_commit['values']), (i, step)
                assert commit['step'] == ref_commit['step']
            assert (record is None) == (ref_record is None), (i, step)
            if record is not None:
                _record_equal(record, ref_record)
                records[i] = record
        step += 1
        assert step <= cap + 2
    total = int(np.prod(shape))
    assert [records[i]['last_count'] for i in range(slots_n)][:3] == [total, total // 2, total - 8]
    assert records[0]['nfe'] == 1 and records[0]['actual'] == 0 and records[2]['actual'] == 1
    assert records[3]['last_count'] == 0 and records[3]['actual'] == cap
    for i in range(slots_n):
        assert np.array_equal(tokens[i].cpu().numpy(), ref_tokens[i])


def _small_batch(sampling, slots=4):
    from streamvoxel_b200 import model as sm, synth
    from streamvoxel_b200.stream.batch import SlotBatch
    from streamvoxel_b200.stream.condition import ModelSpec
    from streamvoxel_b200.stream.fast_ops import FastSlotForward
    cfg = sm.small_test_config()
    sd = sm.synthetic_state_dict(cfg, seed=2, std=0.05)
    spec = ModelSpec.of(cfg)
    forward = FastSlotForward((cfg, sd), spec, 'cuda', slots, 3, 8)
    for i in range(slots):
        forward.load_slot(i, synth.item(40 + i, spec, k=i % 4, far=8))
    forward.wait_loads()
    return cfg, SlotBatch(forward, sampling=sampling, last_eps=1e-4, min_cap=8)


@pytest.mark.parametrize('sampling', ['parity', 'native'])
def test_slot_batch_windows_equal_reference_slot(sampling):
    """The whole-step graph (forward + entropy + selection + draw + commit in one replay) for two windows per slot
    in a row, against the reference slot fed each step's logits: parity mode equals the reference's multinomial draws
    on the same generator seeds; native mode equals the oracle's restatement of the Gumbel-max Philox draw bit for
    bit (both given the kernel's fp32 scores)."""
    from reference_slot import ReferenceSlot
    cfg, batch = _small_batch(sampling)
    n, shape, classes = batch.slots, batch.shape, batch.classes
    caps = [8, 9, 10, 12]
    refs = [ReferenceSlot(shape, classes, last_eps=1e-4) for _ in range(n)]
    natives = [osm.Slot(shape, classes, (0,), 0, 1e-4, 4) for _ in range(n)]
    ref_tokens = [np.full(shape, classes, np.int64) for _ in range(n)]
    windows = [0] * n

    def arm(i):
        seed = 500 + 10 * i + windows[i]
        order = np.random.default_rng(seed).permutation(batch.blocks)
        batch.arm(i, seed, caps[i], order=order)
        refs[i].arm(seed, caps[i], (), order)
        natives[i].arm(seed, caps[i], (), order)
        ref_tokens[i][...] = classes

    for i in range(n):
        arm(i)
    finished, step = 0, 0
    while finished < 2 * n:
        results = batch.step()
        logits = batch.forward.logits
        for i, (record, commit) in results.items():
            scores = batch.scores[i].cpu().numpy()
            if sampling == 'parity':
                want_record, want_commit = refs[i].consume(logits[i], ref_tokens[i], scores)
            else:
                air = logits[i].float().softmax(0)[[0]].sum(0).cpu().numpy()
                host_logits = logits[i].float().cpu().numpy()
                want_record, want_commit = natives[i].consume(host_logits, ref_tokens[i], native=True, scores=scores,
                                                              air=air)
            assert (commit is None) == (want_commit is None), (i, step)
            if commit is not None:
                assert np.array_equal(commit['positions'], want_commit['positions']), (i, step)
                assert np.array_equal(commit['values'], want_commit['values']), (i, step)
                assert commit['step'] == want_commit['step']
            assert (record is None) == (want_record is None), (i, step)
            if record is not None:
                for key in ('nfe', 'actual', 'last_count'):
                    assert record[key] == want_record[key], key
                assert np.array_equal(batch.column(i), ref_tokens[i]), i
                assert np.array_equal(record['column'], ref_tokens[i]), i   # staged by the finishing step
                finished += 1
                windows[i] += 1
                if windows[i] < 2:
                    arm(i)
        step += 1
        assert step < 64


@pytest.mark.parametrize('sampling', ['parity', 'native'])
def test_slot_batch_two_steps_in_flight_equal_one(sampling):
    """`SlotBatch` driven with two steps in flight (`launch` twice, then `collect` the oldest, re-arming finished
    slots while a step runs) commits exactly what the one-step `step()` driver commits, window for window: a slot
    sits out the steps it cannot take (marked but not yet collected, or finished), which changes no window's forwards."""
    def run(two):
        cfg, batch = _small_batch(sampling)
        for i in range(batch.slots):
            batch.arm(i, 900 + 100 * i, 8 + i, order=np.random.default_rng(i).permutation(batch.blocks))
        commits, windows, rearmed = {}, 0, set()
        while windows < 2 * batch.slots:
            if two:
                while batch.in_flight < batch.depth and batch.runnable():
                    batch.launch()
                results = batch.collect()
            else:
                results = batch.step()
            for i, (record, commit) in results.items():
                key = (i, batch.state[i].get('seed'))
                if commit is not None:
                    commits.setdefault(key, []).append((commit['step'], commit['positions'].tolist(),
                                                        commit['values'].tolist()))
                if record is not None:
                    assert np.array_equal(record['column'], batch.column(i))
                    commits.setdefault((i, record['seed']), []).append(('done', record['column'].tobytes()))
                    windows += 1
                    if i not in rearmed:   # a second window per slot, its seed a function of the slot only
                        rearmed.add(i)
                        batch.arm(i, 901 + 100 * i, 8 + i,
                                  order=np.random.default_rng(100 + i).permutation(batch.blocks))
        while batch.in_flight:
            batch.collect()
        return commits

    assert run(True) == run(False)
