"""Generate the golden fixtures under tests/golden/ by running the reference (zzf1955/StreamVoxel) itself.

Run in a container where the reference checkout exists (read-only is fine):

    python tests/golden/make_golden.py --reference <path to the StreamVoxel checkout>

It writes small .npz files (inputs, the reference's outputs, and the RNG draws the reference made) that the CPU
tests compare the oracle and the product's host logic against. Nothing here runs on the GPU box.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print(f'wrote {path} ({os.path.getsize(path)} bytes)')


# ---------------------------------------------------------------------------------------------- sampler

def quota_cases():
    """Inputs/outputs of `block_quota_select`, following the reference test generator
    (`tests/stream/test_live_fast_ops.py:32-49`) plus full-size columns."""
    from streamvoxel.sampling.block_quota import block_quota_select, block_view
    out = {}
    cases = [((16, 8, 8), s) for s in range(25)] + [((256, 16, 16), 100 + s) for s in range(6)]
    for index, (shape, seed) in enumerate(cases):
        b = 4
        g = torch.Generator().manual_seed(seed)
        last = torch.zeros(shape, dtype=torch.bool)
        tops = torch.randint(4, shape[0], shape[1:], generator=g)
        for z in range(shape[1]):
            for x in range(shape[2]):
                last[tops[z, x]:, z, x] = True
        non_last = ~last
        committed_mask = non_last & (torch.rand(shape, generator=g) < torch.rand((), generator=g))
        selectable = non_last & ~committed_mask
        k = int(torch.randint(1, max(2, int(selectable.sum())), (), generator=g))
        if index % 3 == 2:   # quota-sized steps as the live sampler takes them
            k = max(1, min(int(selectable.sum()), int(selectable.sum()) // 7))
        committed = int(committed_mask.sum())
        frac = (committed + k) / int(non_last.sum())
        blocks = int(np.prod(shape)) // b ** 3
        order = torch.randperm(blocks, generator=g)
        n_total = block_view(non_last.contiguous(), b).sum(1)
        score = (torch.randn(shape, generator=g) * 2).round() / 2
        if index % 2:
            score = torch.randn(shape, generator=g)
        chosen = block_quota_select(score, selectable, k, b, order, frac, n_total)
        pre = f'c{index}_'
        out.update({pre + 'score': score.numpy(), pre + 'selectable': selectable.numpy(), pre + 'k': np.int64(k),
                    pre + 'order': order.numpy(), pre + 'frac': np.float64(frac), pre + 'n_total': n_total.numpy(),
                    pre + 'committed': np.int64(committed), pre + 'chosen': chosen.numpy(),
                    pre + 'last': last.numpy()})
    out['count'] = np.int64(len(cases))
    _save('quota_select.npz', **out)


def top_mask_cases():
    from streamvoxel.sampling.block_quota import top_mask
    out = {}
    g = torch.Generator().manual_seed(1)
    for i, count in enumerate((0, 1, 7, 40, 500)):
        scores = torch.randint(-4, 1, (8, 8, 8), generator=g).float()
        eligible = torch.rand((8, 8, 8), generator=g) < .3
        out.update({f't{i}_scores': scores.numpy(), f't{i}_eligible': eligible.numpy(), f't{i}_count': np.int64(count),
                    f't{i}_mask': top_mask(scores, eligible, count).numpy()})
    out['count'] = np.int64(5)
    _save('top_mask.npz', **out)


def schedule_cases():
    from streamvoxel.sampling.low_entropy_last import low_entropy_last_quotas
    from streamvoxel.sampling.schedule import counts, actual_time
    rows = []
    for total, steps, n_last in [(65536, 32, 0), (65536, 32, 4096), (65536, 32, 30000), (65536, 32, 65536),
                                 (1024, 8, 0), (1024, 8, 300), (1024, 9, 1000), (65536, 16, 123), (65536, 64, 777)]:
        q = low_entropy_last_quotas(total, steps, n_last)
        rows.append((total, steps, n_last, q, counts(total, dict(steps=steps, schedule='quartercos', rounding='positive'))))
    flat = {}
    for i, (total, steps, n_last, q, c) in enumerate(rows):
        flat[f's{i}_args'] = np.asarray([total, steps, n_last], np.int64)
        flat[f's{i}_quotas'] = np.asarray(q, np.int64)
        flat[f's{i}_counts'] = np.asarray(c, np.int64)
    fractions = np.linspace(0, 1, 41)
    flat['time_in'] = fractions
    flat['time_out'] = np.asarray([actual_time(f) for f in fractions])
    flat['count'] = np.int64(len(rows))
    _save('schedule.npz', **flat)


def score_cases():
    """`entropy_scores`, the air probability and the per-column last mask on seeded logits."""
    from streamvoxel.sampling.entropy import entropy_scores
    from streamvoxel.sampling.low_entropy_last import low_entropy_last_update
    g = torch.Generator().manual_seed(7)
    out = {}
    for i, (classes, shape, eps) in enumerate([(6, (16, 8, 8), 1e-3), (256, (16, 4, 4), 1e-4), (33, (32, 4, 4), 0.05)]):
        logits = torch.randn((classes, *shape), generator=g) * 2
        logits[0, shape[0] // 2:] += 30.  # certain air above the middle
        logits[0, shape[0] // 2 - 2:shape[0] // 2] += 9.
        air = logits.float().softmax(0)[torch.tensor([0])].sum(0)
        mask = torch.ones(shape, dtype=torch.bool)
        last = low_entropy_last_update(torch.zeros(shape, dtype=torch.bool), mask, air, torch.zeros(shape, dtype=torch.bool),
                                       eps, False, True)
        out.update({f'e{i}_logits': logits.numpy(), f'e{i}_eps': np.float64(eps), f'e{i}_entropy': entropy_scores(logits).numpy(),
                    f'e{i}_air': air.numpy(), f'e{i}_last': last.numpy()})
    out['count'] = np.int64(3)
    _save('scores.npz', **out)


def _fixture_logits(step, ground=8, classes=6, shape=(16, 8, 8)):
    """`tests/stream/test_live_fast_ops.py:63-67`."""
    generator = torch.Generator().manual_seed(step + 1)
    logits = torch.randn((classes, *shape), generator=generator)
    logits[0, ground:] += 30.
    return logits


def slot_cases():
    """Whole windows of the reference `LowEntropyLastSlot` (`streamvoxel/stream/slot.py:50-176`) on the fixture logits
    of `tests/stream/test_live_fast_ops.py:70-91`, with the block order and every categorical draw's exponential
    noise recorded (cloned generator state, same call `torch.multinomial` makes)."""
    from streamvoxel.stream.slot import LowEntropyLastSlot
    shape, classes = (16, 8, 8), 6
    out = {}
    for i, seed in enumerate([3, 11, 12345]):
        slot = LowEntropyLastSlot(shape, classes, air_ids=(0,), air_token=0, last_eps=1e-3, block_size=4, device='cpu')
        tokens = torch.full(shape, classes, dtype=torch.long)
        cap = 8 + i
        slot.arm(seed, cap, (i, 0))
        out[f'w{i}_order'] = slot.order.numpy()
        out[f'w{i}_args'] = np.asarray([seed, cap, 6 + i], np.int64)
        step, draws = 0, []
        while not slot.idle:
            logits = _fixture_logits(step + 31 * i, ground=6 + i)
            noise = None
            if slot.phase == 'solid' and slot.solid_calls < len(slot.quotas):
                k = slot.quotas[slot.solid_calls]
                clone = torch.Generator().set_state(slot.generator.get_state())
                noise = torch.empty((k, classes)).exponential_(generator=clone)
            record, commit = slot.consume(logits, tokens)
            if commit is not None:
                p = logits.permute(1, 2, 3, 0).reshape(-1, classes)[torch.as_tensor(commit['positions']).long()].softmax(-1)
                assert torch.equal((p / noise).argmax(-1).to(torch.int16), torch.as_tensor(commit['values'])), 'multinomial != argmax(p/q)'
                out[f'w{i}_s{step}_positions'] = commit['positions']
                out[f'w{i}_s{step}_values'] = commit['values']
                out[f'w{i}_s{step}_noise'] = noise.numpy()
            step += 1
        out[f'w{i}_steps'] = np.int64(step)
        out[f'w{i}_tokens'] = tokens.numpy()
        out[f'w{i}_step_map'] = record['step_map'].numpy()
        out[f'w{i}_values'] = record['values'].numpy()
        out[f'w{i}_record'] = np.asarray([record['nfe'], record['actual'], record['last_count']], np.int64)
    out['count'] = np.int64(3)
    _save('slot_windows.npz', **out)


EVAL_SPECS = [
    dict(selection='random', schedule='quartercos', steps=8),
    dict(selection='entropy', schedule='linear', steps=6),
    dict(selection='mixed', schedule='halfcos', steps=8, candidate_multiplier=2.0),
    dict(selection='mixed', schedule='reversequarter', steps=5, candidate_multiplier=1.0),
    dict(selection='block', schedule='quartercos', steps=8, block_size=4),
    dict(selection='block', schedule='front2', steps=5, block_size=4),
    dict(selection='entropy', schedule='halfcos', steps=7, rounding='legacy'),
    dict(selection='random', schedule='native_quarter', steps=6),
    dict(selection='entropy', schedule='power2', steps=9),
]


def eval_logits(tokens, classes=6):
    """The evaluation fixtures' forward: fp32 logits [C, Y, Z, X], a pure function of how many voxels are masked."""
    masked = int((torch.as_tensor(tokens) == classes).sum())
    generator = torch.Generator().manual_seed(masked + 7)
    logits = torch.randn((classes, *tuple(tokens.shape)), generator=generator) * 1.5
    logits[0, 10:] += 4.
    return logits


def eval_cases():
    """Whole decodes of the reference evaluation decoder `decode` (`streamvoxel/eval/samplers.py:69-115`) on the CPU
    for every selection mode and several schedules, with every `torch.rand` draw, the exponential noise of every
    categorical draw (replayed from the seeded generator in the reference's call order) and the block order."""
    from streamvoxel.eval.samplers import decode
    shape, classes = (16, 8, 8), 6
    out = {}
    for i, spec in enumerate(EVAL_SPECS):
        seed = 100 + 17 * i
        forward = lambda tokens, t: eval_logits(tokens[0], classes)[None]
        result, meta = decode(forward, dict(spec), seed, 'cpu', shape=shape, classes=classes, trace=True)
        g = torch.Generator().manual_seed(seed)
        for j, ev in enumerate(meta['events']):
            out[f'e{i}_s{j}_draw'] = torch.rand(shape, generator=g).numpy()
            if ev['committed']:
                out[f'e{i}_s{j}_noise'] = torch.empty((ev['committed'], classes)).exponential_(generator=g).numpy()
        if spec['selection'] == 'block':
            bg = torch.Generator().manual_seed(seed + 9173)
            out[f'e{i}_order'] = torch.randperm(int(np.prod(shape)) // 64, generator=bg).numpy()
        out[f'e{i}_tokens'] = result['compact']
        out[f'e{i}_commit'] = result['commit_step'].astype(np.int32)
        keys = sorted({k for ev in meta['events'] for k in ev})
        out[f'e{i}_event_keys'] = np.asarray(keys)
        out[f'e{i}_events'] = np.asarray([[float(ev.get(k, np.nan)) for k in keys] for ev in meta['events']])
        out[f'e{i}_seed'] = np.int64(seed)
    out['count'] = np.int64(len(EVAL_SPECS))
    _save('eval_decode.npz', **out)


# ------------------------------------------------------------------------------------------------ models

def _reinit(model, std, seed):
    torch.manual_seed(seed)
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(std=std)
    return model.eval().requires_grad_(False)


def _state(model):
    return {k: v.detach().numpy() for k, v in model.state_dict().items()}


def model_cases():
    """Tiny time-free DiT and compact ControlNet forwards with every parameter re-drawn (the reference's own init
    zeroes the head, which would make every logit 0). fp32 on the CPU, the reference's CPU numerics."""
    from streamvoxel.models.unconditional_md4_timefree import UnconditionalMD4DiT
    from streamvoxel.models.compact_controlnet import CompactStreamingControlNet
    from streamvoxel.stream.condition import ModelSpec, Item
    from streamvoxel.stream.engine import unpadded_logits, encode_item
    from streamvoxel.stream.fast_ops import FastSlotForward

    cfg = dict(num_classes=5, voxel_shape=(16, 16, 16), hidden_dim=48, depth=3, num_heads=4, time_free=True)
    base = _reinit(UnconditionalMD4DiT(**cfg), 0.05, 11)
    tokens = torch.randint(6, (2, 16, 16, 16), generator=torch.Generator().manual_seed(12))
    logits = base(tokens, timestep=torch.ones(2))
    _save('dit_tiny.npz', tokens=tokens.numpy(), logits=logits.numpy(),
          **{'sd.' + k: v for k, v in _state(base).items()})
    with torch.autocast('cpu', dtype=torch.bfloat16):
        cpu_bf16 = base(tokens, timestep=torch.ones(2)).float()
    _save('dit_tiny_cpu_autocast.npz', logits=cpu_bf16.numpy())

    torch.manual_seed(5)
    base = UnconditionalMD4DiT(num_classes=3, voxel_shape=(16, 16, 16), hidden_dim=48, depth=5, num_heads=4, time_free=True)
    model = CompactStreamingControlNet(base, control_depth=3, control_hidden_dim=24, checkpointing=False,
                                       biome_halo=4, biome_patch=2, struct_classes=0)
    _reinit(model, 0.05, 13)
    spec = ModelSpec(height=16, tile=16, num_classes=3, biome_classes=66, biome_halo=4, y_origin=-64.)
    rng = np.random.default_rng(1)
    items = []
    for n1, n2, seed in ((1, 2, 1), (3, 3, 2), (0, 2, 3)):
        l1 = rng.integers(0, 3, (n1, 16, 16, 16)).astype(np.int16)
        l2 = rng.integers(0, 3, (n2, 16, 16, 16)).astype(np.int16)
        xz1 = np.asarray([[-16, 0], [16, 0], [0, 16]][:n1], np.int64).reshape(-1, 2)
        xz2 = np.asarray([[-32, 0], [32, 16], [0, -32]][:n2], np.int64).reshape(-1, 2)
        biomes = np.zeros((4, 12, 12), np.int64)
        biomes[:, 3:9, 3:9] = rng.integers(0, 66, (4, 6, 6))
        items.append(Item(f'i{seed}', seed, 8, 1.0, l1, xz1, l2, xz2, biomes, None))
    tokens = torch.randint(4, (3, 16, 16, 16), generator=torch.Generator().manual_seed(14))
    out = {'sd.' + k: v for k, v in _state(model).items()}
    engine = FastSlotForward(model, spec, 'cpu', 3, 3, 3, patchify='gather', attention='sdpa', capture=False)
    for i, item in enumerate(items):
        want = unpadded_logits(model, item, spec, tokens[i:i + 1], torch.ones(1))[0]
        layers = engine.encode(item)
        out[f'i{i}_logits'] = want.numpy()
        out[f'i{i}_l1'], out[f'i{i}_l1_xz'] = item.l1_blocks, item.l1_xz
        out[f'i{i}_l2'], out[f'i{i}_l2_xz'] = item.l2_blocks, item.l2_xz
        out[f'i{i}_biomes'] = item.biomes
        out[f'i{i}_k0'], out[f'i{i}_v0'] = layers[0][0][0].numpy(), layers[0][1][0].numpy()
        out[f'i{i}_k2'], out[f'i{i}_v2'] = layers[2][0][0].numpy(), layers[2][1][0].numpy()
        engine.load_slot(i, item)
    engine.tokens.copy_(tokens)
    packed = engine.eager(torch.ones(3))
    out['packed_logits'] = packed.numpy()
    out['lengths'] = engine.packed.lengths.numpy()
    out['tokens'] = tokens.numpy()
    out['layer_indices'] = np.asarray(model.layer_indices, np.int64)
    _save('control_tiny.npz', **out)


def full_size_case():
    """The reference's own fp32 forward of the BASELINE config-2 model (DiT-B/4, d = 768, 8 x 96 heads, V = 256, 12-layer
    ControlNet) on the CPU: `engine.unpadded_logits` (`streamvoxel/stream/engine.py:87-102`) with the seeded
    synthetic weights of `streamvoxel_b200.model.synthetic_state_dict(seed=0)` loaded into the reference module, one
    synthetic window (k = 2 L1 tiles, 80 L2 columns, the biome window) and a partially masked target. Stored: the
    logits of 512 seeded voxels (all 256 classes, fp32)."""
    from streamvoxel.models.compact_controlnet import CompactStreamingControlNet
    from streamvoxel.models.unconditional_md4_timefree import UnconditionalMD4DiT
    from streamvoxel.stream.condition import Item, ModelSpec
    from streamvoxel.stream.engine import install_slot_attention, unpadded_logits
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from streamvoxel_b200 import model as sm, synth
    from streamvoxel_b200.stream.condition import ModelSpec as OurSpec
    cfg = sm.dit_b4_control()
    base = UnconditionalMD4DiT(num_classes=256, voxel_shape=(256, 16, 16), hidden_dim=768, depth=12, num_heads=8,
                               time_free=True)
    model = CompactStreamingControlNet(base, control_depth=12, control_hidden_dim=768, checkpointing=False,
                                       biome_halo=4, biome_patch=4, biome_classes=16, struct_classes=0)
    state = sm.synthetic_state_dict(cfg, seed=0)
    missing, unexpected = model.load_state_dict(state, strict=False)
    assert not unexpected and all(k not in state for k in missing)
    model.eval().requires_grad_(False)
    install_slot_attention(model)   # as FastSlotForward does before the reference numerical gate calls unpadded_logits
    ours = synth.item(701, OurSpec.of(cfg), k=2)
    item = Item(ours.id, ours.seed, ours.steps, ours.temperature, ours.l1_blocks, ours.l1_xz, ours.l2_blocks,
                ours.l2_xz, ours.biomes, None)
    spec = ModelSpec(height=256, tile=16, num_classes=256, biome_classes=16, biome_halo=4, y_origin=-64.)
    tokens = torch.from_numpy(synth.target_tokens(801, OurSpec.of(cfg))[0][None]).long()
    with torch.no_grad():
        logits = unpadded_logits(model, item, spec, tokens, torch.ones(1))[0]
    voxels = np.sort(np.random.default_rng(3).choice(65536, 512, replace=False))
    _save('control_full.npz', voxels=voxels, logits=logits.reshape(256, -1)[:, voxels].numpy(),
          tokens=tokens[0].numpy().astype(np.int16))


# ---------------------------------------------------------------------------------------------- window admission

def _blob(rng, n):
    """A connected committed region: a random walk of n steps from (0, 0)."""
    cells, z, x = set(), 0, 0
    for _ in range(n):
        cells.add((z, x))
        dz, dx = ((1, 0), (-1, 0), (0, 1), (0, -1))[int(rng.integers(0, 4))]
        z, x = z + dz, x + dx
    return cells


def scheduler_cases():
    """The reference scheduler on seeded cases: pick_window, member_shares, window seeds and make_item."""
    from streamvoxel.stream.condition import ModelSpec
    from streamvoxel.stream.scheduler import make_item, member_shares, pick_window, seed
    rng = np.random.default_rng(41)
    out = {}
    for i in range(80):
        committed = _blob(rng, int(rng.integers(1, 48)))
        inflight, diagonal = set(), bool(i % 3 == 0)
        for _ in range(int(rng.integers(0, 7))):
            c = pick_window(committed, inflight, tuple(float(v) for v in rng.uniform(-90, 90, 2)), diagonal=diagonal)
            if c is None:
                break
            inflight.add(c)
        player = rng.uniform(-120, 120, 2)
        got = pick_window(committed, inflight, (float(player[0]), float(player[1])), diagonal=diagonal)
        out[f'p{i}_committed'] = np.asarray(sorted(committed), np.int64).reshape(-1, 2)
        out[f'p{i}_inflight'] = np.asarray(sorted(inflight), np.int64).reshape(-1, 2)
        out[f'p{i}_player'] = player
        out[f'p{i}_diagonal'] = diagonal
        out[f'p{i}_pick'] = np.asarray(got if got is not None else (-(2 ** 40), -(2 ** 40)), np.int64)
    for i in range(60):
        k = int(rng.integers(0, 6))
        wids = sorted(int(w) for w in rng.choice(12, k, replace=False))
        members = [(w, int(rng.integers(1, 17)), int(rng.integers(1, 17))) for w in wids]
        batch = int(rng.integers(0, sum(c for _, c, _ in members) + 4))
        shares = member_shares(batch, members)
        out[f'm{i}_members'] = np.asarray(members, np.int64).reshape(-1, 3)
        out[f'm{i}_batch'] = batch
        out[f'm{i}_shares'] = np.asarray([shares[w] for w, _, _ in members], np.int64)
    cells = [(int(a), int(b)) for a, b in rng.integers(-5000, 5000, (64, 2))]
    out['seed_cells'] = np.asarray(cells, np.int64)
    out['seed_values'] = np.asarray([seed(7, a, b) for a, b in cells], np.uint64)
    spec = ModelSpec(height=64, tile=16, num_classes=32, biome_classes=16, biome_halo=4, y_origin=-64.0)
    biomes = rng.integers(0, 16, (16, 66, 66)).astype(np.int64)
    for i in range(6):
        committed = _blob(rng, int(rng.integers(3, 30)))
        cells = {c: rng.integers(0, 33, (64, 16, 16)).astype(np.int16) for c in sorted(committed)}
        target = sorted(set((a + da, b + db) for a, b in committed for da in (-1, 0, 1) for db in (-1, 0, 1))
                        - committed)[int(rng.integers(0, 4))]
        item = make_item(cells, target, biomes, spec, 7, 32, 5)
        out[f'i{i}_cells'] = np.asarray(sorted(cells), np.int64)
        out[f'i{i}_tiles'] = np.stack([cells[c] for c in sorted(cells)])
        out[f'i{i}_target'] = np.asarray(target, np.int64)
        for name in ('l1_blocks', 'l1_xz', 'l2_blocks', 'l2_xz', 'biomes'):
            out[f'i{i}_{name}'] = getattr(item, name)
        out[f'i{i}_seed'] = np.uint64(item.seed)
    out['biomes'] = biomes
    _save('scheduler.npz', **out)


# ---------------------------------------------------------------------------------------------- commit wire format

def wire_cases():
    """Frame rows, merged commits, packet hashes and batch lines made by the reference's live protocol code."""
    import json
    from streamvoxel.common.live_rows import pack_row, unpack_row
    from streamvoxel.common.live_wire import batch_line, packet_sha
    from streamvoxel.stream.worker import _merge_commits
    rng = np.random.default_rng(53)
    out, rows = {}, []
    for i in range(12):
        n = int(rng.integers(0, 3000)) if i else 0
        positions = rng.choice(65536, n, replace=False).astype(np.int32)
        raw = rng.integers(0, 981, n).astype(np.uint16)
        raw[rng.random(n) < 0.3] = 0
        row = pack_row((int(rng.integers(-50, 50)), int(rng.integers(-50, 50))), positions, raw)
        out[f'r{i}_positions'], out[f'r{i}_raw'] = positions, raw
        out[f'r{i}_row'] = np.array(json.dumps(row, sort_keys=True))
        pos, val = unpack_row(row)
        out[f'r{i}_unpacked_pos'], out[f'r{i}_unpacked_val'] = pos, val
        rows.append(row)
    for i in range(6):
        commits = []
        for step in range(int(rng.integers(1, 4))):
            n = int(rng.integers(1, 500))
            commits.append(dict(positions=rng.integers(0, 2048, n).astype(np.int32),
                                values=rng.integers(0, 256, n).astype(np.int16), step=step + 1, target=(3, -4)))
        merged = _merge_commits(commits)
        for j, c in enumerate(commits):
            out[f'm{i}_c{j}_positions'], out[f'm{i}_c{j}_values'] = c['positions'], c['values']
        out[f'm{i}_count'] = len(commits)
        out[f'm{i}_positions'], out[f'm{i}_values'] = merged['positions'], merged['values']
    packets = []
    for seq in range(5):
        packet = dict(seq=seq, kind='frame' if seq % 2 else 'window_commit', forward=seq * 7, gpu=seq % 2,
                      frames=rows[seq:seq + 2] if seq % 2 else [], target=[seq, -seq], nfe=33, last_frac=0.25)
        packet['sha256'] = packet_sha(packet)
        packets.append(packet)
    out['packets'] = np.array(json.dumps(packets))
    out['batch'] = np.array(json.dumps(batch_line(packets), sort_keys=True))
    _save('wire.npz', **out)


CASES = dict(quota=lambda: quota_cases(), top_mask=lambda: top_mask_cases(), schedule=lambda: schedule_cases(),
             scores=lambda: score_cases(), slots=lambda: slot_cases(), models=lambda: model_cases(),
             scheduler=lambda: scheduler_cases(), wire=lambda: wire_cases(), eval=lambda: eval_cases(),
             full_size=lambda: full_size_case())


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument('--reference', required=True)
    parser.add_argument('--only', nargs='*', choices=sorted(CASES), help='regenerate only these fixture groups')
    args = parser.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for name in (args.only or CASES):
        CASES[name]()


if __name__ == '__main__':
    main()
