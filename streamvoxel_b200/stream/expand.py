"""World expansion on one or more GPUs: the host driver of BASELINE configs 4/5 (a committed start region grown window
by window in `pick_window` order around the player).

Multi-GPU without a collective on the data path (`streamvoxel/stream/scheduler.py:37-151`, `session.py:419-500`):
every rank keeps the same committed snapshot and in-flight set and runs the same deterministic admission, so each
knows which windows it owns; after every engine step the ranks exchange the columns they finished (128 KiB of int16
tokens each) and their free slot counts with one host all-gather (a gloo group), apply all commits in rank order and
admit again. The in-flight windows are pairwise Chebyshev >= 2 apart and condition only on committed columns, so no
rank ever waits for another's window; a rank's in-flight count is bounded by its `member_shares` share of the batch.
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np

from .scheduler import fast_item, member_shares, separated, window_seed


class Expansion:
    """Committed snapshot, in-flight windows and admission of one expansion (one replica per rank)."""

    def __init__(self, committed, biomes, spec, player_zx, region, *, ranks=1, slots=8, cap=32, l2_cap=81, world=0,
                 cell_size=16, diagonal=False, batch=None):
        self.committed = {tuple(c): np.asarray(t, np.int16) for c, t in committed.items()}
        self.biomes, self.spec, self.player = biomes, spec, tuple(float(v) for v in player_zx)
        self.region = {tuple(c) for c in region}
        self.ranks, self.cap, self.l2_cap, self.world = int(ranks), int(cap), int(l2_cap), int(world)
        self.cell_size, self.diagonal = cell_size, diagonal
        total = self.ranks * int(slots) if batch is None else int(batch)
        self.share = member_shares(total, [(r, int(slots), 1) for r in range(self.ranks)])
        self.inflight = {}          # cell -> owning rank
        self.ready = set()          # uncommitted cells with a committed 8-neighbour, inside the region
        for c in self.committed:
            self._touch(c)
        self.blocked_admissions = 0  # free slots left empty because no admissible cell existed

    def _touch(self, cell):
        z, x = cell
        for a in (z - 1, z, z + 1):
            for b in (x - 1, x, x + 1):
                if (a, b) not in self.committed and (a, b) in self.region:
                    self.ready.add((a, b))
        self.ready.discard(cell)

    @property
    def done(self):
        return self.region.issubset(self.committed.keys())

    def pick(self):
        """`pick_window` restricted to the region, over the incrementally kept ready set (same key and rule)."""
        pz, px = self.player
        best_key, best = None, None
        for cell in self.ready:
            if cell in self.inflight or not separated(cell, self.inflight, diagonal=self.diagonal):
                continue
            z, x = cell
            key = (((z + .5) * self.cell_size - pz) ** 2 + ((x + .5) * self.cell_size - px) ** 2, z, x)
            if best_key is None or key < best_key:
                best_key, best = key, cell
        return best

    def apply(self, commits):
        """Commit finished windows [(cell, tokens)] (every rank applies every rank's commits in rank order)."""
        for cell, tokens in commits:
            cell = tuple(cell)
            self.committed[cell] = np.asarray(tokens, np.int16)
            self.inflight.pop(cell, None)
            self._touch(cell)

    def admit(self, free):
        """Windows each rank starts now: round-robin over ranks in order, one admission at a time, each rank up to
        its free slots and its share. Returns {rank: [cell, ...]} (identical on every replica)."""
        active = {r: 0 for r in range(self.ranks)}
        for r in self.inflight.values():
            active[r] += 1
        room = {r: max(0, min(int(free[r]), self.share[r] - active[r])) for r in range(self.ranks)}
        picks = {r: [] for r in range(self.ranks)}
        while any(room.values()):
            for r in range(self.ranks):
                if not room[r]:
                    continue
                cell = self.pick()
                if cell is None:
                    self.blocked_admissions += sum(room.values())
                    return picks
                self.inflight[cell] = r
                picks[r].append(cell)
                room[r] -= 1
        return picks

    def item(self, cell):
        """The window's `Item` (`make_item`'s result; L2 tiles stacked lazily, see `scheduler.fast_item`)."""
        return fast_item(self.committed, cell, self.biomes, self.spec, self.world, self.cap, self.l2_cap)

    def seed(self, cell):
        return window_seed(self.world, *cell)

    def digest(self):
        """Order-independent digest of the committed snapshot (replicas must agree)."""
        import hashlib
        h = hashlib.sha256()
        for cell in sorted(self.committed):
            h.update(np.asarray(cell, np.int64).tobytes())
            h.update(self.committed[cell].tobytes())
        return h.hexdigest()


def _publish(publisher, record, cell, tokens, slot, rank, world, raw_map):
    from . import wire
    record = dict(record, target=cell)
    ids = raw_map if raw_map is not None else np.arange(int(tokens.max()) + 1, dtype=np.uint16)
    row = wire.frame_row(wire.whole_cell_commit(cell, tokens, record['nfe']), ids, slot, rank)
    if row is not None:
        publisher.publish('frame', gpu=rank, world=world, frames=[row])
    publisher.publish('window_commit', **wire.window_commit_fields(record, rank, slot, world))


def host_exchange(obj, group=None):
    """All-gather a picklable object over the host group (identity on one rank)."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return [obj]
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


class DeviceExchange:
    """`host_exchange` of (finished columns, free slots) over a device process group (NCCL), in two forms.

    Called (`exchange(obj)`): a fixed-size header per rank (finished count, free slots, the finished cells)
    all-gathered every round, and the finished columns all-gathered only in rounds where some rank finished one (every
    rank reads the same headers, so all take the same collectives). Returns what `host_exchange` returns.

    Started and finished (`start(obj)`, then `finish()` a round later, as `run` does with this exchange): one
    all-gather per round of the header and all `slots` column buffers, enqueued on the exchange's stream and read back
    a round later, so no rank waits for the others' current round (the round's admission uses the previous round's
    reports; see `_run_pipelined`). Two buffer sets alternate between the rounds in flight.

    The collectives run on a stream of their own, so they do not queue behind the steps in flight, and only the
    columns that exist are copied back to the host."""

    def __init__(self, group, slots, shape, device):
        import contextlib

        import torch
        import torch.distributed as dist
        self.torch, self.dist, self.group = torch, dist, group
        self.ranks = dist.get_world_size(group)
        self.slots, self.shape = int(slots), tuple(shape)
        self.width = 2 + 2 * self.slots
        device = torch.device(device)
        cuda = device.type == 'cuda'
        self.device = device
        # A CPU device (a gloo group) runs the same collectives on the calling thread; it is there for tests.
        self.stream = torch.cuda.Stream(device=device) if cuda else None
        self.context = (lambda: torch.cuda.stream(self.stream)) if cuda else contextlib.nullcontext
        self.header_host = torch.zeros(self.width, dtype=torch.int64, pin_memory=cuda)
        self.header = torch.zeros(self.width, dtype=torch.int64, device=device)
        self.headers = torch.zeros((self.ranks, self.width), dtype=torch.int64, device=device)
        self.columns_host = torch.zeros((self.slots, *self.shape), dtype=torch.int16, pin_memory=cuda)
        self.columns = torch.zeros((self.slots, *self.shape), dtype=torch.int16, device=device)
        self.gathered = torch.zeros((self.ranks, self.slots, *self.shape), dtype=torch.int16, device=device)
        # NCCL has no 16-bit integer type: the columns travel as their bytes.
        self.columns_bytes = self.columns.view(-1).view(torch.uint8)
        self.gathered_bytes = self.gathered.view(-1).view(torch.uint8)
        # the started form: per buffer set, one record of header bytes then the columns, per rank
        self.record_bytes = self.width * 8 + self.columns.numel() * 2
        self.sets = None
        self.in_flight = []   # (set index, event) of started exchanges, oldest first
        self.rounds = 0

    def _pack(self, obj, header, columns):
        torch = self.torch
        finished, free = obj
        if len(finished) > self.slots:
            raise ValueError('more finished windows than slots')
        header.zero_()
        header[0], header[1] = len(finished), int(free)
        for j, (cell, column) in enumerate(finished):
            header[2 + 2 * j], header[3 + 2 * j] = int(cell[0]), int(cell[1])
            columns[j].copy_(torch.from_numpy(np.ascontiguousarray(column, np.int16)))

    def __call__(self, obj):
        torch, dist = self.torch, self.dist
        finished, _ = obj
        self._pack(obj, self.header_host, self.columns_host)
        with self.context():
            self.header.copy_(self.header_host, non_blocking=True)
            dist.all_gather_into_tensor(self.headers.view(-1), self.header, group=self.group)
            headers = self.headers.cpu().numpy()   # waits for this stream only
            out = [([], int(h[1])) for h in headers]
            if int(headers[:, 0].sum()):
                if finished:
                    self.columns[:len(finished)].copy_(self.columns_host[:len(finished)], non_blocking=True)
                dist.all_gather_into_tensor(self.gathered_bytes, self.columns_bytes, group=self.group)
                for r, h in enumerate(headers):
                    count = int(h[0])
                    if count:
                        cols = self.gathered[r, :count].cpu().numpy()
                        out[r] = ([((int(h[2 + 2 * j]), int(h[3 + 2 * j])), cols[j].copy()) for j in range(count)],
                                  int(h[1]))
        return out

    def _set(self, k):
        torch = self.torch
        if self.sets is None:
            cuda = self.device.type == 'cuda'
            self.sets = [dict(host=torch.zeros(self.record_bytes, dtype=torch.uint8, pin_memory=cuda),
                              send=torch.zeros(self.record_bytes, dtype=torch.uint8, device=self.device),
                              recv=torch.zeros(self.ranks * self.record_bytes, dtype=torch.uint8, device=self.device))
                         for _ in range(2)]
        return self.sets[k]

    def start(self, obj):
        """Enqueue this round's exchange of (finished columns, free slots); `finish` returns it."""
        torch, dist = self.torch, self.dist
        if len(self.in_flight) >= 2:
            raise RuntimeError('two exchanges are already in flight; finish one first')
        k = self.rounds % 2
        self.rounds += 1
        buf = self._set(k)
        header = buf['host'][:self.width * 8].view(torch.int64)
        columns = buf['host'][self.width * 8:].view(torch.int16).view(self.slots, *self.shape)
        self._pack(obj, header, columns)
        with self.context():
            buf['send'].copy_(buf['host'], non_blocking=True)
            dist.all_gather_into_tensor(buf['recv'], buf['send'], group=self.group)
            event = torch.cuda.Event() if self.stream is not None else None
            if event is not None:
                event.record(self.stream)
        self.in_flight.append((k, event))

    def finish(self):
        """The oldest started exchange: [(finished [(cell, column)], free slots)] per rank, as `host_exchange`."""
        torch = self.torch
        k, event = self.in_flight.pop(0)
        buf = self._set(k)
        if event is not None:
            event.synchronize()
        recv = buf['recv'].view(self.ranks, self.record_bytes)
        headers = recv[:, :self.width * 8].contiguous().view(torch.int64).view(self.ranks, self.width).cpu().numpy()
        out = []
        for r, h in enumerate(headers):
            count = int(h[0])
            finished = []
            if count:
                cols = recv[r, self.width * 8:].view(torch.int16).view(self.slots, *self.shape)[:count].cpu().numpy()
                finished = [((int(h[2 + 2 * j]), int(h[3 + 2 * j])), cols[j].copy()) for j in range(count)]
            out.append((finished, int(h[1])))
        return out


def run(engine, expansion, rank, *, group=None, max_rounds=1_000_000, publisher=None, raw_map=None, pipelined=None,
        exchange=None):
    """Drive `engine` (a `SlotBatch`, or any object with `slots`, `arm`, `step` and `column`) until the region is
    committed. Returns statistics of this rank. With a `publisher` (`wire.Publisher`), every window this rank
    finishes is published as a frame packet carrying its whole cell (global ids through `raw_map`) followed by its
    `window_commit` packet, as the reference's worker does without progressive frames.

    `exchange`: the callable that all-gathers (finished, free slots) between the ranks (default `host_exchange` over
    `group`; `DeviceExchange` gathers over NCCL).

    Pipelined (the default for an engine with `launch`/`collect`): the windows admitted after a step are built and
    armed while the next step runs on the GPU (their condition encode joins before the step after), so the host's
    admission work overlaps the device; a slot whose window finished sits out one step."""
    if pipelined is None:
        pipelined = hasattr(engine, 'launch') and hasattr(engine, 'collect')
    if exchange is None:
        exchange = lambda obj: host_exchange(obj, group)
    if pipelined:
        return _run_pipelined(engine, expansion, rank, exchange=exchange, max_rounds=max_rounds, publisher=publisher,
                              raw_map=raw_map)
    slot_cell = [None] * engine.slots
    stats = dict(rounds=0, forwards=0, windows=0, committed_voxels=0, admission_seconds=0.0, step_seconds=0.0,
                 item_seconds=0.0, arm_seconds=0.0, exchange_seconds=0.0)
    clock = time.perf_counter
    for _ in range(max_rounds):
        finished = []
        if any(c is not None for c in slot_cell):
            t = clock()
            results = engine.step()
            stats['step_seconds'] += clock() - t
            stats['forwards'] += 1
            for i, (record, _commit) in results.items():
                if record is not None and slot_cell[i] is not None:
                    tokens = engine.column(i)
                    finished.append((slot_cell[i], tokens))
                    if publisher is not None:
                        _publish(publisher, record, slot_cell[i], tokens, i, rank, expansion.ranks, raw_map)
                    stats['windows'] += 1
                    stats['committed_voxels'] += int(tokens.size)
                    slot_cell[i] = None
        t0 = clock()
        free_slots = [i for i, c in enumerate(slot_cell) if c is None]
        gathered = exchange((finished, len(free_slots)))
        stats['exchange_seconds'] += clock() - t0
        for commits, _ in gathered:
            expansion.apply(commits)
        picks = expansion.admit([n for _, n in gathered])
        for cell in picks[rank]:
            i = free_slots.pop(0)
            t = clock()
            item = expansion.item(cell)
            t1 = clock()
            engine.arm(i, expansion.seed(cell), expansion.cap, item=item, target=cell)
            stats['item_seconds'] += t1 - t
            stats['arm_seconds'] += clock() - t1
            slot_cell[i] = cell
        stats['admission_seconds'] += clock() - t0
        stats['rounds'] += 1
        if expansion.done:
            break
        if not expansion.inflight:
            raise RuntimeError('expansion blocked: no window in flight and none admissible')
    stats['blocked_admissions'] = expansion.blocked_admissions
    return stats


def _run_pipelined(engine, expansion, rank, *, exchange, max_rounds, publisher, raw_map):
    """`run` with the host's admission work overlapping the device. One round: launch the next step at once (the
    slots of windows that finished in the previous step sit it out), then -- while it runs -- read the finished
    windows' columns (copies enqueued before the launch), exchange and commit them, admit new windows and arm them
    into the free slots (as many as fit in the step's duration), then collect the step.

    With an exchange that has `start` / `finish` (`DeviceExchange`), the exchange runs a round behind: a round applies
    and admits from the reports every rank started in the previous round, then starts its own report (the columns it
    read, and its free slots after this round's admissions), so no rank waits for the others' current round. Every
    rank applies the same reports in the same round, so the replicas stay identical; a rank's reported free slots can
    only grow before the report is used (collects free slots, only admissions take them), so no slot is given twice."""
    slot_cell = [None] * engine.slots
    to_arm = []      # (slot, cell) admitted, not yet armed
    pending = []     # (cell, record, slot, column reader) of windows the last collect finished
    stats = dict(rounds=0, forwards=0, windows=0, committed_voxels=0, admission_seconds=0.0, step_seconds=0.0,
                 item_seconds=0.0, arm_seconds=0.0, exchange_seconds=0.0, collect_wait_seconds=0.0, pipelined=True,
                 deferred_arms=0, launched_ahead=0)
    clock = time.perf_counter
    step_time = 0.0   # running estimate of one step's wall time (launch to collected)
    read_async = hasattr(engine, 'column_async')
    depth = getattr(engine, 'depth', 1)
    lagged = hasattr(exchange, 'start') and hasattr(exchange, 'finish')
    stalled = 0
    if lagged:   # before the first report: every rank has all its slots free
        previous = [([], engine.slots) for _ in range(expansion.ranks)]
    for _ in range(max_rounds):
        began = clock()
        # keep up to `depth` steps in flight: the next step is queued before the host works on the last one's results
        if hasattr(engine, 'runnable'):
            while engine.in_flight < depth and engine.runnable():
                stats['launched_ahead'] += engine.in_flight > 0
                engine.launch()
            launched = engine.in_flight > 0
        else:
            waiting = {s for s, _ in to_arm}
            launched = any(c is not None and i not in waiting for i, c in enumerate(slot_cell))
            if launched:
                engine.launch()
        stats['step_seconds'] += clock() - began
        t0 = clock()
        finished = []
        for cell, record, slot, read in pending:
            tokens = read()
            finished.append((cell, tokens))
            if publisher is not None:
                _publish(publisher, record, cell, tokens, slot, rank, expansion.ranks, raw_map)
            stats['windows'] += 1
            stats['committed_voxels'] += int(tokens.size)
        pending = []
        free_slots = [i for i, c in enumerate(slot_cell) if c is None]
        if lagged:
            gathered = exchange.finish() if exchange.in_flight else previous
        else:
            gathered = exchange((finished, len(free_slots)))
        stats['exchange_seconds'] += clock() - t0
        for commits, _ in gathered:
            expansion.apply(commits)
        picks = expansion.admit([n for _, n in gathered])
        for cell in picks[rank]:
            i = free_slots.pop(0)
            slot_cell[i] = cell
            to_arm.append((i, cell))
        if lagged:
            t1 = clock()
            exchange.start((finished, len(free_slots)))
            stats['exchange_seconds'] += clock() - t1
        stats['admission_seconds'] += clock() - t0
        # Arm while the step still runs (at least one per step; all of them when nothing runs), so a burst of finishing
        # windows does not idle the device.
        armed = 0
        while to_arm and (not launched or armed == 0 or clock() - began < 0.8 * step_time):
            i, cell = to_arm.pop(0)
            t = clock()
            item = expansion.item(cell)
            t1 = clock()
            engine.arm(i, expansion.seed(cell), expansion.cap, item=item, target=cell, wait=False)
            stats['item_seconds'] += t1 - t
            stats['arm_seconds'] += clock() - t1
            armed += 1
        stats['deferred_arms'] += len(to_arm)
        if launched:
            t = clock()
            results = engine.collect()
            wait = clock() - t
            stats['collect_wait_seconds'] += wait
            if wait > 1e-4:   # the device, not the host's arming, set this step's duration
                elapsed = clock() - began
                step_time = elapsed if step_time == 0.0 else 0.9 * step_time + 0.1 * elapsed
            stats['forwards'] += 1
            for i, (record, _commit) in results.items():
                if record is not None and slot_cell[i] is not None:
                    if 'column' in record:   # the engine copied it out with the step
                        read = (lambda column=record['column']: column)
                    elif read_async:
                        read = engine.column_async(i)
                    else:
                        column = engine.column(i)
                        read = (lambda column=column: column)
                    pending.append((slot_cell[i], record, i, read))
                    slot_cell[i] = None
        stats['rounds'] += 1
        if expansion.done and not pending:   # every rank applies the same reports, so all stop in this round
            break
        # nothing running, read or waiting to be armed: with the lagged exchange, reports still on their way may free
        # cells for a round or two
        stalled = stalled + 1 if not expansion.inflight and not pending and not to_arm else 0
        if stalled > (2 if lagged else 0):
            raise RuntimeError('expansion blocked: no window in flight and none admissible')
    if lagged:
        while exchange.in_flight:   # the last round's reports (no commits once the region is done)
            exchange.finish()
    stats['blocked_admissions'] = expansion.blocked_admissions
    return stats


def start_region(seed, side0, side1, spec, classes=None):
    """A side0 x side0 committed square from the synthetic world generator, centred in the side1 x side1 target
    region (configs 4/5: 32 -> 64 and 32 -> 128), the biome labels and the player at the centre."""
    from streamvoxel_b200 import synth
    cols = synth.world(seed, side1, side1, height=spec.height, tile=spec.tile)
    if classes is not None:
        cols = {c: synth.clip_classes(t, classes) for c, t in cols.items()}
    lo = (side1 - side0) // 2
    committed = {c: t for c, t in cols.items() if lo <= c[0] < lo + side0 and lo <= c[1] < lo + side0}
    region = set(cols)
    rng = np.random.default_rng(seed + 1)
    biomes = rng.integers(0, 16, (spec.height // 4, 66, 66)).astype(np.int64)
    player = (side1 * spec.tile / 2.0, side1 * spec.tile / 2.0)
    return committed, region, biomes, player


def main():
    """python -m streamvoxel_b200.stream.expand [--side0 8 --side1 16] (torchrun for several GPUs): one expansion
    through the real engine; prints one JSON line with committed voxels/s and the admission statistics."""
    import os

    import torch
    import torch.distributed as dist

    from streamvoxel_b200 import model as sm
    from streamvoxel_b200.stream.batch import SlotBatch
    from streamvoxel_b200.stream.condition import ModelSpec
    from streamvoxel_b200.stream.fast_ops import FastSlotForward

    parser = argparse.ArgumentParser()
    parser.add_argument('--side0', type=int, default=8)
    parser.add_argument('--side1', type=int, default=16)
    parser.add_argument('--slots', type=int, default=8)
    parser.add_argument('--small', action='store_true', help='the small test model instead of DiT-B/4 + ControlNet')
    args = parser.parse_args()
    world_size = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    group = None
    if world_size > 1:
        dist.init_process_group('gloo', init_method='env://')
        group = dist.group.WORLD
    cfg = sm.small_test_config() if args.small else sm.dit_b4_control()
    sd = sm.synthetic_state_dict(cfg, seed=0)
    spec = ModelSpec.of(cfg)
    forward = FastSlotForward((cfg, sd), spec, f'cuda:{local}', args.slots, 8, 81)
    engine = SlotBatch(forward)
    committed, region, biomes, player = start_region(11, args.side0, args.side1, spec, classes=cfg.classes)
    exp = Expansion(committed, biomes, spec, player, region, ranks=world_size, slots=args.slots, l2_cap=81)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    stats = run(engine, exp, rank, group=group)
    torch.cuda.synchronize()
    seconds = time.perf_counter() - t0
    totals = host_exchange((stats['committed_voxels'], seconds, exp.digest()), group)
    if rank == 0:
        voxels = sum(t[0] for t in totals)
        wall = max(t[1] for t in totals)
        print(json.dumps(dict(workload=f'expansion {args.side0}^2 -> {args.side1}^2', ranks=world_size,
                              committed_voxels=voxels, seconds=wall, voxels_per_s=voxels / wall,
                              windows=len(region) - len(committed), replicas_agree=len({t[2] for t in totals}) == 1,
                              rank0=stats)))
    if world_size > 1:
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
