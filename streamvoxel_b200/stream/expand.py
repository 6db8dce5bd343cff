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

from .scheduler import fast_item, member_shares, window_seed


class _InFlight(dict):
    """The in-flight windows (cell -> owning rank) with, per cell, how many of them it lies too close to. `separated`
    admits a cell when it keeps Chebyshev distance >= 2 from every in-flight window (Manhattan >= 2 with `diagonal`),
    i.e. when no window lies in its 3x3 block (its 4-neighbour cross with `diagonal`); the blocks are symmetric, so
    a cell is admissible exactly when it is not a key of `near`."""

    def __init__(self, diagonal=False):
        super().__init__()
        self.reach = [(a, b) for a in (-1, 0, 1) for b in (-1, 0, 1) if not diagonal or abs(a) + abs(b) <= 1]
        self.near = {}

    def _count(self, cell, step):
        z, x = cell
        near = self.near
        for a, b in self.reach:
            key = (z + a, x + b)
            count = near.get(key, 0) + step
            if count:
                near[key] = count
            else:
                del near[key]

    def __setitem__(self, cell, rank):
        if cell not in self:
            self._count(cell, 1)
        super().__setitem__(cell, rank)

    def __delitem__(self, cell):
        super().__delitem__(cell)
        self._count(cell, -1)

    def pop(self, cell, *default):
        if cell in self:
            self._count(cell, -1)
        return super().pop(cell, *default)

    def _unsupported(self, *args, **kwargs):
        raise TypeError('in-flight windows change only by item assignment, del and pop')

    update = setdefault = popitem = clear = _unsupported


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
        self.inflight = _InFlight(diagonal)  # cell -> owning rank
        self.ready = {}             # uncommitted cells with a committed 8-neighbour, inside the region -> pick key
        self.open = self.region - self.committed.keys()   # region cells still to commit
        for c in self.committed:
            self._touch(c)
        self.blocked_admissions = 0  # free slots left empty because no admissible cell existed

    def _touch(self, cell):
        z, x = cell
        pz, px, size = self.player[0], self.player[1], self.cell_size
        for a in (z - 1, z, z + 1):
            for b in (x - 1, x, x + 1):
                if (a, b) not in self.committed and (a, b) in self.region and (a, b) not in self.ready:
                    self.ready[(a, b)] = (((a + .5) * size - pz) ** 2 + ((b + .5) * size - px) ** 2, a, b)
        self.ready.pop(cell, None)

    @property
    def done(self):
        return not self.open

    def pick(self):
        """`pick_window` restricted to the region, over the incrementally kept ready set (same key and rule): the
        nearest ready cell that no in-flight window blocks. `_InFlight.near` answers `separated` per cell in O(1)
        and `ready` maps each cell to its key (the player is fixed), so a pick costs one pass over the frontier."""
        near = self.inflight.near
        best_key, best = None, None
        for cell, key in self.ready.items():
            if cell in near:
                continue
            if best_key is None or key < best_key:
                best_key, best = key, cell
        return best

    def apply(self, commits):
        """Commit finished windows [(cell, tokens)] (every rank applies every rank's commits in rank order)."""
        for cell, tokens in commits:
            cell = tuple(cell)
            self.committed[cell] = np.asarray(tokens, np.int16)
            self.open.discard(cell)
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
    """`host_exchange` of (finished columns, free slots) over a device process group (NCCL): a fixed-size header per
    rank (finished count, free slots, the finished cells) all-gathered every round, and the finished columns
    all-gathered only in rounds where some rank finished one (every rank reads the same headers, so all take the same
    collectives). The collectives run on a stream of their own, so they do not queue behind the steps in flight, and
    only the columns that exist are copied back to the host. Returns what `host_exchange` returns."""

    def __init__(self, group, slots, shape, device):
        import contextlib

        import torch
        import torch.distributed as dist
        self.torch, self.dist, self.group = torch, dist, group
        self.ranks = dist.get_world_size(group)
        self.slots, self.shape = int(slots), tuple(shape)
        width = 2 + 2 * self.slots
        device = torch.device(device)
        cuda = device.type == 'cuda'
        # A CPU device (a gloo group) runs the same collectives on the calling thread; it is there for tests.
        self.stream = torch.cuda.Stream(device=device) if cuda else None
        self.context = (lambda: torch.cuda.stream(self.stream)) if cuda else contextlib.nullcontext
        self.header_host = torch.zeros(width, dtype=torch.int64, pin_memory=cuda)
        self.header = torch.zeros(width, dtype=torch.int64, device=device)
        self.headers = torch.zeros((self.ranks, width), dtype=torch.int64, device=device)
        self.columns_host = torch.zeros((self.slots, *self.shape), dtype=torch.int16, pin_memory=cuda)
        self.columns = torch.zeros((self.slots, *self.shape), dtype=torch.int16, device=device)
        self.gathered = torch.zeros((self.ranks, self.slots, *self.shape), dtype=torch.int16, device=device)
        # NCCL has no 16-bit integer type: the columns travel as their bytes.
        self.columns_bytes = self.columns.view(-1).view(torch.uint8)
        self.gathered_bytes = self.gathered.view(-1).view(torch.uint8)

    def __call__(self, obj):
        torch, dist = self.torch, self.dist
        finished, free = obj
        if len(finished) > self.slots:
            raise ValueError('more finished windows than slots')
        header = self.header_host
        header.zero_()
        header[0], header[1] = len(finished), int(free)
        for j, (cell, column) in enumerate(finished):
            header[2 + 2 * j], header[3 + 2 * j] = int(cell[0]), int(cell[1])
            self.columns_host[j].copy_(torch.from_numpy(np.ascontiguousarray(column, np.int16)))
        with self.context():
            self.header.copy_(header, non_blocking=True)
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
    admission work overlaps the device; a slot whose window finished sits out one step.

    Host timers in the statistics: `exchange_seconds` reading finished columns and the all-gather,
    `admission_seconds` applying commits and `admit`, `item_seconds` / `arm_seconds` building and arming windows,
    `collect_wait_seconds` (pipelined) waiting for a step."""
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
        t0_exchange = clock()
        free_slots = [i for i, c in enumerate(slot_cell) if c is None]
        gathered = exchange((finished, len(free_slots)))
        t0 = clock()
        stats['exchange_seconds'] += t0 - t0_exchange
        for commits, _ in gathered:
            expansion.apply(commits)
        picks = expansion.admit([n for _, n in gathered])
        stats['admission_seconds'] += clock() - t0
        for cell in picks[rank]:
            i = free_slots.pop(0)
            t = clock()
            item = expansion.item(cell)
            t1 = clock()
            engine.arm(i, expansion.seed(cell), expansion.cap, item=item, target=cell)
            stats['item_seconds'] += t1 - t
            stats['arm_seconds'] += clock() - t1
            slot_cell[i] = cell
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
    into the free slots (as many as fit in the step's duration), then collect the step."""
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
        gathered = exchange((finished, len(free_slots)))
        t0_admission = clock()
        stats['exchange_seconds'] += t0_admission - t0
        for commits, _ in gathered:
            expansion.apply(commits)
        picks = expansion.admit([n for _, n in gathered])
        for cell in picks[rank]:
            i = free_slots.pop(0)
            slot_cell[i] = cell
            to_arm.append((i, cell))
        stats['admission_seconds'] += clock() - t0_admission
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
        if expansion.done and not pending:
            break
        if not expansion.inflight and not pending and not to_arm:
            raise RuntimeError('expansion blocked: no window in flight and none admissible')
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


class _StandInEngine:
    """A slot batch whose windows take `forwards` steps and commit nothing (for `simulate`): `launch` / `collect` with
    two steps in flight, as `SlotBatch` runs them."""
    depth = 2

    def __init__(self, slots, forwards, shape):
        self.slots, self.forwards, self.shape = slots, forwards, shape
        self.left = [0] * slots
        self.to_launch = [0] * slots
        self.targets = [None] * slots
        self.queue = []

    @property
    def in_flight(self):
        return len(self.queue)

    def runnable(self):
        return any(self.to_launch)

    def arm(self, slot, seed, cap, item=None, target=(), wait=True):
        self.left[slot] = self.to_launch[slot] = self.forwards
        self.targets[slot] = target

    def launch(self):
        entry = [i for i in range(self.slots) if self.to_launch[i]]
        for i in entry:
            self.to_launch[i] -= 1
        self.queue.append(entry)

    def collect(self):
        out = {}
        for i in self.queue.pop(0):
            self.left[i] -= 1
            record = dict(target=self.targets[i], column=np.zeros(self.shape, np.int16)) if self.left[i] == 0 else None
            out[i] = (record, None)
        return out


def simulate(side0, side1, spec, slots, forwards=33, seed=11):
    """The steps an expansion of the side0^2 -> side1^2 region takes under the admission rules (Chebyshev >= 2,
    nearest to the player, at most `slots` windows in flight) when every window takes `forwards` steps: the step count
    that bounds several GPUs before any host or exchange cost (`slots` = GPUs x slots per GPU). Host-only; returns
    the driver's statistics (`forwards` = steps, `blocked_admissions` = slot-rounds left empty)."""
    committed, region, biomes, player = start_region(seed, side0, side1, spec)
    exp = Expansion(committed, biomes, spec, player, region, ranks=1, slots=slots)
    exp.item = lambda cell: None   # the stand-in engine takes no conditions
    return run(_StandInEngine(slots, forwards, (spec.height, spec.tile, spec.tile)), exp, 0)


def main():
    """python -m streamvoxel_b200.stream.expand [--side0 8 --side1 16] (torchrun for several GPUs): one expansion
    through the real engine; prints one JSON line with committed voxels/s and the admission statistics.
    With `--simulate`: the step counts of the admission alone at 1, 2, 4 and 8 times `--slots` (no GPU)."""
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
    parser.add_argument('--simulate', action='store_true', help='admission step counts only (host, no GPU)')
    args = parser.parse_args()
    if args.simulate:
        spec = ModelSpec.of(sm.small_test_config() if args.small else sm.dit_b4_control())
        base = None
        for gpus in (1, 2, 4, 8):
            st = simulate(args.side0, args.side1, spec, gpus * args.slots)
            base = base or st['forwards']
            print(json.dumps(dict(gpus=gpus, slots=gpus * args.slots, windows=st['windows'], steps=st['forwards'],
                                  empty_slot_rounds=st['blocked_admissions'],
                                  step_bound_speedup=round(base / st['forwards'], 3))))
        return
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
