"""The world-expansion driver (streamvoxel_b200.stream.expand) on CPU with a stand-in engine: admission invariants,
the incremental frontier against `pick_window`, and two gloo ranks keeping identical replicas."""
import os
import tempfile

import numpy as np
import torch.multiprocessing as mp

from streamvoxel_b200.stream import expand, scheduler as sch
from streamvoxel_b200.stream.condition import ModelSpec

SPEC = ModelSpec(height=64, tile=16, num_classes=32, biome_classes=16, biome_halo=4, y_origin=-64.0)


class FakeEngine:
    """Finishes every window after `steps` forwards; the column is a function of the window seed only."""

    def __init__(self, slots, steps=3):
        self.slots, self.steps = slots, steps
        self.left, self.seeds, self.targets = [0] * slots, [0] * slots, [None] * slots
        self.armed = []

    def arm(self, slot, seed, cap, item=None, target=()):
        assert item is not None and self.left[slot] == 0
        self.left[slot], self.seeds[slot], self.targets[slot] = self.steps, seed, target
        self.armed.append((target, len(item.l1_blocks), len(item.l2_blocks)))

    def step(self):
        out = {}
        for i in range(self.slots):
            if self.left[i]:
                self.left[i] -= 1
                done = dict(target=self.targets[i], nfe=self.steps, last_frac=0.0, cap=32, actual=self.steps)
                out[i] = (done if self.left[i] == 0 else None, None)
        return out

    def column(self, i):
        return np.random.default_rng(self.seeds[i]).integers(0, 32, (64, 16, 16)).astype(np.int16)


class PipelinedFakeEngine(FakeEngine):
    """`FakeEngine` with `launch` / `collect` and up to two steps in flight: a window's forwards are counted when
    launched, arming a slot of a step in flight is an error, and a window armed while steps are in flight takes its
    first forward in the next step launched."""
    depth = 2

    def __init__(self, slots, steps=3):
        super().__init__(slots, steps)
        self.to_launch = [0] * slots
        self.queue = []

    @property
    def in_flight(self):
        return len(self.queue)

    def runnable(self):
        return any(self.to_launch)

    def arm(self, slot, seed, cap, item=None, target=(), wait=True):
        assert all(slot not in entry for entry in self.queue)
        super().arm(slot, seed, cap, item, target)
        self.to_launch[slot] = self.steps

    def launch(self):
        assert len(self.queue) < self.depth
        entry = [i for i in range(self.slots) if self.to_launch[i]]
        for i in entry:
            self.to_launch[i] -= 1
        self.queue.append(entry)

    def collect(self):
        out = {}
        for i in self.queue.pop(0):
            self.left[i] -= 1
            done = dict(target=self.targets[i], nfe=self.steps, last_frac=0.0, cap=32, actual=self.steps)
            out[i] = (done if self.left[i] == 0 else None, None)
        return out


class CheckedExpansion(expand.Expansion):
    def admit(self, free):
        before = set(self.committed)
        picks = super().admit(free)
        cells = list(self.inflight)
        for a in cells:   # in-flight windows never touch, and each touches the committed snapshot
            assert sch.separated(a, [c for c in cells if c != a])
            assert any((a[0] + dz, a[1] + dx) in before for dz in (-1, 0, 1) for dx in (-1, 0, 1))
        for r, got in picks.items():
            assert sum(1 for o in self.inflight.values() if o == r) <= self.share[r]
        return picks


def _setup(ranks, slots):
    committed, region, biomes, player = expand.start_region(5, 4, 10, SPEC, classes=32)
    return CheckedExpansion(committed, biomes, SPEC, player, region, ranks=ranks, slots=slots, l2_cap=12)


def test_incremental_pick_equals_pick_window():
    rng = np.random.default_rng(0)
    exp = _setup(1, 4)
    for _ in range(40):
        want = sch.pick_window({c for c in exp.committed}, set(exp.inflight), exp.player)
        got = exp.pick()
        if want is not None and want in exp.region:
            assert got == want
        cell = got
        if cell is None:
            break
        exp.inflight[cell] = 0
        if rng.random() < 0.6:   # finish a random in-flight window
            done = list(exp.inflight)[int(rng.integers(0, len(exp.inflight)))]
            exp.apply([(done, np.zeros((64, 16, 16), np.int16))])


def test_block_counts_agree_with_separated():
    """The in-flight block counts admit exactly the cells `separated` admits (both rules), through assignment, pop
    and del, and `pick` stays the nearest such ready cell."""
    rng = np.random.default_rng(3)
    for diagonal in (False, True):
        committed, region, biomes, player = expand.start_region(5, 4, 10, SPEC, classes=32)
        exp = expand.Expansion(committed, biomes, SPEC, player, region, slots=8, diagonal=diagonal)
        cells = [(z, x) for z in range(-2, 13) for x in range(-2, 13)]
        for _ in range(60):
            cell = cells[int(rng.integers(0, len(cells)))]
            if cell in exp.inflight:
                if rng.random() < 0.5:
                    exp.inflight.pop(cell)
                else:
                    del exp.inflight[cell]
            else:
                exp.inflight[cell] = int(rng.integers(0, 2))
            for c in cells:
                assert (c not in exp.inflight.near) == sch.separated(c, exp.inflight, diagonal=diagonal)
            free = [c for c in exp.ready if sch.separated(c, exp.inflight, diagonal=diagonal)]
            want = min(free, key=lambda c: exp.ready[c]) if free else None
            assert exp.pick() == want
        for cell in list(exp.inflight):
            exp.inflight.pop(cell)
        assert not exp.inflight.near
        try:
            exp.inflight.update({(0, 0): 0})
        except TypeError:
            pass
        else:
            raise AssertionError('update bypasses the block counts')


def _run(ranks, slots, rank=0, group=None):
    exp = _setup(ranks, slots)
    engine = FakeEngine(slots)
    stats = expand.run(engine, exp, rank, group=group)
    return exp, engine, stats


def test_single_rank_expansion_commits_the_region():
    exp, engine, stats = _run(1, 4)
    assert exp.done and not exp.inflight
    assert stats['windows'] == 100 - 16 and len(exp.committed) == 100
    assert all(l1 >= 1 for _, l1, _ in engine.armed)


def test_pipelined_expansion_commits_the_same_world():
    """Admission overlapping the steps in flight (two launched ahead, arming idle slots, collecting the oldest)
    commits every window once and the same columns as the serial driver."""
    serial, _, _ = _run(1, 4)
    exp = _setup(1, 4)
    engine = PipelinedFakeEngine(4)
    stats = expand.run(engine, exp, 0)
    assert stats['pipelined'] and exp.done and not exp.inflight
    assert stats['windows'] == 100 - 16 and exp.digest() == serial.digest()


def _worker(rank, world, port, path):
    import torch.distributed as dist
    dist.init_process_group('gloo', init_method=f'tcp://127.0.0.1:{port}', rank=rank, world_size=world)
    exp, engine, stats = _run(world, 3, rank, dist.group.WORLD)
    with open(f'{path}.{rank}', 'w') as f:
        f.write(f"{exp.digest()} {stats['windows']} {len(exp.committed)}")
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_keep_identical_replicas():
    single, _, _ = _run(1, 6)
    port = 29500 + os.getpid() % 2000
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, 'out')
        mp.start_processes(_worker, args=(2, port, path), nprocs=2, join=True, start_method='spawn')
        rows = [open(f'{path}.{r}').read().split() for r in range(2)]
    assert rows[0][0] == rows[1][0] == single.digest()       # same world as one rank: columns depend on seeds only
    assert int(rows[0][1]) + int(rows[1][1]) == 100 - 16     # every window ran on exactly one rank
    assert int(rows[0][1]) > 0 and int(rows[1][1]) > 0


def test_published_packets_rebuild_the_committed_columns():
    from streamvoxel_b200.stream import wire
    exp = _setup(1, 4)
    pub = wire.Publisher()
    raw_map = np.arange(32, dtype=np.uint16) + 100   # compact id -> global id (air stays 0 only if mapped to 0)
    raw_map[0] = 0
    expand.run(FakeEngine(4), exp, 0, publisher=pub, raw_map=raw_map)
    commits = [p for p in pub.packets if p['kind'] == 'window_commit']
    assert len(commits) == 100 - 16
    for seq, packet in enumerate(pub.packets):
        wire.verify_packet(packet, seq)
    for packet in pub.packets:
        if packet['kind'] != 'frame':
            continue
        row = packet['frames'][0]
        pos, ids = wire.unpack_row(row)
        flat = raw_map[exp.committed[tuple(row['target'])].reshape(-1)]
        np.testing.assert_array_equal(pos, np.flatnonzero(flat))
        np.testing.assert_array_equal(ids, flat[flat != 0])
    assert wire.unbatch(wire.batch_line(pub.packets[:10])) == pub.packets[:10]


def test_device_exchange_two_gloo_ranks():
    """`DeviceExchange`'s rounds (header every round, columns only when some rank finished) on two gloo ranks: the
    same host logic the NCCL group runs on GPUs."""
    from exchange_worker import check_rounds, run_two_ranks
    check_rounds(run_two_ranks('gloo'))


def test_simulated_admission_bounds_the_step_count():
    """`expand.simulate`: the admission alone, every window taking a fixed number of steps -- every window admitted
    once, never fewer steps than the work needs, and more slots never taking more steps."""
    steps = []
    for slots in (2, 4, 8):
        st = expand.simulate(4, 10, SPEC, slots, forwards=5, seed=5)
        assert st['windows'] == 100 - 16
        assert st['forwards'] >= (100 - 16) * 5 / slots
        steps.append(st['forwards'])
    assert steps[0] >= steps[1] >= steps[2]
