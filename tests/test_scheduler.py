"""Window admission and the batch split (streamvoxel_b200.stream.scheduler) against fixtures made by the reference
scheduler (`tests/golden/make_golden.py --only scheduler`), plus the properties its own tests state."""
import os

import numpy as np

from streamvoxel_b200.stream import scheduler as sch
from streamvoxel_b200.stream.condition import ModelSpec

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')


def _g():
    return np.load(os.path.join(GOLDEN, 'scheduler.npz'))


def _cells(a):
    return {(int(z), int(x)) for z, x in a.reshape(-1, 2)}


def test_pick_window_matches_reference():
    g = _g()
    for i in range(80):
        got = sch.pick_window(_cells(g[f'p{i}_committed']), _cells(g[f'p{i}_inflight']),
                              tuple(float(v) for v in g[f'p{i}_player']), diagonal=bool(g[f'p{i}_diagonal']))
        want = tuple(int(v) for v in g[f'p{i}_pick'])
        assert (got if got is not None else (-(2 ** 40), -(2 ** 40))) == want, i


def test_member_shares_match_reference():
    g = _g()
    for i in range(60):
        members = [tuple(int(v) for v in m) for m in g[f'm{i}_members'].reshape(-1, 3)]
        got = sch.member_shares(int(g[f'm{i}_batch']), members)
        assert [got[w] for w, _, _ in members] == list(g[f'm{i}_shares']), i


def test_window_seeds_match_reference():
    g = _g()
    for (z, x), want in zip(g['seed_cells'], g['seed_values']):
        assert sch.window_seed(7, int(z), int(x)) == int(want)


def test_make_item_matches_reference():
    g = _g()
    spec = ModelSpec(height=64, tile=16, num_classes=32, biome_classes=16, biome_halo=4, y_origin=-64.0)
    for i in range(6):
        cells = {tuple(int(v) for v in c): t for c, t in zip(g[f'i{i}_cells'], g[f'i{i}_tiles'])}
        item = sch.make_item(cells, tuple(int(v) for v in g[f'i{i}_target']), g['biomes'], spec, 7, 32, 5)
        for name in ('l1_blocks', 'l1_xz', 'l2_blocks', 'l2_xz', 'biomes'):
            np.testing.assert_array_equal(getattr(item, name), g[f'i{i}_{name}'], err_msg=f'{i} {name}')
        assert item.seed == int(g[f'i{i}_seed'])


def test_admission_properties():
    # separation rules (Chebyshev >= gap; Manhattan >= 2 with diagonal)
    assert sch.separated((0, 0), [])
    assert not sch.separated((0, 0), [(1, 1)]) and sch.separated((0, 0), [(1, 1)], diagonal=True)
    assert not sch.separated((0, 0), [(0, 1)], diagonal=True) and sch.separated((0, 0), [(0, 3)], gap=3)
    # nearest first, ties on (z, x); a blocked frontier gives None
    assert sch.pick_window({(0, 0)}, set(), (8., 40.)) == (0, 1)
    assert sch.pick_window({(0, 0)}, {(0, 1), (-1, -1), (1, -1)}, (8., 8.)) is None
    assert sch.pick_window(set(), set(), (0., 0.)) is None
    # slot refill policies and the equal split
    assert sch.plan_inserts([3, 5, 6], 7, 8, 'dynamic') == [3] and sch.plan_inserts([0, 1, 2], 1, 2, 'fixed') == []
    for batch in range(20):
        for ranks in (1, 2, 3):
            shares = [sch.rank_share(batch, ranks, r) for r in range(ranks)]
            assert sum(shares) == batch and shares == sorted(shares, reverse=True)
            assert [sch.member_shares(batch, [(r, 99, 1) for r in range(ranks)])[r] for r in range(ranks)] == shares


def test_fast_item_equals_make_item():
    """The expansion driver's item (`fast_item`: L2 cells by a growing square, L2 tiles stacked lazily) is the
    reference rule's item (`make_item`) field for field, on random committed blobs and targets."""
    from streamvoxel_b200.stream.condition import ModelSpec
    from streamvoxel_b200.stream.scheduler import fast_item, make_item, ready_cells
    spec = ModelSpec(height=16, tile=16, num_classes=8, biome_classes=16, biome_halo=4, y_origin=-64.0)
    rng = np.random.default_rng(3)
    biomes = rng.integers(0, 16, (4, 66, 66)).astype(np.int64)
    for case in range(40):
        cells, z, x = set(), 0, 0
        for _ in range(int(rng.integers(1, 200))):
            cells.add((z, x))
            dz, dx = ((1, 0), (-1, 0), (0, 1), (0, -1))[int(rng.integers(0, 4))]
            z, x = z + dz, x + dx
        snapshot = {c: rng.integers(0, 9, (16, 16, 16)).astype(np.int16) for c in cells}
        frontier = sorted(ready_cells(cells))
        target = frontier[int(rng.integers(0, len(frontier)))]
        cap = int(rng.choice([1, 5, 12, 81]))
        want = make_item(snapshot, target, biomes, spec, 7, 32, cap)
        got = fast_item(snapshot, target, biomes, spec, 7, 32, cap)
        assert got.l2_keys == want.l2_keys and got.seed == want.seed and got.id == want.id
        for name in ('l1_blocks', 'l1_xz', 'l2_xz', 'biomes'):
            assert np.array_equal(getattr(got, name), getattr(want, name)), (case, name)
        assert np.array_equal(np.asarray(got.l2_blocks), want.l2_blocks) and len(got.l2_blocks) == len(want.l2_blocks)
        pick = [i for i in range(len(want.l2_blocks)) if i % 2]
        assert np.array_equal(got.l2_blocks[pick], want.l2_blocks[pick])
