"""The world-expansion driver through the real engine (small model): windows conditioned on committed columns via
`make_item`, sampled by the whole-step graph, committed and re-admitted until the region is full."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_small_expansion_through_the_engine():
    from streamvoxel_b200 import model as sm
    from streamvoxel_b200.stream import expand
    from streamvoxel_b200.stream.batch import SlotBatch
    from streamvoxel_b200.stream.condition import ModelSpec
    from streamvoxel_b200.stream.fast_ops import FastSlotForward
    cfg = sm.small_test_config()
    spec = ModelSpec.of(cfg)
    forward = FastSlotForward((cfg, sm.synthetic_state_dict(cfg, seed=0)), spec, 'cuda', 4, 8, 24)
    engine = SlotBatch(forward)
    committed, region, biomes, player = expand.start_region(3, 2, 4, spec, classes=cfg.classes)
    exp = expand.Expansion(committed, biomes, spec, player, region, slots=4, l2_cap=24)
    stats = expand.run(engine, exp, 0)
    assert exp.done and stats['windows'] == 12 and len(exp.committed) == 16
    for cell in region - set(committed):
        col = exp.committed[cell]
        assert col.shape == (spec.height, spec.tile, spec.tile)
        assert col.min() >= 0 and col.max() < cfg.classes   # no mask id left: every voxel committed
    assert stats['forwards'] > 0 and stats['blocked_admissions'] >= 0


def test_l2_token_cache_gives_identical_keys_and_values():
    import torch
    from streamvoxel_b200 import model as sm
    from streamvoxel_b200.model import L2TokenCache, PreparedModel
    from streamvoxel_b200.stream import expand
    from streamvoxel_b200.stream.condition import ModelSpec
    cfg = sm.small_test_config()
    spec = ModelSpec.of(cfg)
    model = PreparedModel(cfg, sm.synthetic_state_dict(cfg, seed=0), 'cuda')
    committed, region, biomes, player = expand.start_region(3, 4, 6, spec, classes=cfg.classes)
    exp = expand.Expansion(committed, biomes, spec, player, region, slots=4, l2_cap=12)
    cache = L2TokenCache()
    for cell in sorted(exp.ready)[:3]:
        item = exp.item(cell)
        args = (item.l1_blocks, item.l1_xz, item.l2_blocks, item.l2_xz, item.biomes)
        plain = model.encode_item(*args)
        cached = model.encode_item(*args, l2_keys=item.l2_keys, cache=cache)
        for (k0, v0), (k1, v1) in zip(plain, cached):
            assert torch.equal(k0, k1) and torch.equal(v0, v1)
    assert cache.hits > 0 and cache.misses <= len(committed)


def _exchange_worker(rank, world, port, path):
    import torch
    import torch.distributed as dist
    from streamvoxel_b200.stream.expand import DeviceExchange
    torch.cuda.set_device(rank)
    dist.init_process_group('nccl', init_method=f'tcp://127.0.0.1:{port}', rank=rank, world_size=world)
    exchange = DeviceExchange(dist.group.WORLD, 4, (8, 4, 4), torch.device('cuda', rank))
    rounds = []
    for r in range(3):   # round 0: nobody finished; round 1: rank 1 finishes two windows; round 2: both finish one
        finished = []
        if (r == 1 and rank == 1) or r == 2:
            finished = [((rank, r + j), np.full((8, 4, 4), 10 * rank + r + j, np.int16)) for j in range(1 if r == 2 else 2)]
        rounds.append(exchange((finished, 3 - rank)))
    with open(f'{path}.{rank}', 'w') as f:
        f.write(repr([[(len(fin), free, [(c, int(col.sum())) for c, col in fin]) for fin, free in got] for got in rounds]))
    dist.barrier()
    dist.destroy_process_group()


def test_device_exchange_two_ranks():
    """`DeviceExchange` (finished columns and free-slot counts all-gathered over NCCL) gives every rank the same
    rounds, including rounds where nobody or only one rank finished."""
    import tempfile
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two GPUs')
    port = 29700 + os.getpid() % 1000
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, 'x')
        mp.start_processes(_exchange_worker, args=(2, port, path), nprocs=2, join=True, start_method='spawn')
        seen = [open(f'{path}.{r}').read() for r in range(2)]
    assert seen[0] == seen[1]
    rounds = eval(seen[0])
    assert rounds[0] == [(0, 3, []), (0, 2, [])]
    assert rounds[1][0] == (0, 3, []) and rounds[1][1][0] == 2 and rounds[1][1][2][0] == ((1, 1), 11 * 128)
    assert rounds[2][0][2] == [((0, 2), 2 * 128)] and rounds[2][1][2] == [((1, 2), 12 * 128)]
