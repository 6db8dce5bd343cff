"""Worker of the `DeviceExchange` tests: three exchange rounds (nobody finished; rank 1 finished two windows; both
finished one) over a process group of `backend` ('nccl' on GPUs, 'gloo' on CPU). Each rank writes what it received."""
import numpy as np


def exchange_worker(rank, world, port, path, backend):
    import torch
    import torch.distributed as dist
    from streamvoxel_b200.stream.expand import DeviceExchange
    device = torch.device('cpu')
    if backend == 'nccl':
        torch.cuda.set_device(rank)
        device = torch.device('cuda', rank)
    dist.init_process_group(backend, init_method=f'tcp://127.0.0.1:{port}', rank=rank, world_size=world)
    exchange = DeviceExchange(dist.group.WORLD, 4, (8, 4, 4), device)
    rounds = []
    for r in range(3):
        finished = []
        if (r == 1 and rank == 1) or r == 2:
            finished = [((rank, r + j), np.full((8, 4, 4), 10 * rank + r + j, np.int16))
                        for j in range(1 if r == 2 else 2)]
        rounds.append(exchange((finished, 3 - rank)))
    with open(f'{path}.{rank}', 'w') as f:
        f.write(repr([[(len(fin), free, [(c, int(col.sum())) for c, col in fin]) for fin, free in got]
                      for got in rounds]))
    dist.barrier()
    dist.destroy_process_group()


def run_two_ranks(backend):
    """Run the worker on two ranks and return the rounds they agree on (asserts that they agree)."""
    import os
    import tempfile
    import torch.multiprocessing as mp
    port = 29700 + (os.getpid() + (0 if backend == 'nccl' else 500)) % 1000
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, 'x')
        mp.start_processes(exchange_worker, args=(2, port, path, backend), nprocs=2, join=True, start_method='spawn')
        seen = [open(f'{path}.{r}').read() for r in range(2)]
    assert seen[0] == seen[1]
    return eval(seen[0])


def check_rounds(rounds):
    assert rounds[0] == [(0, 3, []), (0, 2, [])]
    assert rounds[1][0] == (0, 3, []) and rounds[1][1][0] == 2 and rounds[1][1][2][0] == ((1, 1), 11 * 128)
    assert rounds[1][1][2][1] == ((1, 2), 12 * 128)
    assert rounds[2][0][2] == [((0, 2), 2 * 128)] and rounds[2][1][2] == [((1, 2), 12 * 128)]
