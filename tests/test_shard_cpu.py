"""Head sharding over 2 gloo ranks on CPU: contiguous unit split, verification gather and the
max-over-ranks timing reduction give the same result as one process."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from vmonarch_b200 import shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, k, v, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    info = shard.init("gloo", timeout_s=60)
    units = shard.unit_range(q.shape[0], info.rank, info.world)
    o, e = oracle.entropy_attention(q[units.start:units.stop], k[units.start:units.stop],
                                    v[units.start:units.stop], 0.125)
    full = shard.gather_units(o, q.shape[0], info.world)
    t = shard.max_over_ranks(float(rank + 1), torch.device("cpu"))
    if rank == 0:
        # numpy, pickled by value: a tensor would be shared through a file descriptor that dies with
        # this process, which may exit before the parent reads the queue
        out_q.put((full.numpy(), t))
    shard.barrier()
    dist.destroy_process_group()


def test_unit_range_partitions():
    for n in (1, 5, 40, 41):
        for w in (1, 2, 3, 8):
            got = [i for r in range(w) for i in shard.unit_range(n, r, w)]
            assert got == list(range(n))


def test_two_rank_gloo_shard_and_gather():
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(5, 40, 64, generator=g) for _ in range(3))
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    full, t = out_q.get(timeout=120)
    full = torch.from_numpy(full)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ref, _ = oracle.entropy_attention(q, k, v, 0.125)
    torch.testing.assert_close(full, ref)
    assert t == 2.0
