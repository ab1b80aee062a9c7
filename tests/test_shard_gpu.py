"""Head sharding over 2 NCCL ranks on 2 GPUs: each rank runs VMonarch forward + backward on its
contiguous block of (batch, head) units with no collective in between, the verification gather
rebuilds the full outputs, and they agree with one GPU running every unit. Skipped with < 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

M, BS, D, ITERS, R = 4, 256, 128, 2, 256


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _units(n=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(n, M * BS, D, generator=g).to(torch.bfloat16) for _ in range(3))
    do = torch.randn(n, M * BS, D, generator=g).to(torch.bfloat16)
    return q, k, v, do


def _run(q, k, v, do, device):
    import vmonarch_b200 as api
    q, k, v = (t.to(device).unsqueeze(0).requires_grad_() for t in (q, k, v))
    z = api.vmonarch_attention(q, k, v, M, BS, ITERS, recompute_tokens=R)
    z.backward(do.to(device).unsqueeze(0))
    return [t.squeeze(0) for t in (z.detach(), q.grad, k.grad, v.grad)]


def _worker(rank, world, port, q, k, v, do, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from vmonarch_b200 import shard
    torch.cuda.set_device(rank)
    info = shard.init("nccl", timeout_s=60)
    device = torch.device("cuda", rank)
    units = shard.unit_range(q.shape[0], info.rank, info.world)
    sl = slice(units.start, units.stop)
    outs = _run(q[sl], k[sl], v[sl], do[sl], device)
    torch.cuda.synchronize(device)
    full = [shard.gather_units(t, q.shape[0], info.world).float().cpu() for t in outs]
    if rank == 0:
        out_q.put([t.numpy() for t in full])  # by value: this process may exit before the parent reads
    shard.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_nccl_head_shard_matches_one_gpu():
    q, k, v, do = _units()
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, do, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    full = [torch.from_numpy(t) for t in out_q.get(timeout=300)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ref = [t.cpu() for t in _run(q, k, v, do, torch.device("cuda", 0))]
    for name, got, want in zip(("z", "dq", "dk", "dv"), full, ref):
        assert got.shape == want.shape, name
        err = (got.float() - want.float()).abs().max().item()
        assert err <= 1e-2 * want.float().abs().max().item() + 1e-3, (name, err)
