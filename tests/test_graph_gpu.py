"""CUDA-graph capture of the product path: the C-ABI entry points launch on torch's current stream,
make no host synchronisation and take their workspaces from torch's allocator, so a whole
forward + backward can be captured once and replayed on new input values. The replay is checked
against an eager call on the same values and against the fp32 oracle."""
import pytest
import torch

import oracle
from conftest import max_rel_err
from vmonarch_b200 import flash_entropy_attention, vmonarch_attention

pytestmark = pytest.mark.gpu


def _capture(step, statics):
    """Warm `step` up on a side stream (the pattern torch documents for whole-network capture),
    then capture it; returns the graph and the outputs it writes on every replay."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step(*statics)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = step(*statics)
    return g, outs


def _vm_step(m, b, iters, r):
    def step(q, k, v, dz):
        z = vmonarch_attention(q, k, v, m, b, iters, recompute_tokens=r)
        return (z, *torch.autograd.grad((z.float() * dz).sum(), (q, k, v)))
    return step


@pytest.mark.parametrize("m, b, iters, r", [(4, 256, 2, 256), (3, 200, 3, 150)])
def test_vmonarch_forward_backward_replays_in_a_cuda_graph(m, b, iters, r):
    B, H, D = 1, 2, 128
    N = m * b
    q, k, v = (torch.zeros(B, H, N, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
               for _ in range(3))
    dz = torch.zeros(B, H, N, D, device="cuda")
    gen = torch.Generator().manual_seed(41)
    with torch.no_grad():
        for t in (q, k, v, dz):
            t.copy_(torch.randn(t.shape, generator=gen))
    step = _vm_step(m, b, iters, r)
    g, outs = _capture(step, (q, k, v, dz))
    for seed in (42, 43):  # new values through the same graph
        gen = torch.Generator().manual_seed(seed)
        vals = [torch.randn(B, H, N, D, generator=gen) for _ in range(4)]
        vals = [t.bfloat16().float() for t in vals[:3]] + [vals[3]]
        with torch.no_grad():
            for t, x in zip((q, k, v, dz), vals):
                t.copy_(x)
        g.replay()
        torch.cuda.synchronize()
        got = [t.detach().float().cpu() for t in outs]
        leaves = [x.cuda().bfloat16().requires_grad_() for x in vals[:3]]
        eager = [t.detach().float().cpu() for t in step(*leaves, vals[3].cuda())]
        for a, e in zip(got, eager):  # fp32 reductions may add in another order: not bitwise
            assert max_rel_err(a, e) <= 1e-2
        ref_leaves = [x.clone().requires_grad_() for x in vals[:3]]
        z_r = oracle.vmonarch_attention(*ref_leaves, m, b, iters, recompute_tokens=r)
        ref = [z_r.detach(), *torch.autograd.grad((z_r * vals[3]).sum(), ref_leaves)]
        assert max_rel_err(got[0], ref[0]) <= 3e-2
        for a, e in zip(got[1:], ref[1:]):
            assert max_rel_err(a, e) <= 5e-2


def test_flash_entropy_attention_replays_in_a_cuda_graph():
    # two sequences of 2100 keys: the forward splits the key range (workspace taken from torch's
    # allocator inside the capture) and the backward runs its tcgen05 kernels
    B, H, N, D = 1, 2, 2100, 128
    q, k, v = (torch.zeros(B, H, N, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
               for _ in range(3))
    do, de = torch.zeros(B, H, N, D, device="cuda"), torch.zeros(B, H, N, device="cuda")

    def step(q, k, v, do, de):
        o, e = flash_entropy_attention(q, k, v)
        return (o, e, *torch.autograd.grad((o.float() * do).sum() + (e * de).sum(), (q, k, v)))

    g, outs = _capture(step, (q, k, v, do, de))
    gen = torch.Generator().manual_seed(44)
    vals = [torch.randn(B, H, N, D, generator=gen).bfloat16().float() for _ in range(3)]
    vals += [torch.randn(B, H, N, D, generator=gen), torch.randn(B, H, N, generator=gen)]
    with torch.no_grad():
        for t, x in zip((q, k, v, do, de), vals):
            t.copy_(x)
    g.replay()
    torch.cuda.synchronize()
    got = [t.detach().float().cpu() for t in outs]
    leaves = [x.clone().requires_grad_() for x in vals[:3]]
    o_r, e_r = oracle.entropy_attention(*leaves, D ** -0.5)
    ref = [o_r.detach(), e_r.detach(), *torch.autograd.grad((o_r * vals[3]).sum() + (e_r * vals[4]).sum(), leaves)]
    assert max_rel_err(got[0], ref[0]) <= 2e-2 and max_rel_err(got[1], ref[1]) <= 2e-2
    for a, e in zip(got[2:], ref[2:]):
        assert max_rel_err(a, e) <= 3e-2


def test_bench_graph_mode_line():
    # bench.py --graph: the timed steps are replays of one captured step; the line says so, and its
    # launch count (kernels per replay x timed steps) equals the eager run's count over the same
    # timed steps (warm-up excluded)
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    lines = {}
    for graph in (False, True):
        cmd = [sys.executable, os.path.join(root, "bench.py"), "--workload", "readme", "--steps", "3", "--warmup", "4",
               "--no-e2e", "--no-cpu-baseline"] + (["--graph"] if graph else [])
        out = subprocess.run(cmd, cwd=root, capture_output=True, text=True, timeout=600, check=True).stdout
        lines[graph] = json.loads([x for x in out.splitlines() if x.startswith("{")][-1])
    assert lines[True]["config"]["cuda_graph"] is True and lines[False]["config"]["cuda_graph"] is False
    assert lines[True]["value"] > 0 and lines[False]["value"] > 0
    assert lines[True]["gpu_launches"] == lines[False]["gpu_launches"] > 0
    assert lines[True]["gpu_launches"] % 3 == 0
    assert "not flushed" in lines[True]["config"]["l2"]
