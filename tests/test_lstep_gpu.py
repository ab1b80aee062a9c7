"""The Monarch L-step kernels through the C ABI against the oracle's L step (fp32)."""
import pytest
import torch

import oracle
from vmonarch_b200 import ops

pytestmark = pytest.mark.gpu


def inputs(m, b, D, Dv, last, seed):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(2, m * b, D, generator=gen).bfloat16()
    out = torch.randn(2, m * b, D + (Dv if last else 0), generator=gen).bfloat16()
    ent = torch.rand(2, m * b, generator=gen) * 4
    return q, out, ent


def oracle_lstep(q, out, ent, m, b, D, last, scale, mcm):
    qg = q.float().view(1, 2, m, b, D)
    kr = out[..., :D].float().view(1, 2, m, b, D) * scale
    e = ent.view(1, 2, m, b)
    if last:
        y = out[..., D:].float().view(1, 2, m, b, -1)
        return oracle.lstep_forward(qg, kr, e, y=y, min_col_mass=mcm).reshape(2, m * b, -1)
    u, _ = oracle.lstep_forward(qg, kr, e, min_col_mass=mcm, scale=scale)
    return u.reshape(2, m * b, D)


# (21, 1560): 780 column groups, more than the persistent tcgen05 forward keeps resident, so its
# CTAs walk several groups each;
# m in (32, 128]: the four- and eight-warp kernels (one CTA per grid column)
@pytest.mark.parametrize("m, b, D, Dv", [(21, 37, 128, 128), (4, 64, 64, 64), (64, 9, 64, 128), (1, 33, 128, 128),
                                         (32, 16, 128, 128), (21, 1560, 128, 128), (33, 17, 128, 128),
                                         (48, 40, 128, 128), (64, 25, 128, 128), (40, 30, 64, 64),
                                         (65, 12, 128, 128), (100, 20, 128, 128), (128, 9, 64, 64),
                                         (128, 17, 128, 128)])
@pytest.mark.parametrize("last, skip_half", [(False, False), (True, False), (True, True)])
def test_lstep_forward_and_backward(m, b, D, Dv, last, skip_half):
    # D = 128 forwards without skipped tokens run the tcgen05 kernel, the others mma.sync
    scale, mcm = D ** -0.5, 0.3
    q, out, ent = inputs(m, b, D, Dv, last, m * 7 + b)
    qc, oc, ec = q.cuda(), out.cuda(), ent.cuda()
    skip = b // 2 if skip_half else 0
    if last:
        z = torch.zeros(2, m * b, Dv, dtype=torch.bfloat16, device="cuda")
        ops.lstep_fwd(qc, oc, ec, m, b, scale, mcm, z=z, skip_rows=skip)
        got = z.float().cpu()
    else:
        u = torch.empty(2, m * b, D, dtype=torch.bfloat16, device="cuda")
        ops.lstep_fwd(qc, oc, ec, m, b, scale, mcm, u=u)
        got = u.float().cpu()
    ref = oracle_lstep(q, out, ent, m, b, D, last, scale, mcm)
    if last:
        ref[:, :skip] = 0
    assert (got - ref).abs().max() <= 1e-2 * max(1.0, ref.abs().max().item())

    # backward against autograd of the oracle L step
    qr, orr = q.float().requires_grad_(), out.float().requires_grad_()
    y_ref = oracle_lstep(qr, orr, ent, m, b, D, last, scale, mcm)
    gen = torch.Generator().manual_seed(1)
    g = torch.randn(y_ref.shape, generator=gen)
    if last:
        g = g.bfloat16().float()
        g[:, :skip] = 0
    dq_ref, do_ref = torch.autograd.grad((y_ref * g).sum(), (qr, orr))
    dq = torch.zeros(2, m * b, D, device="cuda")
    dout = torch.empty_like(oc)
    if last:
        ops.lstep_bwd(qc, oc, ec, m, b, scale, mcm, dq, dout, dz=g.bfloat16().cuda(), skip_rows=skip)
    else:
        ops.lstep_bwd(qc, oc, ec, m, b, scale, mcm, dq, dout, du=g.cuda())
    torch.cuda.synchronize()
    for a, r in ((dq.cpu(), dq_ref), (dout.float().cpu(), do_ref)):
        assert (a - r).abs().max() <= 1e-2 * max(1.0, r.abs().max().item())
