"""The pipeline-timeout path of the tcgen05 forward kernels, exercised without a fault.

Every mbarrier wait of these kernels is bounded; a CTA whose wait runs out records a code in the
kernel's error word, tells its other roles to stop, drains what it has in flight, frees its tensor
memory and exits. vmb_test_pipeline_timeout shortens the limit and holds the loads (a barrier that
nothing completes), so the first waits run out; the test checks that vmb_device_status reports the
code and that the next calls on the same GPU compute correct results again."""
import pytest
import torch

from vmonarch_b200 import _native as N
from vmonarch_b200 import flash_entropy_attention

pytestmark = pytest.mark.gpu


def test_pipeline_timeout_is_reported_and_the_gpu_recovers():
    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(17)
    q, k, v = (torch.randn(1, 2, 300, 128, generator=gen).bfloat16().to(dev) for _ in range(3))
    ref = [flash_entropy_attention(q, k, v), flash_entropy_attention(q, k, k)]
    torch.cuda.synchronize()
    assert N.device_status(dev) == 0
    N.check(N.lib.vmb_test_pipeline_timeout(20000, 1), "vmb_test_pipeline_timeout")
    try:
        flash_entropy_attention(q, k, v)   # separate values: two-query-tile kernel
        flash_entropy_attention(q, k, k)   # values aliasing keys: one-stream kernel
        torch.cuda.synchronize()
        status = N.device_status(dev)
    finally:
        N.check(N.lib.vmb_test_pipeline_timeout(0, 0), "vmb_test_pipeline_timeout")
    assert status & 0xff != 0  # forward kernels' codes in the low byte
    # the context is intact: the same calls give the same results again, with no code recorded
    again = [flash_entropy_attention(q, k, v), flash_entropy_attention(q, k, k)]
    torch.cuda.synchronize()
    assert N.device_status(dev) == 0
    for (o, e), (o_r, e_r) in zip(again, ref):
        assert torch.equal(o, o_r) and torch.equal(e, e_r)


def test_hold_needs_a_short_limit():
    assert N.lib.vmb_test_pipeline_timeout(0, 1) == 1
    assert N.lib.vmb_test_pipeline_timeout(10 ** 9, 1) == 1
    assert N.lib.vmb_test_pipeline_timeout(0, 0) == 0
