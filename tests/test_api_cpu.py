"""Host-side behaviour of the drop-in API that needs no GPU: the reference's assertion errors."""
import pytest
import torch

import vmonarch_b200 as vmb
from vmonarch_b200 import VMonarchAttention, flash_entropy_attention, vmonarch_attention


def test_exports_match_reference():
    assert set(vmb.__all__) == {"VMonarchAttention", "vmonarch_attention", "flash_entropy_attention"}


def test_fea_rejects_fp32_like_the_reference():
    q = torch.randn(1, 1, 16, 64)
    with pytest.raises(AssertionError, match="unsupported dtype"):
        flash_entropy_attention(q, q, q)


def test_fea_rejects_shape_mismatch_and_bad_dims():
    q = torch.randn(1, 1, 16, 64, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        flash_entropy_attention(q, q[..., :32, :], q)
    with pytest.raises(AssertionError):
        flash_entropy_attention(q, q, torch.randn(1, 1, 16, 96, dtype=torch.bfloat16))


def test_fea_needs_cuda_tensors():
    q = torch.randn(1, 1, 16, 64, dtype=torch.bfloat16)
    with pytest.raises(AssertionError, match="CUDA"):
        flash_entropy_attention(q, q, q)


def test_vmonarch_argument_errors():
    q = torch.randn(1, 1, 64, 64, dtype=torch.bfloat16)
    with pytest.raises(AssertionError, match="N=64 != 3 \\* 32"):
        vmonarch_attention(q, q, q, 3, 32)
    with pytest.raises(UnboundLocalError):
        vmonarch_attention(q, q, q, 2, 32, num_iters=0)
    with pytest.raises(AssertionError, match="CUDA"):
        vmonarch_attention(q, q, q, 2, 32)


def test_module_repr_and_defaults():
    m = VMonarchAttention(16, 256)
    assert m.num_iters == 2 and m.min_col_mass == 0.01
    assert m.extra_repr() == "num_blocks=16, block_size=256, num_iters=2"
    assert list(m.parameters()) == []
