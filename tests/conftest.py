import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test: no tcgen05 pipeline wait may have timed out (vmb_device_status)."""
    yield
    if "gpu" in request.keywords and torch.cuda.is_available():
        from vmonarch_b200 import _native
        assert _native.device_status(torch.device("cuda", torch.cuda.current_device())) == 0


def load_golden(name: str) -> dict:
    """Fixture arrays; bf16 bit patterns (uint16) are decoded to fp32 tensors."""
    data = np.load(GOLDEN / f"{name}.npz")
    out = {}
    for key in data.files:
        arr = data[key]
        if arr.dtype == np.uint16:
            out[key] = torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16).float()
        else:
            out[key] = torch.from_numpy(arr.copy())
    return out


FEA_GOLDEN = ["fea_n130_d64", "fea_n72_d128_dv256", "fea_n136_d64_dv128"]
VM_GOLDEN = ["vm_m4_b64_it2_r64", "vm_m3_b40_it3_r40", "vm_m5_b24_it1_r0"]


def max_rel_err(x: torch.Tensor, ref: torch.Tensor) -> float:
    """max |x - ref| / max |ref|: the reference tests' tolerance convention (tests/test_vmonarch.py:22-24).
    The denominator is floored at 1e-3: an all-zero reference (e.g. every gradient of a one-key
    softmax) is compared in absolute terms instead of dividing fp32 rounding noise by zero."""
    return ((x.float() - ref.float()).abs().max() / ref.float().abs().max().clamp_min(1e-3)).item()
