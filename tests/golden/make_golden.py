"""Generate the golden fixtures in tests/golden/ from the REFERENCE implementation itself.

Run in a container where the reference checkout is importable (it is not needed afterwards):

    python tests/golden/make_golden.py --reference /path/to/VMonarch

For each case the script
  1. draws bf16-representable inputs from a seeded CPU generator,
  2. runs the reference's own CPU fp32 path on them — ``entropy_attention_ref`` from the
     reference's tests/test_vmonarch.py:12-15 for FlashEntropyAttention, and the reference's
     ``vmonarch_attention`` (video_monarch_attention/vmonarch.py:29-69) with
     ``_row_block_attention`` patched to that dense fp32 function exactly as
     tests/test_vmonarch.py:55-59 does — and differentiates it with torch autograd,
  3. runs this repository's oracle (``oracle/``) on the same inputs and asserts agreement,
  4. stores inputs (as bf16 bit patterns) and the reference outputs / gradients (fp32) in one
     ``.npz`` per case.
The reference's Triton kernels need a GPU and are not run here.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent

FEA_CASES = [
    # name, B, H, N, D, Dv, seed
    ("fea_n130_d64", 1, 1, 130, 64, 64, 1),
    ("fea_n72_d128_dv256", 1, 1, 72, 128, 256, 2),
    ("fea_n136_d64_dv128", 1, 1, 136, 64, 128, 3),
]
VM_CASES = [
    # name, B, H, m, b, D, iters, recompute, seed
    ("vm_m4_b64_it2_r64", 1, 1, 4, 64, 64, 2, 64, 4),
    ("vm_m3_b40_it3_r40", 1, 1, 3, 40, 64, 3, 40, 5),
    ("vm_m5_b24_it1_r0", 1, 1, 5, 24, 64, 1, 0, 6),
]


def bf16_round(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, str(Path(args.reference) / "tests"))
    sys.path.insert(0, str(ROOT))
    import test_vmonarch as ref_tests                      # reference tests/test_vmonarch.py
    import video_monarch_attention.vmonarch as ref_vm      # reference vmonarch.py
    import oracle

    def ref_row_block(x, k, w):                             # tests/test_vmonarch.py:55-57
        out, ent = ref_tests.entropy_attention_ref(x, k, w, 1.0)
        return out, -ent.detach()

    ref_vm._row_block_attention = ref_row_block

    for name, B, H, N, D, Dv, seed in FEA_CASES:
        g = torch.Generator().manual_seed(seed)
        q, k = bf16_round(torch.randn(B, H, N, D, generator=g)), bf16_round(torch.randn(B, H, N, D, generator=g))
        v = bf16_round(torch.randn(B, H, N, Dv, generator=g))
        do, de = torch.randn(B, H, N, Dv, generator=g), torch.randn(B, H, N, generator=g)
        do = bf16_round(do)
        scale = D ** -0.5
        leaves = [t.clone().requires_grad_() for t in (q, k, v)]
        o, e = ref_tests.entropy_attention_ref(*leaves, scale)
        grads = torch.autograd.grad((o * do).sum() + (e * de).sum(), leaves)
        leaves2 = [t.clone().requires_grad_() for t in (q, k, v)]
        o2, e2 = oracle.entropy_attention(*leaves2, scale)
        grads2 = torch.autograd.grad((o2 * do).sum() + (e2 * de).sum(), leaves2)
        for a_, b_ in zip((o, e, *grads), (o2, e2, *grads2)):
            assert torch.allclose(a_, b_, rtol=1e-5, atol=1e-5), f"{name}: oracle disagrees with reference"
        np.savez_compressed(HERE / f"{name}.npz", q=bf16_bits(q), k=bf16_bits(k), v=bf16_bits(v), do=bf16_bits(do),
                            de=de.numpy(), o=o.detach().numpy(), e=e.detach().numpy(),
                            dq=grads[0].numpy(), dk=grads[1].numpy(), dv=grads[2].numpy(),
                            meta=np.array([B, H, N, D, Dv, seed]))
        print("wrote", name)

    for name, B, H, m, b, D, iters, r, seed in VM_CASES:
        N = m * b
        g = torch.Generator().manual_seed(seed)
        q, k, v = (bf16_round(torch.randn(B, H, N, D, generator=g)) for _ in range(3))
        dz = bf16_round(torch.randn(B, H, N, D, generator=g))
        leaves = [t.clone().requires_grad_() for t in (q, k, v)]
        z = ref_vm.vmonarch_attention(*leaves, m, b, iters, recompute_tokens=r)
        grads = torch.autograd.grad((z * dz).sum(), leaves)
        leaves2 = [t.clone().requires_grad_() for t in (q, k, v)]
        z2 = oracle.vmonarch_attention(*leaves2, m, b, iters, recompute_tokens=r)
        grads2 = torch.autograd.grad((z2 * dz).sum(), leaves2)
        for a_, b_ in zip((z, *grads), (z2, *grads2)):
            err = (a_ - b_).abs().max().item()
            assert err <= 1e-4 * max(1.0, a_.abs().max().item()), f"{name}: oracle disagrees with reference ({err})"
        np.savez_compressed(HERE / f"{name}.npz", q=bf16_bits(q), k=bf16_bits(k), v=bf16_bits(v), dz=bf16_bits(dz),
                            z=z.detach().numpy(), dq=grads[0].numpy(), dk=grads[1].numpy(), dv=grads[2].numpy(),
                            meta=np.array([B, H, m, b, D, iters, r, seed]))
        print("wrote", name)


if __name__ == "__main__":
    main()
