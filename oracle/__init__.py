"""CPU fp32 oracle for the VMonarch hot path — TEST INFRASTRUCTURE, never the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
this package, and only as the checker or the timed CPU baseline. The product path
(``vmonarch_b200``) never imports it and has no CPU fallback.

Contents
  fea.py       entropy attention in fp32 (reference tests/test_vmonarch.py:12-15, the semantics
               of video_monarch_attention/kernel.py:32-151)
  vmonarch.py  VMonarch alternating minimisation + recompute in fp32
               (reference video_monarch_attention/vmonarch.py:19-69 with the R step patched to the
               dense fp32 entropy attention, exactly as tests/test_vmonarch.py:55-62 does)

Pinning: the restatement is checked against the reference itself (imported on CPU with the same
patch) by ``tests/golden/make_golden.py``, which wrote the committed fixtures in
``tests/golden/``; ``tests/test_oracle.py`` re-checks the oracle against those fixtures.
Gradients come from torch autograd on the fp32 graph, as in the reference's own tests.
"""
from .fea import entropy_attention, entropy_attention_rows
from .vmonarch import vmonarch_attention, lstep_forward

__all__ = ["entropy_attention", "entropy_attention_rows", "vmonarch_attention", "lstep_forward"]
