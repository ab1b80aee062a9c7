"""B200-native (sm_100a) VMonarch attention: a drop-in for ``video_monarch_attention``.

Exports the reference's three names (reference ``video_monarch_attention/__init__.py:1-4``).
Importing loads the in-tree CUDA library through its C ABI and raises if it is missing.
"""
from .kernel import flash_entropy_attention
from .vmonarch import VMonarchAttention, vmonarch_attention

__all__ = ["VMonarchAttention", "vmonarch_attention", "flash_entropy_attention"]
