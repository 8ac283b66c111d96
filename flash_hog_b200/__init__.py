"""flash_hog_b200 -- Flash Hog's attention hot path (forward, backward,
double backward) as hand-written sm_100a kernels behind a C ABI.

Public API (mirrors ``flash_hog.jax``):
  * ``dot_product_attention`` -- differentiable twice (``flash_hog/jax/attention.py:19``);
  * ``flash_bwdbwd`` -- the double-backward rule on its own (``flash_hog/jax/_pallas_gpu.py:51``);
  * ``dot_product_attention_varlen`` -- packed variable-length sequences (cu_seqlens);
  * ``MaskType``, ``SlidingWindow``, ``PackedSequences``, ``TuningConfig``.
"""

from flash_hog_b200._attention_impl import MaskType, PackedSequences, SlidingWindow
from flash_hog_b200.attention import dot_product_attention, dot_product_attention_varlen
from flash_hog_b200.bwdbwd import TuningConfig, flash_bwdbwd

__all__ = ["dot_product_attention", "dot_product_attention_varlen", "flash_bwdbwd", "MaskType", "PackedSequences",
           "SlidingWindow", "TuningConfig"]
__version__ = "0.1.0"
