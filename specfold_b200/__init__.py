"""B200-native (sm_100a) SpecFold folded multi-branch verify forward.

Drop-in replacements for the reference's fused generators
(``SpecFoldTritonFastDLLMV2Generation``, ``SpecFoldTritonNLDGeneration``) backed by
hand-written CUDA kernels behind the C ABI in ``include/specfold_b200.h``.
"""

from .folded import FoldedVerifyB200, SpecFoldB200FastDLLMV2Generation, SpecFoldB200NLDGeneration
from .kv_cache import PreallocatedKVCache

__all__ = ["FoldedVerifyB200", "SpecFoldB200FastDLLMV2Generation", "SpecFoldB200NLDGeneration",
           "PreallocatedKVCache"]
