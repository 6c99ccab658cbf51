"""aubier_b200 -- a B200-native (sm_100a) implementation of jmars/aubier's fused MLA
decode-attention path: the ggml custom ops GGML_OP_M4_WKB, GGML_OP_M4_KQKV and GGML_OP_M4_PHASE.

The product is the C-ABI library ``libm4b.so`` (include/m4b.h); ``aubier_b200.m4`` mirrors the
reference's op API over it for torch-allocated device tensors.  Import ``aubier_b200.m4``
explicitly: it loads the CUDA library and fails loudly when it is missing.
"""

__all__ = ["m4", "build"]
