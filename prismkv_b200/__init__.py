"""prismkv_b200 -- PrismKV's quantized-KV hot path, native on B200 (sm_100a).

Drop-in for the ``prismkv`` Python API on that path (quantizer encode/decode,
polar attention, the KV-cache and vLLM offload adapters), backed by
hand-written CUDA kernels behind the C ABI in include/prismkv_b200.h.
"""

from .quantizer import (StackedPlaneQuantizer, LearnedSliceCodebook, BiasTable, LloydMaxQuantizer1D,  # noqa: F401
                        PolarAttentionApprox, calibrate_bias, decode_attention)
from .utils import make_rotation  # noqa: F401

__version__ = "0.1.0"
__all__ = ["StackedPlaneQuantizer", "LearnedSliceCodebook", "BiasTable", "LloydMaxQuantizer1D",
           "PolarAttentionApprox", "calibrate_bias", "decode_attention", "make_rotation"]
