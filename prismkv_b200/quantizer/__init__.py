from .stacked_plane import StackedPlaneQuantizer
from .learned_codebook import LearnedSliceCodebook
from .bias_correction import BiasTable, calibrate_bias
from .lloyd_max import LloydMaxQuantizer1D
from .polar_attention import (PolarAttentionApprox, polar_dot_product, polar_dot_product_from_codes,
                              decode_attention, measure_polar_approx_error)

__all__ = ["StackedPlaneQuantizer", "LearnedSliceCodebook", "BiasTable", "calibrate_bias",
           "LloydMaxQuantizer1D", "PolarAttentionApprox", "polar_dot_product",
           "polar_dot_product_from_codes", "decode_attention", "measure_polar_approx_error"]
