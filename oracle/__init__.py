"""CPU oracle for the PrismKV hot path -- test infrastructure only.

Imported solely by ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs
of ``bench.py``.  The product package ``prismkv_b200`` never imports it.
"""
from .prismkv_oracle import (QuantParams, encode, decode, dequant_rotated, rotate,  # noqa: F401
                             attention, polar_scores, lse_combine, encode_rotated,
                             polar_attention_forward_f32, bin_z, bin_r, bin_theta)
from .ties import classify, TieReport  # noqa: F401
