"""prismkv_b200.cuda -- the reference's ``prismkv.cuda`` entry points on sm_100a.

Mirrors src/prismkv/cuda/__init__.py:15-61: ``CUDA_AVAILABLE`` and
``polar_attn_fwd``.  The reference silently falls back to torch when its
extension is missing (:61, :64-92); here a missing library or device raises.
``polar_attn_decode`` is the fused dequant + flash-decoding entry point.
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _lib
from ..codec import polar_scores

CUDA_AVAILABLE = _lib.available()


def polar_attn_fwd(Q: torch.Tensor, K_codes: torch.Tensor, z_min: float, delta_z: float, r_max: float,
                   delta_r: float, delta_theta: float, scale: float, bits_z: int, bits_r: int,
                   bits_theta: int) -> torch.Tensor:
    """scale * <Q, dequant(K)> from int16 codes; Q (B, H, Sq, d) already rotated by R.

    Returns (B, H, Sq, Sk) fp32 on Q's device (CPU inputs are computed on the
    current CUDA device and copied back).
    """
    dev = Q.device if Q.is_cuda else torch.device("cuda", torch.cuda.current_device())
    if not torch.cuda.is_available():
        raise RuntimeError("polar_attn_fwd needs a CUDA device (the B200 build has no CPU fallback)")
    out = polar_scores(Q.to(dev), K_codes.to(dev), [z_min, delta_z, r_max, delta_r, delta_theta, scale],
                       [bits_z, bits_r, bits_theta])
    return out if Q.is_cuda else out.cpu()


def polar_attn_decode(quantizer, q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor,
                      scale: Optional[float] = None, seq_lens: Optional[torch.Tensor] = None,
                      num_splits: int = 0) -> torch.Tensor:
    """Fused decode attention over packed K/V codes -> (B, Hq, d) fp32 (see pkv_attn_decode)."""
    return quantizer.codec(q.device).attention(q, k_codes, v_codes, scale=scale, seq_lens=seq_lens,
                                               num_splits=num_splits)


__all__ = ["CUDA_AVAILABLE", "polar_attn_fwd", "polar_attn_decode"]
