"""Attention directly from PrismKV codes.

Mirrors ``prismkv.quantizer.polar_attention`` (src/prismkv/quantizer/
polar_attention.py:66-362).  The polar identity
``q_z k_z + q_r k_r cos(q_theta - k_theta) = q_z k_z + q_x k_x + q_y k_y``
means scores from codes equal dot products with the dequantized keys, so
the kernels compute them in Cartesian rotated space:

* ``polar_dot_product_from_codes`` / ``PolarAttentionApprox.attention_scores``
  -> ``pkv_polar_scores`` (dense (B, H, Sq, Sk) logits);
* ``PolarAttentionApprox.forward_codes`` and ``decode_attention`` ->
  ``pkv_attn_decode``, the fused dequant + flash-decoding kernel for one
  query token, with V given as codes and the rotation undone once per output.

``forward`` keeps the reference signature (decoded ``v``, optional additive
mask, weights returned): scores come from the kernel, softmax and the
weighted sum from torch on the same device.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from ..codec import polar_scores


def polar_dot_product(q: torch.Tensor, k_z: torch.Tensor, k_r: torch.Tensor, k_theta: torch.Tensor) -> torch.Tensor:
    """Dot product of Cartesian q with keys given as (z, r, theta) per triplet (polar_attention.py:66-110)."""
    m = k_z.shape[-1]
    qt = q[..., : 3 * m].reshape(*q.shape[:-1], m, 3)
    qz, qx, qy = qt[..., 0], qt[..., 1], qt[..., 2]
    return (qz * k_z + k_r * (qx * torch.cos(k_theta) + qy * torch.sin(k_theta))).sum(dim=-1)


def _params(bits_z, bits_r, bits_theta, z_min, z_max, r_max):
    Cz = 1 << bits_z
    delta_z = (z_max - z_min) / Cz
    return [z_min, delta_z, r_max, r_max / max((1 << bits_r) - 1, 1),
            2.0 * math.pi / max((1 << bits_theta) - 1, 1)]


def polar_dot_product_from_codes(q: torch.Tensor, k_codes: torch.Tensor, bits_z: int, bits_r: int,
                                 bits_theta: int, z_min: float, z_max: float, r_max: float,
                                 R: Optional[torch.Tensor] = None) -> torch.Tensor:
    """(B, H, Sq, d) queries x (B, H, Sk, m) uniform-polar codes -> (B, H, Sq, Sk) dot products.

    With ``R`` the query is first rotated into the codes' space (q @ R^T).
    """
    if not q.is_cuda:
        raise RuntimeError("polar_dot_product_from_codes needs CUDA tensors (no CPU fallback)")
    if R is not None:
        B, H, Sq, d = q.shape
        q = (q.reshape(-1, d).float() @ R.T.to(q.device, torch.float32)).reshape(B, H, Sq, d)
    qp = _params(bits_z, bits_r, bits_theta, z_min, z_max, r_max) + [1.0]
    return polar_scores(q, k_codes.to(q.device), qp, (bits_z, bits_r, bits_theta))


class PolarAttentionApprox:
    """Scaled dot-product attention with keys given as PrismKV codes (polar_attention.py:219-309)."""

    def __init__(self, bits_z: int = 4, bits_r: int = 4, bits_theta: int = 4, z_min: float = -4.0,
                 z_max: float = 4.0, r_max: float = 4.0, scale: Optional[float] = None,
                 R: Optional[torch.Tensor] = None) -> None:
        self.bits_z, self.bits_r, self.bits_theta = bits_z, bits_r, bits_theta
        self.z_min, self.z_max, self.r_max = z_min, z_max, r_max
        self._scale = scale
        self.R = R
        self._quantizer = None

    def attention_scores(self, q: torch.Tensor, k_codes: torch.Tensor) -> torch.Tensor:
        return polar_dot_product_from_codes(q, k_codes, self.bits_z, self.bits_r, self.bits_theta,
                                            self.z_min, self.z_max, self.r_max, R=self.R)

    def forward(self, q: torch.Tensor, k_codes: torch.Tensor, v: torch.Tensor,
                attn_mask: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """softmax(scores * scale + mask) @ v; returns (output, weights)."""
        d = q.shape[-1]
        scale = self._scale or (d ** -0.5)
        scores = self.attention_scores(q, k_codes) * scale
        if attn_mask is not None:
            scores = scores + attn_mask.to(scores.device)
        weights = F.softmax(scores, dim=-1)
        return torch.matmul(weights, v.to(weights.device, weights.dtype)), weights

    def _codec(self, device):
        """Uniform-polar device tables matching this object's ranges and rotation."""
        from .stacked_plane import StackedPlaneQuantizer
        if self.R is None:
            raise RuntimeError("forward_codes needs the quantizer rotation R")
        key = (id(self.R), self.R._version, self.z_min, self.z_max, self.r_max,
               self.bits_z, self.bits_r, self.bits_theta)
        if self._quantizer is None or self._quantizer[0] != key:
            qz = StackedPlaneQuantizer.from_rotation(self.R, self.bits_z, self.bits_r, self.bits_theta,
                                                     z_min=self.z_min, z_max=self.z_max, r_max=self.r_max)
            self._quantizer = (key, qz)
        return self._quantizer[1].codec(device)

    def forward_codes(self, q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor,
                      seq_lens: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Fused decode attention for one query token with K and V as codes.

        q (B, Hq, 1, d); codes (B, Hkv, Sk, m) uint8/int16.  Returns (B, Hq, 1, d) fp32.
        """
        d = q.shape[-1]
        scale = self._scale or (d ** -0.5)
        out = self._codec(q.device).attention(q, k_codes, v_codes, scale=scale, seq_lens=seq_lens)
        return out.unsqueeze(2)


def decode_attention(quantizer, q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor,
                     scale: Optional[float] = None, seq_lens: Optional[torch.Tensor] = None,
                     out: Optional[torch.Tensor] = None, num_splits: int = 0) -> torch.Tensor:
    """Fused dequant + flash-decoding attention for any quantizer state (v1, learned, Lloyd-Max, bias).

    q (B, Hq, d) or (B, Hq, 1, d); k/v codes (B, Hkv, S, m) in compact
    storage (uint8 / int16) on the same CUDA device; grouped query heads
    share KV head h // (Hq // Hkv).  Returns (B, Hq, d) fp32.
    """
    return quantizer.codec(q.device).attention(q, k_codes, v_codes, scale=scale, seq_lens=seq_lens, out=out,
                                               num_splits=num_splits)


def measure_polar_approx_error(q, k, k_codes, bits_z, bits_r, bits_theta, z_min, z_max, r_max, R=None) -> dict:
    """Exact dot products vs scores from codes (polar_attention.py:316-362)."""
    exact = torch.matmul(q, k.transpose(-2, -1))
    approx = polar_dot_product_from_codes(q, k_codes, bits_z, bits_r, bits_theta, z_min, z_max, r_max, R=R)
    diff = (exact - approx).abs()
    cos = F.cosine_similarity(exact.flatten(0, -2), approx.flatten(0, -2), dim=-1).mean().item()
    return {"mean_abs_error": diff.mean().item(), "max_abs_error": diff.max().item(),
            "relative_error": (diff / (exact.abs() + 1e-8)).mean().item(), "cosine_sim": cos}
