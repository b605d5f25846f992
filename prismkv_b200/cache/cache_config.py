"""PrismKVConfig: the per-layer quantization settings of the KV caches.

Same fields, defaults and derived properties as the reference's
``PrismKVConfig`` (cache/cache_config.py:11-48), so configurations written for
the reference construct the same quantizers here.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional


@dataclass
class PrismKVConfig:
    """bits_z / bits_r / bits_theta: bit budgets (16 bins each by default).
    codebook_path: .npz of learned per-z-bin codebooks (None = uniform polar).
    fallback_to_uniform: warn instead of raising when the codebook fails to load.
    rotation_seed: seed of the global rotation (encoder and decoder agree on it)."""

    bits_z: int = 4
    bits_r: int = 4
    bits_theta: int = 4
    codebook_path: Optional[str] = None
    fallback_to_uniform: bool = True
    rotation_seed: int = 42

    @property
    def bits_per_dim(self) -> float:
        return (self.bits_z + self.bits_r + self.bits_theta) / 3

    @property
    def compression_vs_fp16(self) -> float:
        """Theoretical memory reduction vs FP16 storage."""
        return 16 / self.bits_per_dim

    def __repr__(self) -> str:
        return (f"<PrismKVConfig {self.bits_z}+{self.bits_r}+{self.bits_theta} bits per triplet: "
                f"{self.bits_per_dim:.2f} bits/dim, {self.compression_vs_fp16:.2f}x smaller than fp16>")
