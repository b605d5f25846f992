"""CacheBackend protocol and PrismKVBackend on the B200 codec.

Same interface as the reference (cache/backend.py:49-233): ``compress(k, v)``
maps (N, head_dim) float rows to (N, padded_dim / 3) int16 codes and
``decompress`` maps them back to float32 (N, head_dim).  Here both run in the
sm_100a encode / decode kernels.  Tensors on the CPU are processed on the
current CUDA device and the results come back to the caller's device, so
code written against the reference's CPU backend keeps working; there is no
CPU fallback.
"""

from __future__ import annotations

import warnings
from typing import Tuple

import torch

from ..quantizer.stacked_plane import StackedPlaneQuantizer, _cuda_device
from .cache_config import PrismKVConfig
from .dim_aligner import DimAligner


class CacheBackend:
    """Protocol: ``compress`` / ``decompress`` on 2-D flat tensors.

    k, v: (N, head_dim) float; k_codes, v_codes: (N, n_groups) int16 with
    n_groups = padded_dim // 3.
    """

    def compress(self, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        raise NotImplementedError

    def decompress(self, k_codes: torch.Tensor, v_codes: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        raise NotImplementedError

    @property
    def config(self) -> PrismKVConfig:
        raise NotImplementedError

    @property
    def head_dim(self) -> int:
        raise NotImplementedError


def make_quantizer(config: PrismKVConfig, padded_dim: int, what: str = "PrismKVBackend") -> StackedPlaneQuantizer:
    """The quantizer of a config, with the reference's codebook fallback rule (backend.py:158-175)."""
    q = StackedPlaneQuantizer(dim=padded_dim, bits_z=config.bits_z, bits_r=config.bits_r,
                              bits_theta=config.bits_theta, seed=config.rotation_seed)
    if config.codebook_path is not None:
        try:
            q.load_codebooks(config.codebook_path)
        except Exception as e:  # noqa: BLE001 -- same policy as the reference
            if not config.fallback_to_uniform:
                raise
            warnings.warn(f"{what}: failed to load codebook '{config.codebook_path}': {e}. "
                          "Falling back to uniform polar quantization.", stacklevel=3)
    return q


class PrismKVBackend(CacheBackend):
    """CacheBackend backed by StackedPlaneQuantizer's device codec.

    config: bit budgets / codebook / seed; head_dim: the model's (unpadded)
    head dimension; device: where returned tensors live when inputs carry no
    device preference ("cpu" as in the reference, or "cuda").
    """

    def __init__(self, config: PrismKVConfig, head_dim: int, device: str = "cpu") -> None:
        self._config = config
        self._device = device
        self._aligner = DimAligner(head_dim)
        self._quantizer = make_quantizer(config, self._aligner.padded_dim)

    @property
    def quantizer(self) -> StackedPlaneQuantizer:
        return self._quantizer

    def codec(self, device=None):
        return self._quantizer.codec(_cuda_device() if device is None else device)

    def compress(self, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(N, head_dim) float -> (N, n_groups) int16 codes on the input's device."""
        dev = _cuda_device(k)
        codec = self._quantizer.codec(dev)
        out = []
        for x in (k, v):
            xd = self._aligner.pad(x.to(dev))
            codes = codec.encode(xd, code_dtype=torch.int16)
            out.append(codes.to(x.device))
        return out[0], out[1]

    def decompress(self, k_codes: torch.Tensor, v_codes: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(N, n_groups) int16 codes -> (N, head_dim) float32 on the codes' device."""
        dev = _cuda_device(k_codes)
        codec = self._quantizer.codec(dev)
        out = []
        for c in (k_codes, v_codes):
            x = codec.decode(c.to(dev))
            out.append(self._aligner.unpad(x).to(c.device))
        return out[0], out[1]

    @property
    def config(self) -> PrismKVConfig:
        return self._config

    @property
    def head_dim(self) -> int:
        return self._aligner.original_dim

    @property
    def padded_dim(self) -> int:
        return self._aligner.padded_dim

    @property
    def n_groups(self) -> int:
        return self._aligner.padded_dim // 3

    @property
    def aligner(self) -> DimAligner:
        return self._aligner

    def __repr__(self) -> str:
        return (f"PrismKVBackend(head_dim={self.head_dim}, padded={self.padded_dim}, "
                f"{self._config.bits_per_dim:.1f}bits/dim, {self._config.compression_vs_fp16:.1f}× vs FP16)")
