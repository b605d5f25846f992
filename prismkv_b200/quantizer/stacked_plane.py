"""StackedPlaneQuantizer -- the reference API over the sm_100a kernels.

Mirrors ``prismkv.quantizer.stacked_plane.StackedPlaneQuantizer``
(src/prismkv/quantizer/stacked_plane.py:38-430): same constructor, state
attributes, ``encode`` -> (N, m) int64 and ``decode`` -> (N, dim) fp32.
Behind it, ``encode`` / ``decode`` run ``pkv_encode`` / ``pkv_decode`` on the
GPU.  Tensors on the CPU are copied to the current CUDA device and the
result copied back; there is no CPU implementation, and without a CUDA
device every call raises.

Device tables are (re)built from the quantizer state -- ranges, rotation,
learned codebooks, Lloyd-Max boundaries, BiasTable -- whenever that state
changes, and cached per device.
"""

from __future__ import annotations

import math
from pathlib import Path
from typing import Dict, Optional, Tuple

import numpy as np
import torch

from ..codec import DeviceCodec, code_dtype_for
from ..tables import build_host_tables
from ..utils import make_rotation
from .bias_correction import BiasTable, calibrate_bias
from .learned_codebook import LearnedSliceCodebook
from .lloyd_max import LloydMaxQuantizer1D


def _cuda_device(t: Optional[torch.Tensor] = None) -> torch.device:
    if t is not None and t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("PrismKV B200 kernels need a CUDA device (there is no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


class StackedPlaneQuantizer:
    """3-D stacked-plane KV quantizer (rotation, z bins, polar or learned (x, y) bins).

    Parameters follow stacked_plane.py:58-108: ``dim`` (multiple of 3), bit
    widths per component, rotation ``seed`` and optional ranges (default
    +-sqrt(dim)).
    """

    def __init__(self, dim: int, bits_z: int = 4, bits_r: int = 4, bits_theta: int = 4,
                 seed: int = 42, z_min: float | None = None, z_max: float | None = None,
                 r_max: float | None = None):
        if dim % 3 != 0:
            raise ValueError(
                f"dim must be divisible by 3 for StackedPlaneQuantizer, got {dim}. "
                f"Hint: use dim=192, 384, 768, etc.")
        self._setup(dim, bits_z, bits_r, bits_theta, make_rotation(dim, seed), z_min, z_max, r_max)

    @classmethod
    def from_rotation(cls, R: torch.Tensor, bits_z: int = 4, bits_r: int = 4, bits_theta: int = 4,
                      z_min: float | None = None, z_max: float | None = None,
                      r_max: float | None = None) -> "StackedPlaneQuantizer":
        """Quantizer with an explicit rotation (no RNG reseeding)."""
        dim = R.shape[0]
        if dim % 3 != 0 or tuple(R.shape) != (dim, dim):
            raise ValueError(f"R must be square with a side divisible by 3, got {tuple(R.shape)}")
        obj = cls.__new__(cls)
        obj._setup(dim, bits_z, bits_r, bits_theta, R.detach().float().cpu(), z_min, z_max, r_max)
        return obj

    def _setup(self, dim, bits_z, bits_r, bits_theta, R, z_min, z_max, r_max):
        for name, b in (("bits_z", bits_z), ("bits_r", bits_r), ("bits_theta", bits_theta)):
            if not (1 <= int(b) <= 8):
                raise ValueError(f"{name} must be in 1..8, got {b}")
        if bits_z + bits_r + bits_theta > 16:
            raise ValueError("bits_z + bits_r + bits_theta must be <= 16")
        self.dim = dim
        self.bits_z = bits_z
        self.bits_r = bits_r
        self.bits_theta = bits_theta
        self.m = dim // 3
        self.bins_z = 2 ** bits_z
        self.bins_r = 2 ** bits_r
        self.bins_theta = 2 ** bits_theta
        self.R = R
        k = torch.arange(self.m)
        self.z_idx = 3 * k
        self.x_idx = 3 * k + 1
        self.y_idx = 3 * k + 2
        conservative = math.sqrt(dim)
        self.z_min = z_min if z_min is not None else -conservative
        self.z_max = z_max if z_max is not None else conservative
        self.r_max = r_max if r_max is not None else conservative
        self._codebooks: Optional[LearnedSliceCodebook] = None
        self._bias: Optional[BiasTable] = None
        self._lloyd_max_z: Optional[LloydMaxQuantizer1D] = None
        self._dev_cache: Dict[Tuple, DeviceCodec] = {}

    # ------------------------------------------------------------------
    @property
    def R_inv(self) -> torch.Tensor:
        return self.R.T

    def _state_key(self):
        cb = self._codebooks
        bt = self._bias
        lm = self._lloyd_max_z
        return (float(self.z_min), float(self.z_max), float(self.r_max), id(self.R), self.R._version,
                id(cb), None if cb is None else (id(cb.codebooks), cb.codebooks._version),
                id(bt), None if bt is None else (id(bt.table), bt.table._version, bt.delta_z),
                id(lm), None if lm is None or lm.boundaries is None else
                (id(lm.boundaries), lm.boundaries._version, id(lm.centroids), lm.centroids._version))

    def codec(self, device: Optional[torch.device] = None) -> DeviceCodec:
        """Device tables for the current state (cached per device and state)."""
        dev = _cuda_device() if device is None else torch.device(device)
        if dev.type != "cuda":
            raise RuntimeError("PrismKV B200 kernels need a CUDA device (there is no CPU fallback)")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        key = (dev.index,) + self._state_key()
        c = self._dev_cache.get(key)
        if c is None:
            lm = self._lloyd_max_z
            host = build_host_tables(
                self.dim, self.bits_z, self.bits_r, self.bits_theta,
                self.R.detach().float().cpu().numpy(), self.z_min, self.z_max, self.r_max,
                codebook=None if self._codebooks is None else self._codebooks.codebooks.detach().float().cpu().numpy(),
                lloyd_boundaries=None if lm is None else lm.boundaries.detach().float().cpu().numpy(),
                lloyd_centroids=None if lm is None else lm.centroids.detach().float().cpu().numpy(),
                bias_table=None if self._bias is None else self._bias.table.detach().float().cpu().numpy(),
                bias_delta_z=None if self._bias is None else self._bias.delta_z)
            c = DeviceCodec(host, dev)
            self._dev_cache = {k: v for k, v in self._dev_cache.items() if k[0] != dev.index}
            self._dev_cache[key] = c
        return c

    @property
    def code_dtype(self) -> torch.dtype:
        return code_dtype_for(self.bits_z + self.bits_r + self.bits_theta)

    # ------------------------------------------------------------------
    def calibrate(self, vectors: torch.Tensor, percentile_clip: float = 0.0) -> None:
        """Tighten z/r ranges from sample vectors (stacked_plane.py:114-154; offline)."""
        dev = _cuda_device(vectors)
        rot = vectors.to(dev).float() @ self.R.to(dev).T
        z = rot[:, self.z_idx.to(dev)].reshape(-1)
        x = rot[:, self.x_idx.to(dev)]
        y = rot[:, self.y_idx.to(dev)]
        radii = torch.sqrt(x ** 2 + y ** 2).reshape(-1)
        if percentile_clip > 0.0:
            self.z_min = torch.quantile(z, percentile_clip).item()
            self.z_max = torch.quantile(z, 1.0 - percentile_clip).item()
            self.r_max = torch.quantile(radii, 1.0 - percentile_clip).item()
        else:
            self.z_min = z.min().item()
            self.z_max = z.max().item()
            self.r_max = radii.max().item()

    def calibrate_lloyd_max_z(self, vectors: torch.Tensor) -> None:
        """Fit Lloyd-Max z boundaries on sample vectors (stacked_plane.py:156-177; offline)."""
        dev = _cuda_device(vectors)
        rot = vectors.to(dev).float() @ self.R.to(dev).T
        z = rot[:, self.z_idx.to(dev)].reshape(-1).float().cpu()
        self._lloyd_max_z = LloydMaxQuantizer1D(K=self.bins_z).fit(z)

    def load_codebooks(self, path: str | Path | None) -> None:
        """Load learned per-z-bin codebooks (stacked_plane.py:183-204); None reverts to polar bins."""
        if path is None:
            self._codebooks = None
            return
        cb = LearnedSliceCodebook.load(path)
        self.z_min, self.z_max, self.r_max = cb.z_min, cb.z_max, cb.r_max
        self._codebooks = cb

    def save_lloyd_max_z(self, path: str | Path) -> None:
        if self._lloyd_max_z is None:
            raise RuntimeError("Call calibrate_lloyd_max_z() first.")
        self._lloyd_max_z.save(path)

    def load_lloyd_max_z(self, path: str | Path) -> None:
        self._lloyd_max_z = LloydMaxQuantizer1D.load(path)

    def calibrate_bias(self, vectors: torch.Tensor, holdout_fraction: float = 0.2, seed: int = 0) -> None:
        self._bias = calibrate_bias(quantizer=self, vectors=vectors, holdout_fraction=holdout_fraction, seed=seed)

    # ------------------------------------------------------------------
    def encode_compact(self, vectors: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Codes in compact storage (uint8 for <= 8 bits, else int16) on the vectors' CUDA device."""
        dev = _cuda_device(vectors)
        return self.codec(dev).encode(vectors.to(dev), out=out)

    def encode(self, vectors: torch.Tensor) -> torch.Tensor:
        """(N, dim) vectors -> (N, m) int64 codes (stacked_plane.py:210-262)."""
        if vectors.dim() != 2 or vectors.shape[1] != self.dim:
            raise ValueError(f"expected (N, {self.dim}) vectors, got {tuple(vectors.shape)}")
        dev = _cuda_device(vectors)
        x = vectors.to(dev)
        if x.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            x = x.float()
        codes = self.codec(dev).encode(x, code_dtype=torch.int64)
        return codes if vectors.is_cuda else codes.cpu()

    def decode(self, codes: torch.Tensor) -> torch.Tensor:
        """(N, m) codes -> (N, dim) fp32 vectors (stacked_plane.py:268-327)."""
        if codes.dim() != 2 or codes.shape[1] != self.m:
            raise ValueError(f"expected (N, {self.m}) codes, got {tuple(codes.shape)}")
        dev = _cuda_device(codes)
        out = self.codec(dev).decode(codes.to(dev))
        return out if codes.is_cuda else out.cpu()

    # ------------------------------------------------------------------
    def bits_per_dim(self) -> float:
        return (self.bits_z + self.bits_r + self.bits_theta) / 3

    def compression_vs_fp32(self) -> float:
        return 32 / self.bits_per_dim()

    def error_bound(self) -> float:
        """Worst-case per-triplet Euclidean error of the uniform bins (stacked_plane.py:404-422)."""
        delta_r = self.r_max / max(self.bins_r - 1, 1)
        delta_theta = 2 * math.pi / max(self.bins_theta - 1, 1)
        delta_z = (self.z_max - self.z_min) / self.bins_z
        return math.sqrt((delta_r / 2) ** 2 + (self.r_max * delta_theta / 2) ** 2 + (delta_z / 2) ** 2)

    def __repr__(self) -> str:
        return (f"StackedPlaneQuantizer(dim={self.dim}, bits_z={self.bits_z}, bits_r={self.bits_r}, "
                f"bits_theta={self.bits_theta}, {self.bits_per_dim():.1f} bits/dim, "
                f"{self.compression_vs_fp32():.1f}x vs FP32)")
