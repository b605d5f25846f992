"""LloydMaxQuantizer1D -- non-uniform z bins (boundaries + centroids).

Mirrors ``prismkv.quantizer.lloyd_max.LloydMaxQuantizer1D``
(src/prismkv/quantizer/lloyd_max.py:29-227).  ``encode`` is
``bucketize(z, boundaries[1:-1])`` clamped to [0, K-1] and ``decode`` a
centroid gather; inside the fused encode/decode kernels both become table
lookups built from these arrays.  ``fit`` is the classical Lloyd (1982) /
Max (1960) iteration -- boundaries at centroid midpoints, centroids at the
conditional means -- run offline; the npz keys ``z_boundaries`` /
``z_centroids`` are shared with the reference.
"""

from __future__ import annotations

from pathlib import Path
from typing import Optional

import numpy as np
import torch


class LloydMaxQuantizer1D:
    def __init__(self, K: int, max_iter: int = 100, tol: float = 1e-6):
        if K < 2:
            raise ValueError(f"K must be ≥ 2, got {K}")
        self.K = K
        self.max_iter = max_iter
        self.tol = tol
        self.boundaries: Optional[torch.Tensor] = None   # (K+1,)
        self.centroids: Optional[torch.Tensor] = None    # (K,)
        self.n_iters = 0

    @staticmethod
    def _boundaries(c: torch.Tensor, lo: torch.Tensor, hi: torch.Tensor) -> torch.Tensor:
        # open outer bounds one unit beyond the data, midpoints inside
        return torch.cat([lo - 1.0, (c[:-1] + c[1:]) / 2.0, hi + 1.0])

    def fit(self, z: torch.Tensor) -> "LloydMaxQuantizer1D":
        if z.ndim != 1:
            raise ValueError(f"z must be 1-D, got shape {tuple(z.shape)}")
        if len(z) < self.K:
            raise ValueError(f"Need at least K={self.K} samples, got {len(z)}")
        zs = z.float().cpu().sort().values
        n = zs.numel()
        pos = (torch.linspace(0.0, 1.0, self.K + 2)[1:-1] * (n - 1)).long().clamp(0, n - 1)
        c = zs[pos].clone()
        lo, hi = zs[:1], zs[-1:]
        b = self._boundaries(c, lo, hi)
        csum = torch.cat([torch.zeros(1, dtype=torch.float64), zs.double().cumsum(0)])
        for it in range(self.max_iter):
            # bin k holds z in (b[k], b[k+1]]: index range [searchsorted(b[k], right), searchsorted(b[k+1], right))
            edges = torch.searchsorted(zs, b, right=True)
            cnt = (edges[1:] - edges[:-1])
            sums = csum[edges[1:]] - csum[edges[:-1]]
            mid = (b[:-1] + b[1:]) / 2.0
            newc = torch.where(cnt > 0, (sums / cnt.clamp_min(1)).float(), mid)
            shift = (newc - c).abs().max().item()
            c = newc
            b = self._boundaries(c, lo, hi)
            self.n_iters = it + 1
            if shift < self.tol:
                break
        self.centroids = c
        self.boundaries = b
        return self

    def encode(self, z: torch.Tensor) -> torch.Tensor:
        if self.boundaries is None:
            raise RuntimeError("Call fit() before encode()")
        idx = torch.bucketize(z.float(), self.boundaries[1:-1].to(z.device))
        return idx.long().clamp(0, self.K - 1)

    def decode(self, indices: torch.Tensor) -> torch.Tensor:
        if self.centroids is None:
            raise RuntimeError("Call fit() before decode()")
        return self.centroids.to(indices.device)[indices.long().clamp(0, self.K - 1)]

    def mse(self, z: torch.Tensor) -> float:
        return ((z.float() - self.decode(self.encode(z))) ** 2).mean().item()

    def save(self, path: str | Path) -> None:
        path = Path(path)
        existing = dict(np.load(path)) if path.exists() else {}
        existing["z_boundaries"] = self.boundaries.cpu().numpy()
        existing["z_centroids"] = self.centroids.cpu().numpy()
        np.savez(path, **existing)

    @classmethod
    def load(cls, path: str | Path) -> "LloydMaxQuantizer1D":
        data = np.load(path)
        b = torch.from_numpy(data["z_boundaries"].astype(np.float32))
        c = torch.from_numpy(data["z_centroids"].astype(np.float32))
        obj = cls(K=len(c))
        obj.boundaries, obj.centroids = b, c
        return obj
