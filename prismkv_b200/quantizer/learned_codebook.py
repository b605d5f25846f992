"""LearnedSliceCodebook -- per-z-bin (x, y) centroid tables (the learned path).

Mirrors ``prismkv.quantizer.learned_codebook.LearnedSliceCodebook``
(src/prismkv/quantizer/learned_codebook.py:115-339): a (bins_z, K, 2) fp32
table plus the ranges it was trained with, saved as the ``prismkv-cb-v1``
npz format (same keys, so files move between the two implementations).

The encode hot path does not call ``encode_xy``: ``pkv_encode`` searches the
table of bin ``i_z`` inside the fused encode kernel.  ``encode_xy`` /
``decode_xy`` are kept as tensor helpers on whatever device the inputs are.
Training a codebook (the reference's offline k-means) is not part of this
path: tables are trained once, saved, and loaded here.
"""

from __future__ import annotations

from pathlib import Path
from typing import Optional, Tuple

import numpy as np
import torch


class LearnedSliceCodebook:
    FILE_VERSION = "prismkv-cb-v1"

    def __init__(self, codebooks: torch.Tensor, bins_z: int, K: int, z_min: float, z_max: float,
                 r_max: float) -> None:
        if tuple(codebooks.shape) != (bins_z, K, 2):
            raise ValueError(f"Expected codebooks shape ({bins_z}, {K}, 2), got {tuple(codebooks.shape)}")
        self.codebooks = codebooks.float()
        self.bins_z = bins_z
        self.K = K
        self.z_min = z_min
        self.z_max = z_max
        self.r_max = r_max

    def encode_xy(self, xy: torch.Tensor, i_z: torch.Tensor) -> torch.Tensor:
        """(N, m, 2) points, (N, m) bins -> index of the nearest centroid of each point's bin."""
        cb = self.codebooks.to(xy.device)[i_z.long()]                  # (N, m, K, 2)
        d2 = ((xy.float().unsqueeze(-2) - cb) ** 2).sum(-1)
        return d2.argmin(dim=-1)

    def decode_xy(self, i_flat: torch.Tensor, i_z: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        xy = self.codebooks.to(i_flat.device)[i_z.long(), i_flat.long()]
        return xy[..., 0], xy[..., 1]

    def save(self, path: str | Path, metadata: Optional[dict] = None) -> None:
        arrays = {"codebooks": self.codebooks.detach().cpu().numpy(), "z_min": np.float32(self.z_min),
                  "z_max": np.float32(self.z_max), "r_max": np.float32(self.r_max),
                  "bins_z": np.int32(self.bins_z), "K": np.int32(self.K),
                  "version": np.bytes_(self.FILE_VERSION)}
        for k, v in (metadata or {}).items():
            arrays[f"meta_{k}"] = np.array(v)
        np.savez(str(path), **arrays)

    @classmethod
    def load(cls, path: str | Path) -> "LearnedSliceCodebook":
        data = np.load(str(path), allow_pickle=False)
        version = data["version"].item()
        if hasattr(version, "decode"):
            version = version.decode()
        if version != cls.FILE_VERSION:
            raise ValueError(f"Unsupported codebook version '{version}'. Expected '{cls.FILE_VERSION}'.")
        return cls(torch.from_numpy(data["codebooks"].copy()), bins_z=int(data["bins_z"]), K=int(data["K"]),
                   z_min=float(data["z_min"]), z_max=float(data["z_max"]), r_max=float(data["r_max"]))

    def centroid_radii(self) -> torch.Tensor:
        return torch.sqrt(self.codebooks[..., 0] ** 2 + self.codebooks[..., 1] ** 2)

    def __repr__(self) -> str:
        return (f"<LearnedSliceCodebook {self.bins_z} z-bins x {self.K} centroids, "
                f"z in [{self.z_min:.2f}, {self.z_max:.2f}], r <= {self.r_max:.2f}>")
