"""BiasTable -- per-z-bin mean reconstruction bias, subtracted at decode.

Mirrors ``prismkv.quantizer.bias_correction`` (src/prismkv/quantizer/
bias_correction.py:32-181).  In the fused kernels the correction is folded
into the dequant tables (z per bin, (x, y) per code), so ``apply`` is only
a tensor helper.  ``calibrate_bias`` estimates the table offline on a
holdout split, with encode/decode running on the GPU.
"""

from __future__ import annotations

import torch


class BiasTable:
    def __init__(self, table: torch.Tensor, delta_z: float) -> None:
        if table.ndim != 2 or table.shape[1] != 3:
            raise ValueError(f"Expected shape (bins_z, 3), got {tuple(table.shape)}")
        self.table = table.float()
        self.bins_z = table.shape[0]
        self.delta_z = delta_z
        self._clip = delta_z / 2.0

    def apply(self, rotated_q: torch.Tensor, i_z: torch.Tensor, z_idx: torch.Tensor, x_idx: torch.Tensor,
              y_idx: torch.Tensor) -> torch.Tensor:
        """Subtract clamp(table[i_z], +-delta_z/2) from each triplet (z, x, y)."""
        out = rotated_q.clone()
        bias = self.table.to(rotated_q.device)[i_z.long()].clamp(-self._clip, self._clip)
        out[:, z_idx] -= bias[..., 0]
        out[:, x_idx] -= bias[..., 1]
        out[:, y_idx] -= bias[..., 2]
        return out

    def max_abs_bias_per_dim(self) -> float:
        return self.table.abs().max().item()

    def mean_abs_bias(self) -> float:
        return self.table.abs().mean().item()

    def __repr__(self) -> str:
        return (f"BiasTable(bins_z={self.bins_z}, max_abs={self.max_abs_bias_per_dim():.4f}, "
                f"mean_abs={self.mean_abs_bias():.4f})")


def calibrate_bias(quantizer, vectors: torch.Tensor, holdout_fraction: float = 0.2, seed: int = 0) -> BiasTable:
    """Mean (reconstruction - truth) per uniform z-bin and coordinate, on a seeded holdout."""
    n = vectors.shape[0]
    gen = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n, generator=gen)
    hold = vectors[perm[:max(1, int(n * holdout_fraction))]]
    dev = vectors.device if vectors.is_cuda else torch.device("cuda", torch.cuda.current_device())
    hold = hold.to(dev).float()
    R = quantizer.R.to(dev)
    rot = hold @ R.T
    bins = quantizer.bins_z
    dz = (quantizer.z_max - quantizer.z_min) / bins
    z = rot[:, quantizer.z_idx.to(dev)]
    iz = ((z - quantizer.z_min) / dz).floor().long().clamp(0, bins - 1).reshape(-1)
    recon = quantizer.decode(quantizer.encode(hold)).to(dev)
    diff = recon @ R.T - rot
    table = torch.zeros(bins, 3, device=dev)
    counts = torch.bincount(iz, minlength=bins).float()
    for c, idx in enumerate((quantizer.z_idx, quantizer.x_idx, quantizer.y_idx)):
        table[:, c].index_add_(0, iz, diff[:, idx.to(dev)].reshape(-1))
    nz = counts > 0
    table[nz] /= counts[nz, None]
    return BiasTable(table.cpu(), delta_z=dz)
