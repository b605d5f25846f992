"""Zero-padding of head dimensions that are not a multiple of 3.

Mirrors the reference's ``DimAligner`` (cache/dim_aligner.py:19-48): d=64 is
padded to 66 with zero columns before encoding and the padding is sliced off
after decoding.  The padding runs on whatever device holds the tensor.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


class DimAligner:
    def __init__(self, original_dim: int) -> None:
        self.original_dim = original_dim
        self.pad_width = (3 - original_dim % 3) % 3
        self.padded_dim = original_dim + self.pad_width

    def pad(self, x: torch.Tensor) -> torch.Tensor:
        """Append ``pad_width`` zero columns to the last dimension."""
        return x if self.pad_width == 0 else F.pad(x, (0, self.pad_width))

    def unpad(self, x: torch.Tensor) -> torch.Tensor:
        """Strip the columns added by ``pad``."""
        return x if self.pad_width == 0 else x[..., : self.original_dim]

    def __repr__(self) -> str:
        return (f"<DimAligner {self.original_dim} -> {self.padded_dim} dims "
                f"({self.pad_width} zero pad)>")
