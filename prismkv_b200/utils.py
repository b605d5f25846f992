"""Rotation utility (mirrors src/prismkv/utils.py:9-28 of the reference).

The rotation is the quantizer's key: encoder and decoder agree on it by
(dim, seed).  It is generated on the host exactly as the reference does --
seed the global torch RNG, draw a Gaussian matrix, take Q of its QR
factorisation -- so that codes written by either implementation decode in
the other.  Like the reference, this reseeds torch's global RNG.
"""

from __future__ import annotations

import torch


def make_rotation(dim: int, seed: int = 42) -> torch.Tensor:
    """(dim, dim) orthogonal matrix Q with Q @ Q.T == I, deterministic in (dim, seed)."""
    torch.manual_seed(seed)
    g = torch.randn(dim, dim)
    q, _ = torch.linalg.qr(g)
    return q
