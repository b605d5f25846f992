"""Seeded synthetic workloads with the shapes of the benchmark configurations.

No KV data or model weights ship with this project, so every workload is
synthetic: Gaussian K/V (with the per-head scales or outlier channels a
configuration names) encoded with the quantizer into packed codes, and
Gaussian queries.  All draws use explicit ``torch.Generator`` seeds; the
rotation is ``make_rotation(96, 42)`` drawn first (it reseeds the global RNG).

Configurations (head_dim 96 = 32 triplets throughout):
  cpu-roundtrip    B=1,  8/8 heads,   S=1024,   4+4+4 uniform polar, fp32 q
  phi3-decode      B=8,  32/32 heads, S=4096,   4+4+4 uniform polar, bf16 q
  aggressive-332   B=32, 32/32 heads, S=16384,  3+3+2 (uint8 codes), per-head scale U[0.5, 2]
  learned-gqa      B=16, 32/8 heads,  S=32768,  learned 16x256 codebooks + BiasTable, bf16 q;
                   encode workload: 32768 new tokens x 8 KV heads (K and V)
  longctx-splitseq B=4,  32/8 heads,  S=131072, 4+4+4, 1% of channels x8 (outliers)
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Optional, Tuple

import torch

from .quantizer import BiasTable, LearnedSliceCodebook, StackedPlaneQuantizer


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    q_heads: int
    kv_heads: int
    seq_len: int
    bits: Tuple[int, int, int] = (4, 4, 4)
    learned: bool = False
    head_scale: bool = False
    outliers: bool = False
    q_dtype: torch.dtype = torch.bfloat16
    dim: int = 96

    @property
    def m(self) -> int:
        return self.dim // 3

    @property
    def code_bytes(self) -> int:
        return 1 if sum(self.bits) <= 8 else 2

    def scaled(self, **kw) -> "Workload":
        return replace(self, **kw)

    def kv_code_bytes(self) -> int:
        """Packed K + V bytes of the whole workload."""
        return 2 * self.batch * self.kv_heads * self.seq_len * self.m * self.code_bytes

    def decode_bytes(self) -> int:
        """Algorithmic bytes of one decode step: codes once + query + fp32 output."""
        qb = torch.finfo(self.q_dtype).bits // 8
        return self.kv_code_bytes() + self.batch * self.q_heads * self.dim * (qb + 4)


WORKLOADS = {
    "cpu-roundtrip": Workload("cpu-roundtrip", 1, 8, 8, 1024, q_dtype=torch.float32),
    "phi3-decode": Workload("phi3-decode", 8, 32, 32, 4096),
    "aggressive-332": Workload("aggressive-332", 32, 32, 32, 16384, bits=(3, 3, 2), head_scale=True),
    "learned-gqa": Workload("learned-gqa", 16, 32, 8, 32768, learned=True),
    "longctx-splitseq": Workload("longctx-splitseq", 4, 32, 8, 131072, outliers=True),
}


def synthetic_codebook(Cz: int, K: int, r_max: float, seed: int) -> torch.Tensor:
    """(Cz, K, 2) centroids: uniform angle, radius sqrt(U) * 0.6 r_max."""
    g = torch.Generator().manual_seed(seed)
    ang = (torch.rand(Cz, K, generator=g) * 2 - 1) * math.pi
    rad = torch.sqrt(torch.rand(Cz, K, generator=g)) * r_max * 0.6
    return torch.stack([rad * torch.cos(ang), rad * torch.sin(ang)], dim=-1).float()


def synthetic_bias(Cz: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(Cz, 3, generator=g) * 0.05).float()


def make_quantizer(w: Workload, seed: int = 42) -> StackedPlaneQuantizer:
    q = StackedPlaneQuantizer(w.dim, *w.bits, seed=seed)
    if w.learned:
        Cz, K = 1 << w.bits[0], 1 << (w.bits[1] + w.bits[2])
        q._codebooks = LearnedSliceCodebook(synthetic_codebook(Cz, K, q.r_max, 11), Cz, K,
                                            q.z_min, q.z_max, q.r_max)
        q._bias = BiasTable(synthetic_bias(Cz, 12), delta_z=(q.z_max - q.z_min) / Cz)
    return q


def _kv_rows(w: Workload, g: torch.Generator, device, rows: int, head_of_row: torch.Tensor,
             scales: Optional[torch.Tensor], outlier_ch: Optional[torch.Tensor]) -> torch.Tensor:
    x = torch.randn(rows, w.dim, generator=g, device=device)
    if scales is not None:
        x *= scales[head_of_row].unsqueeze(1)
    if outlier_ch is not None:
        x[:, outlier_ch] *= 8.0
    return x


def _workload_layout(w: Workload, device) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
    """The per-KV-head scales and the outlier channels of a workload (fixed across seeds)."""
    gh = torch.Generator().manual_seed(1)
    scales = (0.5 + 1.5 * torch.rand(w.kv_heads, generator=gh)).to(device) if w.head_scale else None
    outlier = None
    if w.outliers:
        n_out = max(1, round(0.01 * w.dim))
        outlier = torch.randperm(w.dim, generator=gh)[:n_out].to(device)
    return scales, outlier


def make_kv_codes(w: Workload, quantizer: StackedPlaneQuantizer, device, seed: int = 0,
                  chunk_rows: int = 1 << 21) -> Tuple[torch.Tensor, torch.Tensor]:
    """(B, Hkv, S, m) packed K and V codes: Gaussian vectors encoded on the GPU in chunks.

    ``seed`` draws the vectors.  The per-head scales and the outlier channels are a
    property of the workload, fixed across seeds, so that shards drawn with different
    seeds on different ranks belong to one cache.
    """
    device = torch.device(device)
    g = torch.Generator(device=device).manual_seed(seed)
    scales, outlier = _workload_layout(w, device)
    codec = quantizer.codec(device)
    shape = (w.batch, w.kv_heads, w.seq_len, w.m)
    dt = quantizer.code_dtype
    out = []
    total = w.batch * w.kv_heads * w.seq_len
    for _ in range(2):
        codes = torch.empty(shape, dtype=dt, device=device)
        flat = codes.view(total, w.m)
        for s in range(0, total, chunk_rows):
            n = min(chunk_rows, total - s)
            head = (torch.arange(s, s + n, device=device) // w.seq_len) % w.kv_heads
            x = _kv_rows(w, g, device, n, head, scales, outlier)
            codec.encode(x, out=flat[s:s + n])
        out.append(codes)
    return out[0], out[1]


def make_query(w: Workload, device, seed: int = 1) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(w.batch, w.q_heads, w.dim, generator=g, device=device).to(w.q_dtype)


def make_encode_input(w: Workload, device, tokens: int = 32768, seed: int = 2,
                      dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """New K and V vectors of one layer: (2 * tokens * kv_heads, dim)."""
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(2 * tokens * w.kv_heads, w.dim, generator=g, device=device).to(dtype)
