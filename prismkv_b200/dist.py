"""Multi-GPU decode over packed KV codes: one process per GPU, ``torch.distributed``.

Two partitionings of the decode-attention path:

* **Sequence shards** (split-sequence decode for long contexts).  Rank r holds
  tokens ``shard_range(S, N, r)`` of every (batch, kv head).  Each rank runs
  the fused kernel in partial mode, giving rotated-space softmax partials
  ``[m, l, o]`` (natural-log max, weight sum, unnormalised output) per
  (batch, q head).  One all-gather exchanges them (NCCL over NVLink; 4 B x
  (dim + 2) per row and rank), and every rank merges them with
  ``pkv_lse_combine``, which also applies ``R`` once.  The merge is the
  log-sum-exp rule ``o = sum_i e^(m_i - M) o_i / sum_i e^(m_i - M) l_i``.
* **Batch shards.**  Rank r holds batch rows ``shard_range(B, N, r)``; the
  ranks share nothing and no collective runs.

The query is replicated on every rank (a decode step's query is tiny).  The
reference has no multi-GPU path: it decodes on one CPU (polar_attention.py
:277-309); sequence sharding is the decomposition of that same softmax.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous share [start, stop) of n items for `rank`; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_partials(partials: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather (rows, dim + 2) partials from every rank -> (world, rows, dim + 2).

    NCCL gathers into one contiguous buffer; other backends (gloo, for CPU
    tests) gather a list.  Every rank must call it, in the same order.
    """
    partials = partials.contiguous()
    world = dist.get_world_size(group)
    if world == 1:
        return partials.unsqueeze(0)
    out = torch.empty((world,) + tuple(partials.shape), dtype=partials.dtype, device=partials.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, partials, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), partials, group=group)
    return out


def split_sequence_decode(quantizer, q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor,
                          scale: Optional[float] = None, group=None,
                          out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode attention with the sequence sharded over the ranks of `group`.

    q: (B, Hq, dim), identical on every rank.  k_codes / v_codes: this rank's
    (B, Hkv, S_r, m) token shard (S_r may be 0).  Returns (B, Hq, dim) fp32,
    the attention over the concatenation of all ranks' shards in rank order.
    """
    if q.dim() == 4:
        q = q[:, :, 0, :]
    codec = quantizer.codec(q.device)
    B, Hq, D = q.shape
    part = codec.attention(q, k_codes, v_codes, scale=scale, partial=True)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        parts = gather_partials(part.view(B * Hq, D + 2), group)
    else:
        parts = part.view(1, B * Hq, D + 2)
    res = codec.combine(parts, out=None if out is None else out.view(B * Hq, D))
    return res.view(B, Hq, D)


def batch_shard_decode(quantizer, q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor,
                       scale: Optional[float] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode attention of this rank's batch rows (no exchange): q (B_r, Hq, dim), codes (B_r, ...)."""
    return quantizer.codec(q.device).attention(q, k_codes, v_codes, scale=scale, out=out)


__all__ = ["shard_range", "gather_partials", "split_sequence_decode", "batch_shard_decode"]
