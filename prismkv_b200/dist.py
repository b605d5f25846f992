"""Multi-GPU decode over packed KV codes: one process per GPU, ``torch.distributed``.

Two partitionings of the decode-attention path:

* **Sequence shards** (split-sequence decode for long contexts).  Rank r holds
  tokens ``shard_range(S, N, r)`` of every (batch, kv head).  Each rank runs
  the fused kernel in partial mode, giving rotated-space softmax partials
  ``[m, l, o]`` (natural-log max, weight sum, unnormalised output) per
  (batch, q head).  Either one NCCL all-gather exchanges them (4 B x
  (dim + 2) per row and rank) and ``pkv_lse_combine`` merges them, or
  (``PeerExchange``) each rank writes them into symmetric memory and, after
  one device-side barrier, ``pkv_lse_combine_gather`` reads every rank's rows
  over NVLink; both apply ``R`` once.  The merge is the
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


class PeerExchange:
    """Split-sequence exchange through symmetric memory instead of an all-gather.

    Every rank holds a buffer of `rows` partial rows ([m, l, o_rot], dim + 2
    floats each) in symmetric memory, twice (calls alternate between the two
    halves).  The attention kernel writes its partials straight into this
    rank's half; one device-side barrier makes every rank's partials visible;
    then every rank's ``pkv_lse_combine_gather`` reads all ranks' rows over
    NVLink through the peer pointers and merges them.  Alternating halves make
    one barrier per call enough: a rank rewrites a half only after a later
    barrier, which every peer reaches after its reads of that half.
    """

    def __init__(self, rows: int, dim: int, device, group=None):
        import torch.distributed._symmetric_memory as symm
        self.group = group or dist.group.WORLD
        self.rows, self.dim = rows, dim
        self.slot = rows * (dim + 2)
        if hasattr(symm, "enable_symm_mem_for_group") and not symm.is_symm_mem_enabled_for_group(
                self.group.group_name):
            symm.enable_symm_mem_for_group(self.group.group_name)
        self.buf = symm.empty(2 * self.slot, dtype=torch.float32, device=device)
        self.handle = symm.rendezvous(self.buf, self.group.group_name)
        self.world = self.handle.world_size
        self.parity = 0

    def next_half(self):
        """(this rank's half as a (rows, dim + 2) view, its offset in floats) for the next call."""
        off = self.parity * self.slot
        self.parity ^= 1
        return self.buf[off:off + self.slot].view(self.rows, self.dim + 2), off


def split_sequence_decode(quantizer, q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor,
                          scale: Optional[float] = None, group=None,
                          out: Optional[torch.Tensor] = None,
                          exchange: Optional[PeerExchange] = None) -> torch.Tensor:
    """Decode attention with the sequence sharded over the ranks of `group`.

    q: (B, Hq, dim), identical on every rank.  k_codes / v_codes: this rank's
    (B, Hkv, S_r, m) token shard (S_r may be 0).  Returns (B, Hq, dim) fp32,
    the attention over the concatenation of all ranks' shards in rank order.
    With `exchange` (a PeerExchange of B * Hq rows) the partials cross NVLink
    through symmetric memory; otherwise one NCCL all-gather moves them.
    """
    if q.dim() == 4:
        q = q[:, :, 0, :]
    codec = quantizer.codec(q.device)
    B, Hq, D = q.shape
    if exchange is not None:
        half, off = exchange.next_half()
        codec.attention(q, k_codes, v_codes, scale=scale, partial=True, partial_out=half)
        exchange.handle.barrier(channel=0)
        res = codec.combine_gather(exchange.handle.buffer_ptrs_dev, exchange.world, off, B * Hq,
                                   out=None if out is None else out.view(B * Hq, D))
        return res.view(B, Hq, D)
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


__all__ = ["shard_range", "gather_partials", "split_sequence_decode", "batch_shard_decode", "PeerExchange"]
