"""Multi-GPU decode over packed KV codes: one process per GPU, ``torch.distributed``.

Two partitionings of the decode-attention path:

* **Sequence shards** (split-sequence decode for long contexts).  Rank r holds
  tokens ``shard_range(S, N, r)`` of every (batch, kv head).  Each rank runs
  the fused kernel in partial mode, giving rotated-space softmax partials
  ``[m, l, o]`` (natural-log max, weight sum, unnormalised output) per
  (batch, q head).  Either one NCCL all-gather exchanges them (4 B x
  (dim + 2) per row and rank) and ``pkv_lse_combine`` merges them, or
  (``SequenceExchange``, the fast path) the attention kernel itself stores
  each finished unit's partial rows into every rank's CUDA-IPC-mapped buffer
  as flagged 8-byte words, and after its last item every CTA of every rank
  waits for the flags of its share of the units, merges them and applies
  ``R`` -- one launch per step, no fences or counters, every cross-GPU wait
  bounded.  The merge is the log-sum-exp rule
  ``o = sum_i e^(m_i - M) o_i / sum_i e^(m_i - M) l_i``.
* **Batch shards.**  Rank r holds batch rows ``shard_range(B, N, r)``; the
  ranks share nothing and no collective runs.

The query is replicated on every rank (a decode step's query is tiny).  The
reference has no multi-GPU path: it decodes on one CPU (polar_attention.py
:277-309); sequence sharding is the decomposition of that same softmax.
"""

from __future__ import annotations

import ctypes
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


class _DeviceArray:
    """A float32 array in device memory that torch can wrap without a copy (CUDA array interface)."""

    def __init__(self, ptr: int, shape, device):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}
        self.device = device


class SequenceExchange:
    """The split-sequence exchange of pkv_attn_decode_xr: one buffer per rank, merged in-kernel.

    Every rank allocates one zeroed device buffer (pkv_xr_alloc: plain cudaMalloc memory, not
    bound to any NVSwitch object) and exports its CUDA IPC handle; the handles are all-gathered over the process group
    and every rank maps every peer's buffer (pkv_xr_open, plain peer memory over NVLink).  A
    decode step is then ONE kernel launch per rank: the kernel stores each finished unit's
    partial rows into every rank's buffer as (value, call flag) words, and every rank merges
    the world partials of each unit in its own buffer once their flags are in, applies R and
    stores its output rows.  ``out`` is this rank's copy of those rows, (B, Hq, dim) fp32; a
    step overwrites it, so read it before the next step.  Every cross-rank wait is bounded by
    ``wait_ms`` of device time; after an expiry (``check`` raises) every rank must ``reset``.

    The buffer layout follows the kernel plan of the example tensors (batch, heads, codec and
    query dtype); later calls must have the same shapes apart from the token count.
    ``SequenceExchange.single_process`` builds ``world`` buffers on one device with this process
    as rank 0 -- world 1 runs the whole protocol on one GPU; with world > 1 nothing plays the
    other ranks, so the wait for their partials runs out (a test of the bounded wait).
    """

    def __init__(self, quantizer, q: torch.Tensor, k_codes: torch.Tensor, group=None, wait_ms: float = 1000.0,
                 _single_world: Optional[int] = None):
        from . import _lib
        self.lib = _lib.load()
        self.codec = quantizer.codec(q.device)
        self.device = q.device
        if _single_world is None:
            self.group = group or dist.group.WORLD
            self.world, self.rank = dist.get_world_size(self.group), dist.get_rank(self.group)
        else:
            self.group = None
            self.world, self.rank = _single_world, 0
        if not 1 <= self.world <= _lib.XR_MAX_RANKS:
            raise ValueError(f"the split-sequence exchange supports 1..{_lib.XR_MAX_RANKS} ranks, not {self.world}")
        if q.dim() == 4:
            q = q[:, :, 0, :]
        self.shape = tuple(q.shape)
        self.layout = self._layout(q, k_codes)
        self._checked = set()
        self.owned, self.opened = [], []
        with torch.cuda.device(self.device):
            n_own = 1 if _single_world is None else self.world
            handles = []
            for _ in range(n_own):
                ptr, handle = ctypes.c_void_p(), (ctypes.c_char * _lib.IPC_HANDLE_BYTES)()
                _lib.check(self.lib.pkv_xr_alloc(self.layout.bytes, ctypes.byref(ptr), handle), "pkv_xr_alloc")
                self.owned.append(ptr.value)
                handles.append(bytes(handle))
            if _single_world is None:
                gathered = [None] * self.world
                dist.all_gather_object(gathered, handles[0], group=self.group)
                buffers = []
                for r in range(self.world):
                    if r == self.rank:
                        buffers.append(self.owned[0])
                        continue
                    ptr = ctypes.c_void_p()
                    _lib.check(self.lib.pkv_xr_open(gathered[r], ctypes.byref(ptr)), "pkv_xr_open")
                    self.opened.append(ptr.value)
                    buffers.append(ptr.value)
            else:
                buffers = list(self.owned)
        x = _lib.PkvExchange()
        x.world, x.rank = self.world, self.rank
        for r, b in enumerate(buffers):
            x.buffers[r] = b
        x.wait_limit_us = max(1, int(wait_ms * 1000))
        self.struct = x
        B, Hq, D = self.shape
        self.out = torch.as_tensor(_DeviceArray(buffers[self.rank] + self.layout.out_offset, (B, Hq, D),
                                                self.device), device=self.device)

    @classmethod
    def single_process(cls, quantizer, q, k_codes, world: int = 1, wait_ms: float = 1000.0) -> "SequenceExchange":
        return cls(quantizer, q, k_codes, wait_ms=wait_ms, _single_world=world)

    def _layout(self, q, k_codes):
        from . import _lib
        a = self.codec._attn_args(q, k_codes, k_codes, self.codec.dim ** -0.5, None, None, 0, None)
        lay = _lib.PkvXrLayout()
        with torch.cuda.device(self.device):
            _lib.check(self.lib.pkv_xr_layout_for(ctypes.byref(self.codec.struct), ctypes.byref(a), self.world,
                                                  ctypes.byref(lay)), "pkv_xr_layout_for")
        return lay

    def run(self, q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor, scale: Optional[float] = None,
            num_splits: int = 0) -> torch.Tensor:
        """One decode step over this rank's token shard; returns ``out`` (all ranks' merged rows)."""
        from . import _lib
        if q.dim() == 4:
            q = q[:, :, 0, :]
        if tuple(q.shape) != self.shape:
            raise ValueError(f"exchange built for queries {self.shape}, got {tuple(q.shape)}")
        key = (q.dtype, k_codes.dtype, tuple(k_codes.shape), num_splits)
        if key not in self._checked:                      # plan each call shape once
            lay = self._layout(q, k_codes)
            if (lay.bytes, lay.units) != (self.layout.bytes, self.layout.units):
                raise ValueError("this call's kernel plan splits the heads into other units than the exchange's")
            self._checked.add(key)
        self.codec.attention(q, k_codes, v_codes, scale=scale, num_splits=num_splits, exchange=self)
        return self.out

    def check(self) -> None:
        """Raise if a bounded wait ran out (synchronises the device)."""
        from . import _lib
        with torch.cuda.device(self.device):
            err = _lib.device_error(clear=True)
        if err:
            raise RuntimeError(f"split-sequence exchange: device error {err} (a rank's wait ran out); "
                               "every rank must reset() the exchange before the next step")

    def reset(self, q: torch.Tensor, k_codes: torch.Tensor) -> None:
        """Zero this rank's counters (after a failed step, on every rank, between steps)."""
        from . import _lib
        if q.dim() == 4:
            q = q[:, :, 0, :]
        a = self.codec._attn_args(q, k_codes, k_codes, self.codec.dim ** -0.5, None, None, 0, None)
        with torch.cuda.device(self.device):
            _lib.check(self.lib.pkv_xr_reset(ctypes.byref(self.codec.struct), ctypes.byref(a),
                                             ctypes.byref(self.struct), _lib.stream_ptr(self.device)),
                       "pkv_xr_reset")

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: no rank frees a buffer that a
        peer may still write)."""
        from . import _lib
        if not self.owned:
            return
        torch.cuda.synchronize(self.device)
        if self.group is not None:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for ptr in self.opened:
                _lib.check(self.lib.pkv_xr_close(ptr), "pkv_xr_close")
            if self.group is not None:
                dist.barrier(group=self.group)
            for ptr in self.owned:
                _lib.check(self.lib.pkv_xr_free(ptr), "pkv_xr_free")
        self.owned, self.opened = [], []


def split_sequence_decode(quantizer, q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor,
                          scale: Optional[float] = None, group=None,
                          out: Optional[torch.Tensor] = None,
                          exchange: Optional[SequenceExchange] = None) -> torch.Tensor:
    """Decode attention with the sequence sharded over the ranks of `group`.

    q: (B, Hq, dim), identical on every rank.  k_codes / v_codes: this rank's
    (B, Hkv, S_r, m) token shard (S_r may be 0).  Returns (B, Hq, dim) fp32,
    the attention over the concatenation of all ranks' shards in rank order.
    With `exchange` (a SequenceExchange) the merge happens inside the one
    attention kernel and the result is the exchange's ``out`` (copied into
    `out` when given); otherwise one NCCL all-gather moves the partials and
    ``pkv_lse_combine`` merges them.
    """
    if q.dim() == 4:
        q = q[:, :, 0, :]
    codec = quantizer.codec(q.device)
    B, Hq, D = q.shape
    if exchange is not None:
        res = exchange.run(q, k_codes, v_codes, scale=scale)
        if out is not None:
            out.copy_(res)
            return out
        return res
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


__all__ = ["shard_range", "gather_partials", "split_sequence_decode", "batch_shard_decode", "SequenceExchange"]
