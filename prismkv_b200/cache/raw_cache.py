"""RawKVCache: framework-agnostic compressed KV cache, resident on the GPU.

Same public API as the reference's RawKVCache (cache/raw_cache.py:57-292):
``update``, ``get``, ``get_codes``, ``get_seq_length``, ``clear``,
``cached_layers``, ``memory_footprint``.  The storage is B200-native:

* per layer, K and V codes live in one device buffer each, shaped
  (groups, capacity, m) with groups = the product of the leading dims
  (batch x heads) and compact codes (uint16 for 12-bit, uint8 for 8-bit);
* ``update`` encodes the new tokens straight into slots [len, len + s) of
  every group (``pkv_encode_append``) instead of ``torch.cat`` of flat
  int16 rows; capacity doubles when it runs out;
* ``attention(layer, q)`` runs the fused dequant + flash-decoding kernel on
  the buffer in place (its head stride is the capacity), so a decode step
  reads each cached code once and never materialises the context.

``update`` still returns the full decompressed context, as the reference's
does, decoded from the buffer by ``pkv_decode_cache``.  One difference is
deliberate: the reference appends each update's flat rows after the previous
ones and reshapes the concatenation, which interleaves heads once a layer
with more than one (batch, head) group has seen two updates; here every
group keeps its own tokens in order.  Shapes, dtypes and single-group values
are the reference's.
"""

from __future__ import annotations

import math
import threading
from dataclasses import dataclass
from typing import Dict, Optional, Tuple, Union

import torch

from ..quantizer.stacked_plane import _cuda_device
from .backend import CacheBackend, PrismKVBackend
from .cache_config import PrismKVConfig


@dataclass
class _LayerCodes:
    k: torch.Tensor            # (groups, capacity, m)
    v: torch.Tensor
    length: int
    leading: Tuple[int, ...]   # leading dims of the updates, e.g. (batch, heads)

    @property
    def groups(self) -> int:
        return self.k.shape[0]

    @property
    def capacity(self) -> int:
        return self.k.shape[1]


class RawKVCache:
    """backend: one CacheBackend for every layer, or a dict keyed by layer index.
    initial_capacity: token slots allocated per group on a layer's first update."""

    def __init__(self, backend: Union[CacheBackend, Dict[int, CacheBackend]], initial_capacity: int = 256) -> None:
        if isinstance(backend, dict):
            self._backends: Dict[int, CacheBackend] = dict(backend)
            self._default_backend: Optional[CacheBackend] = None
        else:
            self._backends = {}
            self._default_backend = backend
        self._initial_capacity = max(1, int(initial_capacity))
        self._layers: Dict[int, _LayerCodes] = {}
        self._lock = threading.Lock()

    # ------------------------------------------------------------------
    def _store_new(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor):
        """Encode (..., s, head_dim) K/V into the layer's buffers; returns (store, backend, s)."""
        head_dim, s = k.shape[-1], k.shape[-2]
        leading = tuple(k.shape[:-2])
        groups = math.prod(leading) if leading else 1
        backend = self._get_backend(layer_idx, head_dim)
        dev = _cuda_device(k)
        codec = backend.codec(dev)
        xk = backend.aligner.pad(k.to(dev).reshape(groups, s, head_dim))
        xv = backend.aligner.pad(v.to(dev).reshape(groups, s, head_dim))
        with self._lock:
            st = self._layers.get(layer_idx)
            if st is not None and (st.groups != groups or st.k.device != dev):
                raise ValueError(f"layer {layer_idx}: update with {groups} groups on {dev}, "
                                 f"cache holds {st.groups} on {st.k.device}")
            if st is None:
                cap = max(self._initial_capacity, s)
                dt = backend.quantizer.code_dtype
                st = _LayerCodes(torch.empty((groups, cap, codec.m), dtype=dt, device=dev),
                                 torch.empty((groups, cap, codec.m), dtype=dt, device=dev), 0, leading)
                self._layers[layer_idx] = st
            elif st.length + s > st.capacity:
                cap = max(2 * st.capacity, st.length + s)
                for name in ("k", "v"):
                    old = getattr(st, name)
                    new = torch.empty((groups, cap, codec.m), dtype=old.dtype, device=dev)
                    new[:, :st.length].copy_(old[:, :st.length])
                    setattr(st, name, new)
            pos = st.length
            codec.encode_append(xk, st.k, pos)
            codec.encode_append(xv, st.v, pos)
            st.length = pos + s
            if leading:
                st.leading = leading
        return st, backend

    def update(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Compress and append new K/V tokens (..., s, head_dim); return the full
        decompressed context (..., total, head_dim) in the input's dtype and device."""
        st, backend = self._store_new(layer_idx, k, v)
        out_shape = (*st.leading, st.length, k.shape[-1]) if k.dim() > 2 else (st.length, k.shape[-1])
        res = []
        for codes in (st.k, st.v):
            x = backend.codec(codes.device).decode_cache(codes, 0, st.length)
            res.append(backend.aligner.unpad(x).reshape(out_shape).to(device=k.device, dtype=k.dtype))
        return res[0], res[1]

    def append(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> int:
        """Compress and append without decoding the context; returns the new length."""
        return self._store_new(layer_idx, k, v)[0].length

    def attention(self, layer_idx: int, q: torch.Tensor, scale: Optional[float] = None) -> torch.Tensor:
        """Decode attention of q (B, Hq, head_dim) over the layer's cached codes.

        The cached leading dims must be (B, Hkv) with Hq a multiple of Hkv; the
        fused kernel reads the codes in place.  Returns (B, Hq, head_dim) fp32.
        """
        st = self._layers[layer_idx]
        backend = self._get_backend(layer_idx)
        if len(st.leading) != 2:
            raise ValueError("attention needs updates shaped (batch, kv_heads, seq, head_dim)")
        B, Hkv = st.leading
        codec = backend.codec(st.k.device)
        kc = st.k.view(B, Hkv, st.capacity, codec.m)[:, :, :st.length]
        vc = st.v.view(B, Hkv, st.capacity, codec.m)[:, :, :st.length]
        if scale is None:
            scale = backend.head_dim ** -0.5
        qp = backend.aligner.pad(q.to(st.k.device))
        out = codec.attention(qp, kc, vc, scale=scale)
        return backend.aligner.unpad(out)

    def get(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Full decompressed K/V of a layer as flat (N, head_dim) float32 rows."""
        if layer_idx not in self._layers:
            raise KeyError(f"Layer {layer_idx} has no cached data.")
        st = self._layers[layer_idx]
        backend = self._get_backend(layer_idx)
        res = []
        for codes in (st.k, st.v):
            x = backend.codec(codes.device).decode_cache(codes, 0, st.length)
            res.append(backend.aligner.unpad(x).reshape(st.groups * st.length, -1))
        return res[0], res[1]

    def get_codes(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Codes of a layer as flat (N, n_groups) int16 rows, group by group."""
        if layer_idx not in self._layers:
            raise KeyError(f"Layer {layer_idx} has no cached data.")
        st = self._layers[layer_idx]
        return tuple(c[:, :st.length].reshape(-1, c.shape[2]).to(torch.int16) for c in (st.k, st.v))

    def get_code_buffers(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor, int]:
        """The device buffers themselves: (groups, capacity, m) K and V codes and the length."""
        st = self._layers[layer_idx]
        return st.k, st.v, st.length

    def get_seq_length(self, layer_idx: int = 0) -> int:
        st = self._layers.get(layer_idx)
        return 0 if st is None else st.length

    def clear(self, layer_idx: Optional[int] = None) -> None:
        with self._lock:
            if layer_idx is None:
                self._layers.clear()
            else:
                self._layers.pop(layer_idx, None)

    @property
    def cached_layers(self) -> list:
        return sorted(self._layers.keys())

    def memory_footprint(self) -> dict:
        """codes_bytes (valid K + V codes), fp16_bytes (the same tokens in FP16), compression, n_layers."""
        codes_bytes = fp16_bytes = 0
        for layer_idx, st in self._layers.items():
            n_tokens = st.groups * st.length
            codes_bytes += 2 * n_tokens * st.k.shape[2] * st.k.element_size()
            fp16_bytes += n_tokens * self._get_backend(layer_idx).head_dim * 2 * 2
        return {"codes_bytes": codes_bytes, "fp16_bytes": fp16_bytes,
                "compression": fp16_bytes / codes_bytes if codes_bytes else float("nan"),
                "n_layers": len(self._layers)}

    def _get_backend(self, layer_idx: int, head_dim: Optional[int] = None) -> CacheBackend:
        if layer_idx in self._backends:
            return self._backends[layer_idx]
        if self._default_backend is not None:
            return self._default_backend
        if head_dim is not None:
            backend = PrismKVBackend(PrismKVConfig(), head_dim=head_dim)
            self._backends[layer_idx] = backend
            return backend
        raise KeyError(f"No backend for layer {layer_idx}. Pass a backend dict or "
                       "ensure the default backend is set.")

    def __repr__(self) -> str:
        fp = self.memory_footprint()
        return f"RawKVCache(n_layers={fp['n_layers']}, compression={fp['compression']:.1f}× vs FP16)"
