"""PrismKVCache: compressed KV cache for HuggingFace models (a DynamicCache).

Same behaviour as the reference's PrismKVCache (cache/kv_cache.py:47-292):
``update`` encodes the incoming key/value states, keeps the codes, decodes
them and hands the decoded tensors to ``DynamicCache.update``, so attention
and every parent method work unchanged.  Here the codes stay on the GPU in
(batch x heads, capacity, m) buffers filled by ``pkv_encode_append``, and only
the new tokens are decoded (``pkv_decode_cache``).  The decoded values are
bit-identical to encode -> decode of the same rows.
"""

from __future__ import annotations

import threading
from typing import Dict, List, Optional

import torch

from ..quantizer.stacked_plane import StackedPlaneQuantizer, _cuda_device
from .backend import make_quantizer
from .cache_config import PrismKVConfig
from .dim_aligner import DimAligner

try:
    from transformers import DynamicCache
    HAS_TRANSFORMERS = True
except ImportError:                      # pragma: no cover - transformers is in the image
    HAS_TRANSFORMERS = False
    DynamicCache = object


def _require_transformers() -> None:
    if not HAS_TRANSFORMERS:
        raise ImportError("transformers is required for PrismKVCache (pip install transformers)")


class PrismKVCache(DynamicCache):
    """config: one PrismKVConfig for every layer; configs: per-layer configs (overrides config)."""

    def __init__(self, config: Optional[PrismKVConfig] = None,
                 configs: Optional[List[PrismKVConfig]] = None, initial_capacity: int = 256) -> None:
        _require_transformers()
        super().__init__()
        self._default_config = config or PrismKVConfig()
        self._per_layer_configs = configs
        self._initial_capacity = max(1, int(initial_capacity))
        self._key_codes: List[Optional[torch.Tensor]] = []     # (batch * heads, capacity, m) per layer
        self._val_codes: List[Optional[torch.Tensor]] = []
        self._lengths: List[int] = []
        self._shapes: List[Optional[tuple]] = []                # (batch, heads)
        self._quantizers: Dict[int, StackedPlaneQuantizer] = {}
        self._aligners: Dict[int, DimAligner] = {}
        self._lock = threading.Lock()

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int, *args, **kwargs):
        """key_states / value_states: (batch, heads, new_seq, head_dim)."""
        batch, n_heads, s, head_dim = key_states.shape
        q, aligner = self._get_quantizer_and_aligner(layer_idx, head_dim)
        dev = _cuda_device(key_states)
        codec = q.codec(dev)
        G = batch * n_heads
        with self._lock:
            while len(self._key_codes) <= layer_idx:
                self._key_codes.append(None)
                self._val_codes.append(None)
                self._lengths.append(0)
                self._shapes.append(None)
            kc, vc, n = self._key_codes[layer_idx], self._val_codes[layer_idx], self._lengths[layer_idx]
            if kc is None or kc.shape[0] != G:
                cap = max(self._initial_capacity, s)
                kc = torch.empty((G, cap, codec.m), dtype=q.code_dtype, device=dev)
                vc = torch.empty_like(kc)
                n = 0
            elif n + s > kc.shape[1]:
                cap = max(2 * kc.shape[1], n + s)
                k2 = torch.empty((G, cap, codec.m), dtype=kc.dtype, device=dev)
                v2 = torch.empty_like(k2)
                k2[:, :n].copy_(kc[:, :n])
                v2[:, :n].copy_(vc[:, :n])
                kc, vc = k2, v2
            decoded = []
            for states, codes in ((key_states, kc), (value_states, vc)):
                x = aligner.pad(states.to(dev).reshape(G, s, head_dim))
                codec.encode_append(x, codes, n)
                d = aligner.unpad(codec.decode_cache(codes, n, s)).reshape(batch, n_heads, s, head_dim)
                decoded.append(d.to(device=key_states.device, dtype=key_states.dtype))
            self._key_codes[layer_idx], self._val_codes[layer_idx] = kc, vc
            self._lengths[layer_idx] = n + s
            self._shapes[layer_idx] = (batch, n_heads)
        return super().update(decoded[0], decoded[1], layer_idx, *args, **kwargs)

    def get_codes(self, layer_idx: int):
        """(batch, heads, seq, m) K and V codes of a layer (views of the device buffers)."""
        kc, vc, n = self._key_codes[layer_idx], self._val_codes[layer_idx], self._lengths[layer_idx]
        B, H = self._shapes[layer_idx]
        return (kc.view(B, H, kc.shape[1], -1)[:, :, :n], vc.view(B, H, vc.shape[1], -1)[:, :, :n])

    def memory_footprint(self) -> dict:
        codes_bytes = fp16_bytes = 0
        n_layers = 0
        for layer_idx, kc in enumerate(self._key_codes):
            if kc is None:
                continue
            n_layers += 1
            n_tokens = kc.shape[0] * self._lengths[layer_idx]
            codes_bytes += 2 * n_tokens * kc.shape[2] * kc.element_size()
            if layer_idx in self._aligners:
                fp16_bytes += n_tokens * self._aligners[layer_idx].original_dim * 2 * 2
        return {"codes_bytes": codes_bytes, "fp16_bytes": fp16_bytes,
                "compression": fp16_bytes / codes_bytes if codes_bytes else float("nan"), "n_layers": n_layers}

    def compression_ratio(self) -> float:
        return self.memory_footprint()["compression"]

    def crop(self, max_length: int) -> None:
        """Crop to max_length tokens; the code buffers follow the parent's layers."""
        super().crop(max_length)
        for layer_idx in range(len(self._key_codes)):
            if self._key_codes[layer_idx] is None or layer_idx >= len(self.layers):
                continue
            layer = self.layers[layer_idx]
            if layer.is_initialized:
                self._lengths[layer_idx] = min(self._lengths[layer_idx], layer.keys.shape[-2])

    def reorder_cache(self, beam_idx: torch.LongTensor) -> None:
        """Beam reorder of the parent's tensors and of the code buffers (batch dim)."""
        super().reorder_cache(beam_idx)
        for layer_idx, kc in enumerate(self._key_codes):
            if kc is None:
                continue
            B, H = self._shapes[layer_idx]
            idx = beam_idx.to(kc.device)
            for lst in (self._key_codes, self._val_codes):
                c = lst[layer_idx]
                lst[layer_idx] = c.view(B, H, c.shape[1], -1).index_select(0, idx).reshape(B * H, c.shape[1], -1)

    def _get_config(self, layer_idx: int) -> PrismKVConfig:
        if self._per_layer_configs is not None and layer_idx < len(self._per_layer_configs):
            return self._per_layer_configs[layer_idx]
        return self._default_config

    def _get_quantizer_and_aligner(self, layer_idx: int, head_dim: int):
        if layer_idx not in self._quantizers:
            aligner = DimAligner(head_dim)
            self._quantizers[layer_idx] = make_quantizer(self._get_config(layer_idx), aligner.padded_dim,
                                                         "PrismKVCache")
            self._aligners[layer_idx] = aligner
        return self._quantizers[layer_idx], self._aligners[layer_idx]

    def __repr__(self) -> str:
        fp = self.memory_footprint()
        return (f"PrismKVCache({self._default_config!r}, n_layers_cached={fp['n_layers']}, "
                f"compression={fp['compression']:.1f}× vs FP16)")
