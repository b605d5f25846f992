"""save_cache / load_cache: PrismKVCache codes to and from .npz files.

The file format is the reference's (cache/cache_store.py:1-15): per layer i,
``codes_key_{i}`` / ``codes_val_{i}`` int16 (N, m) arrays, plus ``config_bz``,
``config_br``, ``config_bt`` and ``n_layers``.  Files written by either
implementation load in the other.  Two keys are added, and readers that do
not know them ignore them: ``shape_{i}`` = (batch, heads, seq) restores the
layer's structure (the reference reloads every layer as batch 1, head 1), and
``head_dim_{i}`` records the unpadded head dimension, which the reference
infers from the code width and gets wrong for padded dims such as 64 -> 66.
Without those keys, loading follows the reference exactly.
"""

from __future__ import annotations

from pathlib import Path
from typing import Union

import numpy as np
import torch

from ..quantizer.stacked_plane import _cuda_device
from .cache_config import PrismKVConfig


def save_cache(cache, path: Union[str, Path]) -> None:
    """Write a PrismKVCache's codes (not its decoded tensors) to ``path``."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    arrays = {}
    n_layers = len(cache._key_codes)
    for i in range(n_layers):
        if cache._key_codes[i] is None:
            continue
        kc, vc = cache.get_codes(i)                    # (B, H, S, m)
        arrays[f"codes_key_{i}"] = kc.reshape(-1, kc.shape[-1]).to(torch.int16).cpu().numpy()
        arrays[f"codes_val_{i}"] = vc.reshape(-1, vc.shape[-1]).to(torch.int16).cpu().numpy()
        arrays[f"shape_{i}"] = np.asarray(kc.shape[:3], dtype=np.int64)
        arrays[f"head_dim_{i}"] = np.int32(cache._aligners[i].original_dim)
    cfg = cache._default_config
    arrays["config_bz"] = np.int32(cfg.bits_z)
    arrays["config_br"] = np.int32(cfg.bits_r)
    arrays["config_bt"] = np.int32(cfg.bits_theta)
    arrays["n_layers"] = np.int32(n_layers)
    np.savez_compressed(str(path), **arrays)


def _infer_head_dim(m: int) -> int:
    """The reference's guess for files without ``head_dim_{i}``: the padded width itself."""
    return 3 * m


def load_cache(path: Union[str, Path], device: str = "cpu"):
    """Read a file written by save_cache (either implementation) into a new PrismKVCache.

    Codes go to the GPU; the decoded tensors handed to the parent DynamicCache
    land on ``device``.
    """
    from transformers import DynamicCache

    from .kv_cache import PrismKVCache
    data = np.load(str(path))
    cfg = PrismKVConfig(bits_z=int(data["config_bz"]), bits_r=int(data["config_br"]),
                        bits_theta=int(data["config_bt"]))
    cache = PrismKVCache(config=cfg)
    gpu = _cuda_device()
    for i in range(int(data["n_layers"])):
        if f"codes_key_{i}" not in data:
            continue
        kc = torch.from_numpy(data[f"codes_key_{i}"]).to(gpu)
        vc = torch.from_numpy(data[f"codes_val_{i}"]).to(gpu)
        m = kc.shape[-1]
        head_dim = int(data[f"head_dim_{i}"]) if f"head_dim_{i}" in data else _infer_head_dim(m)
        B, H, S = (int(x) for x in data[f"shape_{i}"]) if f"shape_{i}" in data else (1, 1, kc.shape[0])
        q, aligner = cache._get_quantizer_and_aligner(i, head_dim)
        codec = q.codec(gpu)
        while len(cache._key_codes) <= i:
            cache._key_codes.append(None)
            cache._val_codes.append(None)
            cache._lengths.append(0)
            cache._shapes.append(None)
        dec = []
        stores = []
        for codes in (kc, vc):
            store = codes.reshape(B * H, S, m).to(q.code_dtype).contiguous()
            stores.append(store)
            x = aligner.unpad(codec.decode_cache(store, 0, S)).reshape(B, H, S, head_dim)
            dec.append(x.to(device))
        cache._key_codes[i], cache._val_codes[i] = stores
        cache._lengths[i] = S
        cache._shapes[i] = (B, H)
        DynamicCache.update(cache, dec[0], dec[1], layer_idx=i)
    return cache
