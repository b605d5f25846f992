"""VLLMSwapCompressor: PrismKV codes for vLLM KV blocks at the swap boundary.

Same interface as the reference's adapter (cache/vllm_adapter.py:73-291):
``compress_block`` / ``decompress_block`` / ``evict_block`` / ``attach``.  The
B200 difference is where the work happens.  The reference copies each fp16
block to the host as fp32 and encodes it on the CPU; here the block is
encoded on the GPU where it lives, and only the codes cross PCIe: 2 bytes per
triplet instead of 4 bytes per element, a 6x cut (3x against fp16), and the
codes land in pinned host memory with an asynchronous copy.  Swap-in copies
the codes back and decodes them on the GPU.
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from ..quantizer.stacked_plane import _cuda_device
from .backend import PrismKVBackend
from .cache_config import PrismKVConfig


def _require_vllm() -> None:
    try:
        import vllm  # noqa: F401
    except ImportError as e:
        raise ImportError("vllm is required for VLLMSwapCompressor (pip install vllm)") from e


class VLLMSwapCompressor:
    """config: compression settings; head_dim: attention head dim; n_layers: layers;
    device: where compressed blocks are stored ("cpu" = pinned host memory)."""

    def __init__(self, config: Optional[PrismKVConfig] = None, head_dim: int = 128, n_layers: int = 32,
                 device: str = "cpu") -> None:
        self._config = config or PrismKVConfig()
        self._head_dim = head_dim
        self._n_layers = n_layers
        self._device = device
        self._backends: Dict[int, PrismKVBackend] = {
            i: PrismKVBackend(self._config, head_dim=head_dim, device=device) for i in range(n_layers)}
        self._compressed: Dict[Tuple[int, int], Tuple[torch.Tensor, torch.Tensor]] = {}

    def compress_block(self, layer_idx: int, block_id: int, k_block: torch.Tensor,
                       v_block: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(num_heads, block_size, head_dim) blocks -> (num_heads * block_size, n_groups) int16 codes
        stored on the compressor's device."""
        n_heads, block_size, head_dim = k_block.shape
        N = n_heads * block_size
        backend = self._backends[layer_idx]
        dev = _cuda_device(k_block)
        codec = backend.codec(dev)
        out = []
        for blk in (k_block, v_block):
            x = backend.aligner.pad(blk.to(dev).reshape(N, head_dim))
            codes = codec.encode(x, code_dtype=torch.int16)
            if torch.device(self._device).type == "cpu":
                host = torch.empty(codes.shape, dtype=codes.dtype, pin_memory=True)
                host.copy_(codes, non_blocking=True)
                out.append(host)
            else:
                out.append(codes.to(self._device))
        torch.cuda.current_stream(dev).synchronize()
        self._compressed[(layer_idx, block_id)] = (out[0], out[1])
        return out[0], out[1]

    def decompress_block(self, layer_idx: int, block_id: int, n_heads: int, block_size: int,
                         dtype: torch.dtype = torch.float16, device: str = "cuda") -> Tuple[torch.Tensor, torch.Tensor]:
        """Stored codes -> (num_heads, block_size, head_dim) blocks of `dtype` on `device`."""
        key = (layer_idx, block_id)
        if key not in self._compressed:
            raise KeyError(f"No compressed block for layer={layer_idx}, block={block_id}. "
                           "Was compress_block called for this block?")
        k_codes, v_codes = self._compressed[key]
        backend = self._backends[layer_idx]
        target = torch.device(device)
        dev = target if target.type == "cuda" else _cuda_device()
        codec = backend.codec(dev)
        out = []
        for codes in (k_codes, v_codes):
            x = codec.decode(codes.to(dev, non_blocking=True), out_dtype=torch.float32)
            blk = backend.aligner.unpad(x).reshape(n_heads, block_size, self._head_dim)
            out.append(blk.to(dtype=dtype, device=target))
        return out[0], out[1]

    def evict_block(self, layer_idx: int, block_id: int) -> None:
        """Drop a compressed block (the block was freed in vLLM)."""
        self._compressed.pop((layer_idx, block_id), None)

    def attach(self, engine: object) -> None:
        """Wrap ``engine.cache_engine`` swap_out / swap_in (vLLM 0.4-0.6 CacheEngine API).

        As in the reference (vllm_adapter.py:193-243) the wrappers call the
        original swaps; routing blocks through compress_block / decompress_block
        needs the engine's per-layer block tables and stays an extension point.
        """
        _require_vllm()
        cache_engines = getattr(engine, "cache_engine", None)
        if cache_engines is None:
            raise AttributeError("engine has no 'cache_engine' attribute. "
                                 "Expected a vLLM LLMEngine with cache_engine list.")
        for ce in (cache_engines if isinstance(cache_engines, list) else [cache_engines]):
            orig_out, orig_in = ce.swap_out, ce.swap_in

            def patched_swap_out(src_to_dst, _orig=orig_out):
                _orig(src_to_dst)

            def patched_swap_in(src_to_dst, _orig=orig_in):
                _orig(src_to_dst)

            ce.swap_out = patched_swap_out
            ce.swap_in = patched_swap_in

    @property
    def n_compressed_blocks(self) -> int:
        return len(self._compressed)

    def __repr__(self) -> str:
        return (f"VLLMSwapCompressor(head_dim={self._head_dim}, n_layers={self._n_layers}, "
                f"{self._config.bits_per_dim:.1f}bits/dim, compressed_blocks={len(self._compressed)})")
