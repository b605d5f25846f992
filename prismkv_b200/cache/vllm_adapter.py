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

from typing import Dict, List, Optional, Tuple

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
        # pinned host buffers of evicted blocks, reused by size: a swap loop allocates pinned
        # memory only until the pool covers its working set
        self._pool: Dict[Tuple[int, ...], List[torch.Tensor]] = {}
        # device -> host copies not yet known to be complete: (block key, event)
        self._pending: Dict[Tuple[int, int], torch.cuda.Event] = {}

    def _host_buffer(self, shape) -> torch.Tensor:
        free = self._pool.get(tuple(shape))
        if free:
            return free.pop()
        return torch.empty(shape, dtype=torch.int16, pin_memory=True)

    def compress_block(self, layer_idx: int, block_id: int, k_block: torch.Tensor,
                       v_block: torch.Tensor, sync: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
        """(num_heads, block_size, head_dim) blocks -> (num_heads * block_size, n_groups) int16 codes
        stored on the compressor's device.

        With host storage the codes go to pinned buffers (reused from evicted blocks) by an
        asynchronous copy.  ``sync=True`` (the reference's behaviour) waits for this block's
        copies before returning; ``sync=False`` returns at once -- the codes are complete after
        ``synchronize()``, and ``decompress_block`` of the block on the same stream needs no wait.
        """
        n_heads, block_size, head_dim = k_block.shape
        N = n_heads * block_size
        backend = self._backends[layer_idx]
        dev = _cuda_device(k_block)
        codec = backend.codec(dev)
        key = (layer_idx, block_id)
        out = []
        for blk in (k_block, v_block):
            x = backend.aligner.pad(blk.to(dev).reshape(N, head_dim))
            codes = codec.encode(x, code_dtype=torch.int16)
            if torch.device(self._device).type == "cpu":
                host = self._host_buffer(codes.shape)
                host.copy_(codes, non_blocking=True)
                out.append(host)
            else:
                out.append(codes.to(self._device))
        if torch.device(self._device).type == "cpu":
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(dev))
            if sync:
                ev.synchronize()
            else:
                self._pending[key] = ev
        self._release(key)
        self._compressed[key] = (out[0], out[1])
        return out[0], out[1]

    def synchronize(self) -> None:
        """Wait until every block compressed with ``sync=False`` is in host memory."""
        for ev in self._pending.values():
            ev.synchronize()
        self._pending.clear()

    def _release(self, key) -> None:
        """Return a block's pinned buffers to the pool (after its copies are done)."""
        old = self._compressed.pop(key, None)
        ev = self._pending.pop(key, None)
        if ev is not None:
            ev.synchronize()
        if old is not None and torch.device(self._device).type == "cpu":
            for t in old:
                if t.is_pinned():
                    self._pool.setdefault(tuple(t.shape), []).append(t)

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
        """Drop a compressed block (the block was freed in vLLM); its pinned buffers are reused."""
        self._release((layer_idx, block_id))

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
        return (f"<VLLMSwapCompressor head_dim {self._head_dim}, {self._n_layers} layers, "
                f"{len(self._compressed)} blocks held>")
