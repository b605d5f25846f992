"""ctypes binding of libprismkv_b200.so (the C ABI in include/prismkv_b200.h).

The library is built in-tree by ``python -m prismkv_b200.build``.  There is no
fallback: if the library or a CUDA device is missing, every call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_float, c_int32, c_int64, c_size_t, c_void_p, c_char_p

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libprismkv_b200.so")

PKV_OK = 0
PKV_F32, PKV_BF16, PKV_F16 = 0, 1, 2
PKV_CODEC_Z_UNIFORM = 1
PKV_CODEC_FP32_ATTN = 2
DTYPE_CODES = {torch.float32: PKV_F32, torch.bfloat16: PKV_BF16, torch.float16: PKV_F16}

EXPORTED = ("pkv_abi_version", "pkv_strerror", "pkv_device_error", "pkv_encode", "pkv_decode",
            "pkv_attn_workspace_size", "pkv_workspace_init", "pkv_attn_decode", "pkv_lse_combine",
            "pkv_polar_scores", "pkv_attn_decode_noalloc", "pkv_attn_describe", "pkv_encode_append",
            "pkv_decode_cache", "pkv_lse_combine_gather", "pkv_xr_layout_for", "pkv_xr_alloc", "pkv_xr_open",
            "pkv_xr_close", "pkv_xr_free", "pkv_xr_reset", "pkv_attn_decode_xr")
XR_MAX_RANKS = 8
IPC_HANDLE_BYTES = 64


class PkvCodec(ctypes.Structure):
    _fields_ = [("dim", c_int32), ("bits_z", c_int32), ("bits_r", c_int32), ("bits_theta", c_int32),
                ("xy_mode", c_int32), ("xy_per_z", c_int32), ("z_nan_bin", c_int32), ("z_hi", c_float),
                ("r_max", c_float), ("flags", c_int32),
                ("R", c_void_p), ("z_thr", c_void_p), ("r2_thr", c_void_p), ("th_thr", c_void_p),
                ("codebook", c_void_p), ("dec_z", c_void_p), ("dec_xy", c_void_p), ("bias_xy", c_void_p),
                ("cell_idx", c_void_p), ("cell_cnt", c_void_p), ("cell_grid", c_int32), ("cell_half_width", c_float),
                ("R_bf16x3", c_void_p)]


class PkvAttnArgs(ctypes.Structure):
    _fields_ = [("batch", c_int32), ("q_heads", c_int32), ("kv_heads", c_int32), ("seq_len", c_int32),
                ("q", c_void_p), ("q_dtype", c_int32),
                ("q_batch_stride", c_int64), ("q_head_stride", c_int64),
                ("k_codes", c_void_p), ("v_codes", c_void_p), ("code_bytes", c_int32),
                ("kv_batch_stride", c_int64), ("kv_head_stride", c_int64),
                ("seq_lens", c_void_p), ("scale", c_float),
                ("out", c_void_p), ("out_batch_stride", c_int64), ("out_head_stride", c_int64),
                ("num_splits", c_int32), ("partial_only", c_int32), ("partial_out", c_void_p)]


class PkvAttnPlan(ctypes.Structure):
    _fields_ = [("kernel", c_int32), ("num_splits", c_int32), ("tokens_per_split", c_int32),
                ("threads", c_int32), ("smem_bytes", c_int32), ("ctas_per_sm", c_int32), ("balanced", c_int32)]


class PkvExchange(ctypes.Structure):
    _fields_ = [("world", c_int32), ("rank", c_int32), ("buffers", c_void_p * 8), ("wait_limit_us", ctypes.c_uint32)]


class PkvXrLayout(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_uint64), ("out_offset", ctypes.c_uint64), ("rows", c_int32), ("units", c_int32)]


KERNEL_NAMES = {1: "attn_mha12_kernel", 2: "attn_polar_kernel", 3: "attn_lut_kernel", 4: "attn_tc_kernel",
                5: "attn_mha8_kernel", 6: "attn_mha12_stream_kernel", 7: "attn_gqa12_kernel",
                8: "attn_gqa12_mma_kernel"}

_lock = threading.Lock()
_lib = None


def _declare(lib):
    P = ctypes.POINTER
    lib.pkv_abi_version.restype = c_int32
    lib.pkv_abi_version.argtypes = []
    lib.pkv_strerror.restype = c_char_p
    lib.pkv_strerror.argtypes = [c_int32]
    lib.pkv_device_error.restype = c_int32
    lib.pkv_device_error.argtypes = [P(c_int32), c_int32]
    lib.pkv_encode.restype = c_int32
    lib.pkv_encode.argtypes = [P(PkvCodec), c_void_p, c_int32, c_int64, c_int64, c_void_p, c_int32, c_int64, c_void_p]
    lib.pkv_decode.restype = c_int32
    lib.pkv_decode.argtypes = [P(PkvCodec), c_void_p, c_int32, c_int64, c_int64, c_void_p, c_int32, c_int64, c_void_p]
    lib.pkv_encode_append.restype = c_int32
    lib.pkv_encode_append.argtypes = [P(PkvCodec), c_void_p, c_int32, c_int64, c_int64, c_int64, c_void_p, c_int32,
                                      c_int64, c_int64, c_int64, c_void_p]
    lib.pkv_decode_cache.restype = c_int32
    lib.pkv_decode_cache.argtypes = [P(PkvCodec), c_void_p, c_int32, c_int64, c_int64, c_int64, c_int64, c_int64,
                                     c_void_p, c_int32, c_int64, c_void_p]
    lib.pkv_attn_workspace_size.restype = c_size_t
    lib.pkv_attn_workspace_size.argtypes = [P(PkvCodec), P(PkvAttnArgs)]
    lib.pkv_workspace_init.restype = c_int32
    lib.pkv_workspace_init.argtypes = [c_void_p, c_size_t, c_void_p]
    lib.pkv_attn_decode.restype = c_int32
    lib.pkv_attn_decode.argtypes = [P(PkvCodec), P(PkvAttnArgs), c_void_p, c_size_t, c_void_p]
    lib.pkv_attn_decode_noalloc.restype = c_int32
    lib.pkv_attn_decode_noalloc.argtypes = [P(PkvCodec), P(PkvAttnArgs), c_void_p]
    lib.pkv_attn_describe.restype = c_int32
    lib.pkv_attn_describe.argtypes = [P(PkvCodec), P(PkvAttnArgs), P(PkvAttnPlan)]
    lib.pkv_lse_combine.restype = c_int32
    lib.pkv_lse_combine.argtypes = [P(PkvCodec), c_void_p, c_int32, c_int64, c_int32, c_void_p, c_int64, c_void_p]
    lib.pkv_lse_combine_gather.restype = c_int32
    lib.pkv_lse_combine_gather.argtypes = [P(PkvCodec), c_void_p, c_int32, c_int64, c_int32, c_void_p, c_int64,
                                           c_void_p]
    lib.pkv_xr_layout_for.restype = c_int32
    lib.pkv_xr_layout_for.argtypes = [P(PkvCodec), P(PkvAttnArgs), c_int32, P(PkvXrLayout)]
    lib.pkv_xr_alloc.restype = c_int32
    lib.pkv_xr_alloc.argtypes = [ctypes.c_uint64, P(c_void_p), c_void_p]
    lib.pkv_xr_open.restype = c_int32
    lib.pkv_xr_open.argtypes = [c_void_p, P(c_void_p)]
    lib.pkv_xr_close.restype = c_int32
    lib.pkv_xr_close.argtypes = [c_void_p]
    lib.pkv_xr_free.restype = c_int32
    lib.pkv_xr_free.argtypes = [c_void_p]
    lib.pkv_xr_reset.restype = c_int32
    lib.pkv_xr_reset.argtypes = [P(PkvCodec), P(PkvAttnArgs), P(PkvExchange), c_void_p]
    lib.pkv_attn_decode_xr.restype = c_int32
    lib.pkv_attn_decode_xr.argtypes = [P(PkvCodec), P(PkvAttnArgs), c_void_p, c_size_t, P(PkvExchange), c_void_p]
    lib.pkv_polar_scores.restype = c_int32
    lib.pkv_polar_scores.argtypes = [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
                                     P(c_float), P(c_int32), c_void_p, c_void_p]


def load():
    """Load the library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m prismkv_b200.build` "
                    "(the PrismKV B200 path has no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            _declare(lib)
            if lib.pkv_abi_version() != 1:
                raise RuntimeError("libprismkv_b200.so ABI version mismatch; rebuild it")
            _lib = lib
    return _lib


def available() -> bool:
    """True when the library loads and a CUDA device is present."""
    try:
        load()
    except (RuntimeError, OSError):
        return False
    return torch.cuda.is_available()


def check(rc: int, what: str) -> None:
    if rc != PKV_OK:
        msg = load().pkv_strerror(rc).decode()
        raise RuntimeError(f"{what} failed: {msg} (status {rc})")


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_error(clear: bool = True) -> int:
    flag = c_int32(0)
    check(load().pkv_device_error(ctypes.byref(flag), int(clear)), "pkv_device_error")
    return int(flag.value)
