"""Device-resident quantizer state and the calls into the C ABI.

``DeviceCodec`` owns one device copy of a quantizer's tables (rotation,
thresholds, LUTs) and exposes the hot-path operations on CUDA tensors:
``encode``, ``decode``, ``attention`` (fused dequant + flash decoding) and
``combine`` (log-sum-exp merge of split-sequence partials).  All compute runs
in libprismkv_b200.so; torch only provides memory and streams.
"""

from __future__ import annotations

import ctypes
import math
from typing import Dict, Optional

import numpy as np
import torch

from . import _lib
from .tables import HostTables

CODE_DTYPES = {torch.uint8: 1, torch.int16: 2, torch.uint16: 2, torch.int64: 8}


def code_dtype_for(bits_total: int) -> torch.dtype:
    """Compact storage for a code of ``bits_total`` bits: uint8 up to 8 bits, else int16."""
    return torch.uint8 if bits_total <= 8 else torch.int16


def split_bf16x3(R: np.ndarray) -> np.ndarray:
    """R (fp32) as three bf16 parts, returned as their uint16 bit patterns (3, *R.shape).

    R1 and R2 truncate toward zero and R3 rounds to nearest, so every part has
    the sign of R and R1 + R2 + R3 equals R to within 2^-24 |R|.  A part that
    comes out exactly zero for a non-zero entry becomes the smallest bf16
    normal (2^-126) with R's sign: an infinite input then meets no zero and no
    opposite-signed part, and rotates to the same +-inf (or NaN) as an fp32
    dot product, while finite results move by less than 2^-126 |x|.
    """
    r = np.ascontiguousarray(R, dtype=np.float32)
    bits = r.view(np.uint32)
    r1 = (bits & 0xFFFF0000).view(np.float32)
    rem = (r - r1).astype(np.float32)
    r2 = (rem.view(np.uint32) & 0xFFFF0000).view(np.float32)
    rem2 = (r - r1 - r2).astype(np.float32)
    r3 = torch.from_numpy(rem2).to(torch.bfloat16).float().numpy()       # round to nearest even
    parts = []
    tiny = np.where(np.signbit(r), np.float32(-2.0 ** -126), np.float32(2.0 ** -126)).astype(np.float32)
    for part in (r1, r2, r3):
        part = np.where((part == 0) & (r != 0), tiny, part).astype(np.float32)
        parts.append((part.view(np.uint32) >> 16).astype(np.uint16))
    return np.stack(parts)


class DeviceCodec:
    def __init__(self, host: HostTables, device: torch.device):
        self.host = host
        self.device = torch.device(device)
        self.dim = host.dim
        self.m = host.dim // 3
        self.bits = host.bits
        self.bits_total = sum(host.bits)

        def up(a, min_len=1):
            a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
            if a.size < min_len:
                a = np.concatenate([a, np.zeros(min_len - a.size, np.float32)])
            return torch.from_numpy(a).to(self.device)

        self._R = up(host.R)
        self._R_bf16x3 = torch.from_numpy(split_bf16x3(host.R)).view(torch.bfloat16).to(self.device)
        self._z_thr = up(host.z_thr)
        self._r2 = up(host.r2_thr)
        self._th = up(host.th_thr)
        self._cb = up(host.codebook)
        self._dz = up(host.dec_z)
        self._dxy = up(host.dec_xy)
        self._bxy = up(host.bias_xy) if host.bias_xy is not None else None
        self._cell_idx = self._cell_cnt = None
        if host.cell_idx is not None:
            self._cell_idx = torch.from_numpy(np.ascontiguousarray(host.cell_idx).reshape(-1)).to(self.device)
            self._cell_cnt = torch.from_numpy(np.ascontiguousarray(host.cell_cnt).reshape(-1)).to(self.device)
        s = _lib.PkvCodec()
        s.dim = host.dim
        s.bits_z, s.bits_r, s.bits_theta = host.bits
        s.xy_mode = host.xy_mode
        s.xy_per_z = host.xy_per_z
        s.z_nan_bin = host.z_nan_bin
        s.z_hi = host.z_hi
        s.r_max = host.r_max
        s.flags = _lib.PKV_CODEC_Z_UNIFORM if host.z_uniform else 0
        s.R = self._R.data_ptr()
        s.z_thr = self._z_thr.data_ptr()
        s.r2_thr = self._r2.data_ptr()
        s.th_thr = self._th.data_ptr()
        s.codebook = self._cb.data_ptr()
        s.dec_z = self._dz.data_ptr()
        s.dec_xy = self._dxy.data_ptr()
        s.bias_xy = self._bxy.data_ptr() if self._bxy is not None else None
        s.R_bf16x3 = self._R_bf16x3.data_ptr()
        if self._cell_idx is not None:
            s.cell_idx = self._cell_idx.data_ptr()
            s.cell_cnt = self._cell_cnt.data_ptr()
            s.cell_grid = host.cell_idx.shape[1]
            s.cell_half_width = host.cell_half_width
        self.struct = s
        self._ws: Dict[int, torch.Tensor] = {}
        self.R = self._R.view(host.dim, host.dim)

    @property
    def fp32_attention(self) -> bool:
        """Attention arithmetic in fp32 throughout: the grouped 12-bit decode then runs on the fp32
        kernel instead of the fp16-pair tensor-core one (both are within 1e-5 of fp64)."""
        return bool(self.struct.flags & _lib.PKV_CODEC_FP32_ATTN)

    @fp32_attention.setter
    def fp32_attention(self, on: bool) -> None:
        if on:
            self.struct.flags |= _lib.PKV_CODEC_FP32_ATTN
        else:
            self.struct.flags &= ~_lib.PKV_CODEC_FP32_ATTN

    # ------------------------------------------------------------------
    def _stream(self) -> int:
        return _lib.stream_ptr(self.device)

    def encode(self, x: torch.Tensor, out: Optional[torch.Tensor] = None,
               code_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """(N, dim) float tensor on this device -> (N, m) codes."""
        _lib.require_cuda(x, "vectors")
        if x.dim() != 2 or x.shape[1] != self.dim:
            raise ValueError(f"expected (N, {self.dim}) vectors, got {tuple(x.shape)}")
        if x.dtype not in _lib.DTYPE_CODES:
            x = x.float()
        if x.stride(1) != 1:
            x = x.contiguous()
        n = x.shape[0]
        if out is None:
            out = torch.empty((n, self.m), dtype=code_dtype or code_dtype_for(self.bits_total), device=self.device)
        if out.dtype not in CODE_DTYPES or out.shape != (n, self.m) or out.stride(1) != 1:
            raise ValueError("codes output must be (N, m) uint8/int16/uint16/int64 with unit inner stride")
        lib = _lib.load()
        with torch.cuda.device(self.device):
            rc = lib.pkv_encode(ctypes.byref(self.struct), x.data_ptr(), _lib.DTYPE_CODES[x.dtype], n,
                                x.stride(0), out.data_ptr(), CODE_DTYPES[out.dtype], out.stride(0),
                                self._stream())
        _lib.check(rc, "pkv_encode")
        return out

    def encode_append(self, x: torch.Tensor, cache: torch.Tensor, pos: int) -> None:
        """Encode x (G, n, dim) into slots [pos, pos + n) of a (G, capacity, m) code cache."""
        _lib.require_cuda(x, "vectors")
        _lib.require_cuda(cache, "cache")
        if x.dim() != 3 or x.shape[2] != self.dim or cache.dim() != 3 or cache.shape[0] != x.shape[0]:
            raise ValueError("expected x (G, n, dim) and cache (G, capacity, m)")
        if cache.shape[2] != self.m or cache.stride(2) != 1 or cache.stride(1) != self.m:
            raise ValueError("cache rows must be compact (m codes per slot)")
        G, n, _ = x.shape
        if pos < 0 or pos + n > cache.shape[1]:
            raise ValueError(f"slots [{pos}, {pos + n}) outside capacity {cache.shape[1]}")
        if x.dtype not in _lib.DTYPE_CODES:
            x = x.float()
        x = x.contiguous()
        lib = _lib.load()
        with torch.cuda.device(self.device):
            rc = lib.pkv_encode_append(ctypes.byref(self.struct), x.data_ptr(), _lib.DTYPE_CODES[x.dtype], G, n,
                                       self.dim, cache.data_ptr(), CODE_DTYPES[cache.dtype], cache.stride(0),
                                       cache.stride(1), pos, self._stream())
        _lib.check(rc, "pkv_encode_append")

    def decode_cache(self, cache: torch.Tensor, pos: int, n: int,
                     out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Slots [pos, pos + n) of a (G, capacity, m) code cache -> (G, n, dim) vectors."""
        _lib.require_cuda(cache, "cache")
        if cache.dim() != 3 or cache.shape[2] != self.m or cache.stride(2) != 1:
            raise ValueError("expected a (G, capacity, m) cache with unit code stride")
        if pos < 0 or n < 0 or pos + n > cache.shape[1]:
            raise ValueError(f"slots [{pos}, {pos + n}) outside capacity {cache.shape[1]}")
        G = cache.shape[0]
        out = torch.empty((G, n, self.dim), dtype=out_dtype, device=self.device)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            rc = lib.pkv_decode_cache(ctypes.byref(self.struct), cache.data_ptr(), CODE_DTYPES[cache.dtype], G, n,
                                      cache.stride(0), cache.stride(1), pos, out.data_ptr(),
                                      _lib.DTYPE_CODES[out_dtype], self.dim, self._stream())
        _lib.check(rc, "pkv_decode_cache")
        return out

    def decode(self, codes: torch.Tensor, out: Optional[torch.Tensor] = None,
               out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """(N, m) codes on this device -> (N, dim) vectors."""
        _lib.require_cuda(codes, "codes")
        if codes.dim() != 2 or codes.shape[1] != self.m:
            raise ValueError(f"expected (N, {self.m}) codes, got {tuple(codes.shape)}")
        if codes.dtype not in CODE_DTYPES:
            codes = codes.to(torch.int64)
        if codes.stride(1) != 1:
            codes = codes.contiguous()
        n = codes.shape[0]
        if out is None:
            out = torch.empty((n, self.dim), dtype=out_dtype, device=self.device)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            rc = lib.pkv_decode(ctypes.byref(self.struct), codes.data_ptr(), CODE_DTYPES[codes.dtype], n,
                                codes.stride(0), out.data_ptr(), _lib.DTYPE_CODES[out.dtype], out.stride(0),
                                self._stream())
        _lib.check(rc, "pkv_decode")
        return out

    # ------------------------------------------------------------------
    def _attn_args(self, q, k_codes, v_codes, scale, seq_lens, out, num_splits, partial_out):
        B, Hq, D = q.shape
        _, Hkv, S, m = k_codes.shape
        a = _lib.PkvAttnArgs()
        a.batch, a.q_heads, a.kv_heads, a.seq_len = B, Hq, Hkv, S
        a.q = q.data_ptr()
        a.q_dtype = _lib.DTYPE_CODES[q.dtype]
        a.q_batch_stride, a.q_head_stride = q.stride(0), q.stride(1)
        a.k_codes, a.v_codes = k_codes.data_ptr(), v_codes.data_ptr()
        a.code_bytes = CODE_DTYPES[k_codes.dtype]
        a.kv_batch_stride, a.kv_head_stride = k_codes.stride(0), k_codes.stride(1)
        a.seq_lens = seq_lens.data_ptr() if seq_lens is not None else None
        a.scale = float(scale)
        a.out = out.data_ptr() if out is not None else None
        a.out_batch_stride = out.stride(0) if out is not None else 0
        a.out_head_stride = out.stride(1) if out is not None else 0
        a.num_splits = int(num_splits)
        a.partial_only = int(partial_out is not None)
        a.partial_out = partial_out.data_ptr() if partial_out is not None else None
        return a

    def describe(self, q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor,
                 num_splits: int = 0) -> dict:
        """The kernel and split plan ``attention`` would use for these tensors (launches nothing)."""
        if q.dim() == 4:
            q = q[:, :, 0, :]
        a = self._attn_args(q, k_codes, v_codes, self.dim ** -0.5, None, None, num_splits, None)
        plan = _lib.PkvAttnPlan()
        with torch.cuda.device(self.device):
            rc = _lib.load().pkv_attn_describe(ctypes.byref(self.struct), ctypes.byref(a), ctypes.byref(plan))
        _lib.check(rc, "pkv_attn_describe")
        d = {f: int(getattr(plan, f)) for f, _ in plan._fields_}
        d["kernel"] = _lib.KERNEL_NAMES[d["kernel"]]
        return d

    def workspace(self, nbytes: int) -> torch.Tensor:
        """Per-stream workspace, zeroed once when (re)allocated; calls leave it zeroed."""
        key = self._stream()
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=self.device)
            self._ws[key] = ws
        return ws

    def attention(self, q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor,
                  scale: Optional[float] = None, seq_lens: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None, num_splits: int = 0,
                  partial: bool = False, workspace: Optional[torch.Tensor] = None,
                  partial_out: Optional[torch.Tensor] = None, exchange=None) -> torch.Tensor:
        """Decode attention over packed codes.

        q (B, Hq, dim) [or (B, Hq, 1, dim)], k/v codes (B, Hkv, S, m) with unit
        token/triplet strides.  Returns (B, Hq, dim) fp32, or with
        ``partial=True`` the (B, Hq, dim + 2) rotated-space partials
        [m_max, l, o] for a cross-shard merge.  With ``exchange`` (a
        ``dist.SequenceExchange``) the codes are this rank's token shard and the
        merged rows of all ranks land in ``exchange.out`` (pkv_attn_decode_xr).
        """
        for t, n in ((q, "q"), (k_codes, "k_codes"), (v_codes, "v_codes")):
            _lib.require_cuda(t, n)
        if q.dim() == 4:
            if q.shape[2] != 1:
                raise ValueError("fused decode attention takes one query token (Sq == 1)")
            q = q[:, :, 0, :]
        if q.dtype not in _lib.DTYPE_CODES:
            q = q.float()
        if q.stride(2) != 1:
            q = q.contiguous()
        if k_codes.shape != v_codes.shape or k_codes.dtype != v_codes.dtype:
            raise ValueError("k_codes and v_codes must have the same shape and dtype")
        if k_codes.dtype not in (torch.uint8, torch.int16, torch.uint16):
            raise ValueError("codes must be stored as uint8 or 16-bit integers")
        if k_codes.stride() != v_codes.stride():
            raise ValueError("k_codes and v_codes must share strides")
        if k_codes.stride(3) != 1 or k_codes.stride(2) != self.m:
            raise ValueError("codes need unit triplet stride and token stride m")
        B, Hq, D = q.shape
        if D != self.dim or k_codes.shape[3] != self.m or k_codes.shape[0] != B:
            raise ValueError("shape mismatch between q and codes")
        if scale is None:
            scale = self.dim ** -0.5
        if seq_lens is not None:
            seq_lens = seq_lens.to(device=self.device, dtype=torch.int32).contiguous()
        if exchange is not None:
            partial, out, partial_out = False, None, None
        if partial:
            if partial_out is None:
                partial_out = torch.empty((B, Hq, self.dim + 2), dtype=torch.float32, device=self.device)
            elif (partial_out.dtype != torch.float32 or partial_out.numel() != B * Hq * (self.dim + 2)
                  or not partial_out.is_contiguous()):
                raise ValueError("partial_out must be a contiguous float32 tensor of B * Hq * (dim + 2)")
        else:
            partial_out = None
            if out is None and exchange is None:
                out = torch.empty((B, Hq, self.dim), dtype=torch.float32, device=self.device)
        a = self._attn_args(q, k_codes, v_codes, scale, seq_lens, out, num_splits, partial_out)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            a_ws = a
            if exchange is not None:            # the workspace size needs an output to plan with
                a_ws = self._attn_args(q, k_codes, v_codes, scale, seq_lens, exchange.out, num_splits, None)
            need = lib.pkv_attn_workspace_size(ctypes.byref(self.struct), ctypes.byref(a_ws))
            ws = workspace if workspace is not None else (self.workspace(need) if need else None)
            if exchange is not None:
                rc = lib.pkv_attn_decode_xr(ctypes.byref(self.struct), ctypes.byref(a),
                                            ws.data_ptr() if ws is not None else None,
                                            ws.numel() if ws is not None else 0, ctypes.byref(exchange.struct),
                                            self._stream())
                _lib.check(rc, "pkv_attn_decode_xr")
                return exchange.out
            rc = lib.pkv_attn_decode(ctypes.byref(self.struct), ctypes.byref(a),
                                     ws.data_ptr() if ws is not None else None,
                                     ws.numel() if ws is not None else 0, self._stream())
        _lib.check(rc, "pkv_attn_decode")
        return partial_out if partial else out

    def combine_gather(self, part_ptrs: int, n_parts: int, part_offset: int, rows: int,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Merge partials that live behind a device array of n_parts pointers (peer buffers)."""
        if out is None:
            out = torch.empty((rows, self.dim), dtype=torch.float32, device=self.device)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            rc = lib.pkv_lse_combine_gather(ctypes.byref(self.struct), part_ptrs, n_parts, part_offset, rows,
                                            out.data_ptr(), out.stride(0), self._stream())
        _lib.check(rc, "pkv_lse_combine_gather")
        return out

    def combine(self, partials: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Merge (n_parts, rows, dim + 2) partials into (rows, dim) outputs (with R applied)."""
        _lib.require_cuda(partials, "partials")
        partials = partials.float().contiguous()
        n_parts, rows = partials.shape[0], partials.shape[1]
        if out is None:
            out = torch.empty((rows, self.dim), dtype=torch.float32, device=self.device)
        lib = _lib.load()
        with torch.cuda.device(self.device):
            rc = lib.pkv_lse_combine(ctypes.byref(self.struct), partials.data_ptr(), n_parts,
                                     rows * (self.dim + 2), rows, out.data_ptr(), out.stride(0), self._stream())
        _lib.check(rc, "pkv_lse_combine")
        return out


def polar_scores(q_rot: torch.Tensor, k_codes: torch.Tensor, q_params, bits) -> torch.Tensor:
    """Dense scores of ``prismkv_cuda.polar_attn_fwd`` (see pkv_polar_scores)."""
    _lib.require_cuda(q_rot, "Q")
    _lib.require_cuda(k_codes, "K_codes")
    if q_rot.dim() != 4 or k_codes.dim() != 4:
        raise RuntimeError("Q must be (B, H, Sq, d) and K_codes (B, H, Sk, m)")
    B, H, Sq, d = q_rot.shape
    B2, H2, Sk, m = k_codes.shape
    if (B, H) != (B2, H2):
        raise RuntimeError("K_codes batch/head dims must match Q")
    if d != 3 * m:
        raise RuntimeError(f"Q head_dim d must equal 3 * m (K_codes triplet count); got d={d} m={m}")
    q = q_rot.float().contiguous()
    kc = k_codes.contiguous()
    if kc.dtype not in (torch.int16, torch.uint16, torch.uint8):
        kc = kc.to(torch.int16)
    cb = 1 if kc.dtype == torch.uint8 else 2
    out = torch.empty((B, H, Sq, Sk), dtype=torch.float32, device=q.device)
    qp = (ctypes.c_float * 6)(*[float(v) for v in q_params])
    bt = (ctypes.c_int32 * 3)(*[int(v) for v in bits])
    lib = _lib.load()
    with torch.cuda.device(q.device):
        rc = lib.pkv_polar_scores(q.data_ptr(), kc.data_ptr(), cb, B, H, Sq, Sk, d, qp, bt, out.data_ptr(),
                                  _lib.stream_ptr(q.device))
    _lib.check(rc, "pkv_polar_scores")
    return out
