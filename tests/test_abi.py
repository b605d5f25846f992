"""The C ABI library loads, exports every symbol the header declares, and
rejects malformed arguments with status codes (checks that run before any
CUDA call, so they need no GPU)."""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from prismkv_b200 import _lib

HEADER = os.path.join(ROOT, "include", "prismkv_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"PKV_API\s+[\w\s\*]+?\b(pkv_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_abi_version_and_strerror():
    lib = _lib.load()
    assert lib.pkv_abi_version() == 1
    assert lib.pkv_strerror(0) == b"ok"
    for code in range(1, 8):
        assert lib.pkv_strerror(code) and lib.pkv_strerror(code) != b"unknown status"
    assert lib.pkv_strerror(99) == b"unknown status"


def _codec(dim=96, bits=(4, 4, 4), R=1):
    c = _lib.PkvCodec()
    c.dim = dim
    c.bits_z, c.bits_r, c.bits_theta = bits
    c.R = R
    c.z_thr = c.r2_thr = c.th_thr = c.codebook = c.dec_z = c.dec_xy = 1
    return c


@pytest.mark.parametrize("kw,code", [
    (dict(dim=95), 1), (dict(dim=0), 1), (dict(dim=195), 2), (dict(bits=(0, 4, 4)), 1),
    (dict(bits=(9, 4, 4)), 1), (dict(bits=(8, 8, 8)), 1), (dict(R=None), 1)])
def test_encode_rejects_bad_codec(kw, code):
    lib = _lib.load()
    c = _codec(**kw)
    rc = lib.pkv_encode(ctypes.byref(c), 1, 0, 10, 96, 1, 2, 32, None)
    assert rc == code


def test_encode_rejects_bad_arguments_and_accepts_empty():
    lib = _lib.load()
    c = _codec()
    assert lib.pkv_encode(ctypes.byref(c), 1, 7, 10, 96, 1, 2, 32, None) == 1      # dtype
    assert lib.pkv_encode(ctypes.byref(c), 1, 0, 10, 96, 1, 3, 32, None) == 1      # code bytes
    assert lib.pkv_encode(ctypes.byref(c), 1, 0, 10, 96, 1, 1, 32, None) == 1      # 12-bit code in uint8
    assert lib.pkv_encode(ctypes.byref(c), 1, 0, 10, 95, 1, 2, 32, None) == 1      # row stride < dim
    assert lib.pkv_encode(ctypes.byref(c), None, 0, 10, 96, 1, 2, 32, None) == 1   # null input
    assert lib.pkv_encode(ctypes.byref(c), None, 0, 0, 96, None, 2, 32, None) == 0  # empty: no launch
    assert lib.pkv_decode(ctypes.byref(c), None, 2, 0, 32, None, 0, 96, None) == 0


def test_attention_rejects_bad_arguments():
    lib = _lib.load()
    c = _codec()
    a = _lib.PkvAttnArgs()
    a.batch, a.q_heads, a.kv_heads, a.seq_len = 1, 6, 4, 16       # 6 % 4 != 0
    a.code_bytes, a.scale = 2, 0.1
    a.q = a.k_codes = a.v_codes = a.out = 1
    a.kv_head_stride = 16 * 32
    assert lib.pkv_attn_decode(ctypes.byref(c), ctypes.byref(a), None, 0, None) == 1
    a.q_heads = 40                                              # group of 10 > 8
    assert lib.pkv_attn_decode(ctypes.byref(c), ctypes.byref(a), None, 0, None) == 2
    a.q_heads = 8
    a.kv_head_stride = 15 * 32                                  # overlapping heads
    assert lib.pkv_attn_decode(ctypes.byref(c), ctypes.byref(a), None, 0, None) == 1
    a.kv_head_stride = 16 * 32
    a.scale = float("nan")
    assert lib.pkv_attn_decode(ctypes.byref(c), ctypes.byref(a), None, 0, None) == 1
    a.scale = 0.1
    a.batch = 0
    assert lib.pkv_attn_decode(ctypes.byref(c), ctypes.byref(a), None, 0, None) == 0
    assert lib.pkv_attn_workspace_size(ctypes.byref(c), ctypes.byref(a)) == 0


def test_polar_scores_rejects_bad_arguments():
    lib = _lib.load()
    qp = (ctypes.c_float * 6)(-9.8, 1.2, 9.8, 0.6, 0.4, 0.1)
    bits = (ctypes.c_int32 * 3)(4, 4, 4)
    assert lib.pkv_polar_scores(1, 1, 2, 1, 1, 1, 1, 95, qp, bits, 1, None) == 1
    assert lib.pkv_polar_scores(1, 1, 1, 1, 1, 1, 1, 96, qp, bits, 1, None) == 1     # 12 bits in uint8
    assert lib.pkv_polar_scores(1, 1, 2, 0, 1, 1, 1, 96, qp, bits, 1, None) == 0     # empty


def test_product_raises_without_cuda_device():
    import torch
    from prismkv_b200 import StackedPlaneQuantizer
    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    q = StackedPlaneQuantizer(96)
    with pytest.raises(RuntimeError, match="CUDA"):
        q.encode(torch.randn(4, 96))
