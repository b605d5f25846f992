"""pkv_attn_decode_noalloc (split scratch in a static device array) against
pkv_attn_decode (caller workspace), both called through the C ABI.

The no-alloc entry point exists for callers that cannot allocate device
memory on the decode path; it must give the same outputs as the workspace
entry point on the same inputs.  Tolerance 1e-6 absolute: both run the same
kernel and merge, so any difference beyond float noise is a scratch bug.
Each case calls the no-alloc entry point twice in a row, which checks that a
call leaves the arrival counters at zero for the next one.  This file is
named to be collected last, so that a full run reaches it after every other
GPU test; it passes on its own too (``pytest tests/test_zz_no_alloc.py`` in a
fresh process), where its first call is the library's first touch of the
scratch array.
"""

import ctypes

import pytest
import torch

from prismkv_b200 import StackedPlaneQuantizer, _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-6


def _codes(q, B, H, S, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    k = torch.randn(B * H * S, q.dim, generator=g, device=DEV)
    v = torch.randn(B * H * S, q.dim, generator=g, device=DEV) * 1.5
    return q.encode_compact(k).view(B, H, S, q.m), q.encode_compact(v).view(B, H, S, q.m)


def _args(codec, qv, kc, vc, out, num_splits=0):
    return codec._attn_args(qv, kc, vc, codec.dim ** -0.5, None, out, num_splits, None)


def _noalloc(codec, a):
    lib = _lib.load()
    return lib.pkv_attn_decode_noalloc(ctypes.byref(codec.struct), ctypes.byref(a),
                                       torch.cuda.current_stream().cuda_stream)


def _workspace_bytes(codec, a):
    return _lib.load().pkv_attn_workspace_size(ctypes.byref(codec.struct), ctypes.byref(a))


CASES = [
    # B, Hq, Hkv, S, bits, qdtype, splits
    (2, 8, 8, 16384, (4, 4, 4), torch.bfloat16, 0),    # 12-bit one-pass kernel, planner's splits
    (1, 32, 8, 9000, (4, 4, 4), torch.float32, 0),     # GQA, one query head per unit
    (2, 4, 4, 3000, (2, 3, 3), torch.float16, 6),      # 8-bit codes (polar kernel), forced splits
    (1, 8, 8, 777, (4, 4, 4), torch.float32, 3),       # two-pass 12-bit kernel, ragged last split
    (2, 8, 8, 20000, (3, 3, 2), torch.float32, 0),     # one-byte kernel, planner's splits
    (1, 16, 4, 5000, (3, 3, 2), torch.bfloat16, 4),    # tensor-core kernel, forced splits
]


@pytest.mark.parametrize("B,Hq,Hkv,S,bits,qdt,splits", CASES)
def test_noalloc_matches_workspace_entry_point(cuda_ready, B, Hq, Hkv, S, bits, qdt, splits):
    q = StackedPlaneQuantizer(96, *bits, seed=42)
    codec = q.codec(torch.device(DEV))
    kc, vc = _codes(q, B, Hkv, S, seed=B * 131 + S)
    qv = torch.randn(B, Hq, 96, generator=torch.Generator(device=DEV).manual_seed(S), device=DEV).to(qdt)
    ref = codec.attention(qv, kc, vc, num_splits=splits)
    a_ref = _args(codec, qv, kc, vc, ref, splits)
    assert _workspace_bytes(codec, a_ref) > 0, "case must use split scratch"
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        rc = _noalloc(codec, _args(codec, qv, kc, vc, out, splits))
        _lib.check(rc, "pkv_attn_decode_noalloc")
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        torch.testing.assert_close(out, ref, atol=TOL, rtol=0)


def test_noalloc_shapes_in_turn_share_counters(cuda_ready):
    """A large split call, a small one whose partials would overlap the large
    call's counters under a workspace layout, then the large one again."""
    q = StackedPlaneQuantizer(96, 4, 4, 4, seed=42)
    codec = q.codec(torch.device(DEV))
    big = _codes(q, 4, 8, 20000, seed=1)
    small = _codes(q, 1, 2, 5000, seed=2)
    qb = torch.randn(4, 8, 96, device=DEV)
    qs = torch.randn(1, 2, 96, device=DEV)
    ref_b = codec.attention(qb, *big)
    ref_s = codec.attention(qs, *small, num_splits=5)
    for qv, (kc, vc), ref, ns in ((qb, big, ref_b, 0), (qs, small, ref_s, 5), (qb, big, ref_b, 0)):
        out = torch.full_like(ref, float("nan"))
        _lib.check(_noalloc(codec, _args(codec, qv, kc, vc, out, ns)), "pkv_attn_decode_noalloc")
        torch.cuda.synchronize()
        torch.testing.assert_close(out, ref, atol=TOL, rtol=0)


def test_noalloc_rejects_scratch_beyond_limit(cuda_ready):
    """64 x 32 heads x 16 splits x 98 floats = 12.8 MB of partials > 8 MiB - 64 KiB."""
    q = StackedPlaneQuantizer(96, 4, 4, 4, seed=42)
    codec = q.codec(torch.device(DEV))
    B, H, S = 64, 32, 4096
    kc = torch.zeros(B, H, S, 32, dtype=torch.int16, device=DEV)
    qv = torch.randn(B, H, 96, device=DEV)
    out = torch.full((B, H, 96), float("nan"), device=DEV)
    a = _args(codec, qv, kc, kc, out, 16)
    need = _workspace_bytes(codec, a)
    assert need - B * H * 4 > (8 << 20) - (64 << 10)
    rc = _noalloc(codec, a)
    assert rc == 7
    assert b"static array" in _lib.load().pkv_strerror(rc)
    torch.cuda.synchronize()
    assert torch.isnan(out).all()          # nothing was launched


def test_noalloc_without_splits_needs_no_scratch(cuda_ready):
    q = StackedPlaneQuantizer(96, 4, 4, 4, seed=42)
    codec = q.codec(torch.device(DEV))
    kc, vc = _codes(q, 64, 8, 300, seed=3)
    qv = torch.randn(64, 8, 96, device=DEV)
    ref = codec.attention(qv, kc, vc)
    out = torch.full_like(ref, float("nan"))
    a = _args(codec, qv, kc, vc, out)
    assert _workspace_bytes(codec, a) == 0
    _lib.check(_noalloc(codec, a), "pkv_attn_decode_noalloc")
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref, atol=TOL, rtol=0)
