"""The attention planner's kernel choice for the benchmark workloads and its edges,
through pkv_attn_describe.  Planning reads only the codec's shape fields and the
pointers' alignment and launches nothing, so it runs without a GPU (the SM count
falls back to the B200's 148)."""

import ctypes

import pytest

from prismkv_b200 import _lib

ALIGNED = 1 << 12                # stand-in device addresses: planning never dereferences them


def _codec(bits=(4, 4, 4), learned=False, bias=False, lloyd=False, fp32=False, r_max=9.8):
    c = _lib.PkvCodec()
    c.dim = 96
    c.bits_z, c.bits_r, c.bits_theta = bits
    c.xy_mode = 1 if learned else 0
    c.xy_per_z = 1 if (learned or bias) else 0
    c.r_max = r_max
    c.flags = 0 if (learned or bias or lloyd) else _lib.PKV_CODEC_Z_UNIFORM
    if fp32:
        c.flags |= _lib.PKV_CODEC_FP32_ATTN
    c.R = c.z_thr = c.r2_thr = c.th_thr = c.dec_z = c.dec_xy = ALIGNED
    c.codebook = ALIGNED if learned else None
    c.bias_xy = ALIGNED if bias else None
    return c


def _args(B, Hq, Hkv, S, bits, qdt=_lib.PKV_F32, splits=0):
    a = _lib.PkvAttnArgs()
    a.batch, a.q_heads, a.kv_heads, a.seq_len = B, Hq, Hkv, S
    a.q_dtype = qdt
    a.code_bytes = 1 if sum(bits) <= 8 else 2
    a.q = a.k_codes = a.v_codes = ALIGNED
    a.q_head_stride, a.q_batch_stride = 96, Hq * 96
    a.kv_head_stride, a.kv_batch_stride = S * 32, Hkv * S * 32
    a.scale = 96 ** -0.5
    a.num_splits = splits
    return a


def _plan(c, a):
    p = _lib.PkvAttnPlan()
    rc = _lib.load().pkv_attn_describe(ctypes.byref(c), ctypes.byref(a), ctypes.byref(p))
    assert rc == 0, _lib.load().pkv_strerror(rc)
    return p


BF16 = _lib.PKV_BF16


@pytest.mark.parametrize("name,codec_kw,args,kernel", [
    ("phi3-decode", {}, (8, 32, 32, 4096, (4, 4, 4), BF16), "attn_mha12_kernel"),
    ("aggressive-332", dict(bits=(3, 3, 2)), (32, 32, 32, 16384, (3, 3, 2), BF16), "attn_mha8_kernel"),
    ("learned-gqa", dict(learned=True, bias=True), (16, 32, 8, 32768, (4, 4, 4), BF16), "attn_tc_kernel"),
    ("longctx-splitseq", {}, (4, 32, 8, 131072, (4, 4, 4), BF16), "attn_gqa12_mma_kernel"),
    ("longctx, one rank of eight", {}, (4, 32, 8, 16384, (4, 4, 4), BF16), "attn_gqa12_mma_kernel"),
    ("group 8, 12-bit, fp32", {}, (2, 16, 2, 3000, (4, 4, 4), _lib.PKV_F32), "attn_gqa12_mma_kernel"),
    ("longctx, fp32 arithmetic asked for", dict(fp32=True), (4, 32, 8, 131072, (4, 4, 4), BF16),
     "attn_gqa12_kernel"),
    ("longctx, radii past the fp16 pairs", dict(r_max=1e5), (4, 32, 8, 131072, (4, 4, 4), BF16),
     "attn_gqa12_kernel"),
    ("group 2, 12-bit: one query head per unit", {}, (2, 8, 4, 3000, (4, 4, 4), BF16), "attn_mha12_kernel"),
    ("group 2, long: one query head per unit", {}, (2, 8, 4, 9000, (4, 4, 4), BF16), "attn_mha12_stream_kernel"),
    ("cpu-roundtrip", {}, (1, 8, 8, 1024, (4, 4, 4), _lib.PKV_F32), "attn_mha12_kernel"),
    ("learned, fp32 queries", dict(learned=True, bias=True), (2, 32, 8, 4096, (4, 4, 4), _lib.PKV_F32),
     "attn_lut_kernel"),
    ("Lloyd-Max z, one-byte codes", dict(bits=(3, 3, 2), lloyd=True), (2, 8, 8, 4096, (3, 3, 2), BF16),
     "attn_polar_kernel"),
    ("64 (r, theta) cells, one-byte codes", dict(bits=(2, 3, 3)), (2, 8, 8, 4096, (2, 3, 3), BF16),
     "attn_polar_kernel"),
    ("grouped one-byte, bf16", dict(bits=(3, 3, 2)), (2, 32, 8, 4096, (3, 3, 2), BF16), "attn_tc_kernel"),
    ("grouped one-byte, fp32", dict(bits=(3, 3, 2)), (2, 32, 8, 4096, (3, 3, 2), _lib.PKV_F32),
     "attn_mha8_kernel"),
    ("just past one item", {}, (1, 8, 8, 4097, (4, 4, 4), BF16), "attn_mha12_stream_kernel"),
])
def test_planner_picks_kernel(name, codec_kw, args, kernel):
    p = _plan(_codec(**codec_kw), _args(*args))
    assert _lib.KERNEL_NAMES[p.kernel] == kernel, name
    assert p.num_splits >= 1 and 0 < p.smem_bytes <= 227 * 1024 and p.threads % 32 == 0


def test_planner_splits_cover_the_sequence():
    for S in (1, 255, 4096, 4097, 20000, 131072):
        for bits in ((4, 4, 4), (3, 3, 2)):
            p = _plan(_codec(bits=bits), _args(2, 8, 8, S, bits, BF16))
            assert p.num_splits * p.tokens_per_split >= S
            assert (p.num_splits - 1) * p.tokens_per_split < S


def test_planner_honours_forced_splits():
    p = _plan(_codec(), _args(1, 8, 8, 12345, (4, 4, 4), BF16, splits=5))
    assert p.num_splits == 5


def test_one_head_kernels_fill_the_grid():
    """One CTA per SM for the one-byte and the grouped 12-bit kernels, two for the one-head 12-bit kernels."""
    assert _plan(_codec(bits=(3, 3, 2)), _args(32, 32, 32, 16384, (3, 3, 2), BF16)).ctas_per_sm == 1
    assert _plan(_codec(), _args(8, 32, 32, 4096, (4, 4, 4), BF16)).ctas_per_sm == 2
    assert _plan(_codec(), _args(8, 32, 32, 8192, (4, 4, 4), BF16)).ctas_per_sm == 2
    assert _plan(_codec(), _args(4, 32, 8, 131072, (4, 4, 4), BF16)).ctas_per_sm == 1


def test_grouped_12bit_kernel_streams_balanced_ranges():
    """longctx (32 units of 131072 tokens on 148 SMs): every CTA streams an equal share of tiles."""
    p = _plan(_codec(), _args(4, 32, 8, 131072, (4, 4, 4), BF16))
    assert p.balanced == 1 and p.smem_bytes <= 227 * 1024 and p.threads == 16 * 32
    p = _plan(_codec(fp32=True), _args(4, 32, 8, 131072, (4, 4, 4), BF16))
    assert p.balanced == 1 and p.smem_bytes <= 227 * 1024 and p.threads == 20 * 32


@pytest.mark.parametrize("world", [1, 2, 8])
def test_exchange_layout_holds_flagged_slots_for_two_calls(world):
    """The split-sequence exchange buffer: partial slots of 8-byte (value, call flag) words for
    two call parities and every rank, then the output rows, then the control words."""
    B, Hq, Hkv, S = 4, 32, 8, 16384
    lay = _lib.PkvXrLayout()
    rc = _lib.load().pkv_xr_layout_for(ctypes.byref(_codec()), ctypes.byref(_args(B, Hq, Hkv, S, (4, 4, 4), BF16)),
                                       world, ctypes.byref(lay))
    assert rc == 0
    rows = B * Hq
    assert lay.rows == rows and lay.units == B * Hq // 4          # grouped 12-bit: four query heads a unit
    assert lay.out_offset % 256 == 0 and lay.out_offset >= 2 * world * rows * (96 + 2) * 8
    assert lay.bytes >= lay.out_offset + rows * 96 * 4 + 8
    bad = _lib.load().pkv_xr_layout_for(ctypes.byref(_codec()), ctypes.byref(_args(B, Hq, Hkv, S, (4, 4, 4), BF16)),
                                        _lib.XR_MAX_RANKS + 1, ctypes.byref(lay))
    assert bad != 0
