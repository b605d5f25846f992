"""GPU parity of the fused dequant + flash-decoding kernel (pkv_attn_decode).

Outputs are compared with the oracle's fp64 attention over the same codes
(and with the reference's own outputs in the golden fixtures).  Tolerance:
max abs error <= 1e-3 for every query dtype on the fp32 kernels (the stated
bound for bf16 queries is 2e-2; those kernels compute in fp32 on the exactly
upcast query), 2e-2 on the tensor-core kernel, whose operands are bf16/fp16.
"""

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden, params_from, quantizer_from
from prismkv_b200 import BiasTable, LearnedSliceCodebook, StackedPlaneQuantizer, decode_attention
from prismkv_b200.synthetic import synthetic_bias, synthetic_codebook

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-3
TOL_TC = 2e-2       # bf16 / fp16 queries on the tensor-core kernel (bf16 operands): the stated bf16 bound


def test_attention_matches_reference_polar_attention(cuda_ready):
    f = load_golden("attn_v1")
    q = quantizer_from(f)
    qt = torch.from_numpy(f["q"]).to(DEV)
    out = decode_attention(q, qt, torch.from_numpy(f["k_codes"]).to(DEV), torch.from_numpy(f["v_codes"]).to(DEV))
    np.testing.assert_allclose(out.cpu().numpy(), f["out"][:, :, 0], atol=TOL)


def test_attention_matches_reference_learned_gqa(cuda_ready):
    f = load_golden("attn_v2_gqa")
    q = quantizer_from(f)
    out = decode_attention(q, torch.from_numpy(f["q"]).to(DEV), torch.from_numpy(f["k_codes"]).to(DEV),
                           torch.from_numpy(f["v_codes"]).to(DEV))
    np.testing.assert_allclose(out.cpu().numpy(), f["out"][:, :, 0], atol=TOL)


def _setup(variant, bits, dim=96, seed=0):
    q = StackedPlaneQuantizer(dim, *bits, seed=42)
    Cz, K = 1 << bits[0], 1 << (bits[1] + bits[2])
    if "learned" in variant:
        q._codebooks = LearnedSliceCodebook(synthetic_codebook(Cz, K, q.r_max, 11), Cz, K, q.z_min, q.z_max, q.r_max)
    if "bias" in variant:
        q._bias = BiasTable(synthetic_bias(Cz, 12), delta_z=(q.z_max - q.z_min) / Cz)
    if "lloyd" in variant:
        q.calibrate_lloyd_max_z(torch.randn(2048, dim, generator=torch.Generator().manual_seed(5)).to(DEV))
    p = oracle.QuantParams(dim=dim, bits_z=bits[0], bits_r=bits[1], bits_theta=bits[2],
                           z_min=q.z_min, z_max=q.z_max, r_max=q.r_max)
    if q._codebooks is not None:
        p.codebook = q._codebooks.codebooks.numpy()
    if q._lloyd_max_z is not None:
        p.lloyd_boundaries = q._lloyd_max_z.boundaries.numpy()
        p.lloyd_centroids = q._lloyd_max_z.centroids.numpy()
    if q._bias is not None:
        p.bias_table = q._bias.table.numpy()
        p.bias_delta_z = q._bias.delta_z
    return q, p


def _codes(q, B, H, S, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    k = torch.randn(B * H * S, q.dim, generator=g, device=DEV)
    v = torch.randn(B * H * S, q.dim, generator=g, device=DEV) * 1.5
    kc = q.encode_compact(k).view(B, H, S, q.m)
    vc = q.encode_compact(v).view(B, H, S, q.m)
    return kc, vc


CASES = [
    # B, Hq, Hkv, S, variant, bits, qdtype, splits
    (1, 8, 8, 1024, "v1", (4, 4, 4), torch.float32, 0),          # cpu-roundtrip shape
    (2, 8, 8, 1, "v1", (4, 4, 4), torch.float32, 0),
    (2, 8, 8, 3, "v1", (4, 4, 4), torch.float32, 0),
    (2, 8, 8, 63, "v1", (4, 4, 4), torch.bfloat16, 0),
    (2, 8, 8, 65, "v1", (4, 4, 4), torch.float16, 0),
    (2, 8, 8, 257, "v1", (4, 4, 4), torch.float32, 0),
    (2, 32, 8, 1000, "learned_bias", (4, 4, 4), torch.bfloat16, 0),  # learned-gqa shape, short
    (1, 4, 4, 700, "lloyd", (4, 4, 4), torch.float32, 0),
    (1, 8, 4, 900, "lloyd_learned_bias", (4, 4, 4), torch.float32, 0),
    (2, 4, 4, 513, "v1", (3, 3, 2), torch.float32, 0),            # uint8 codes (one-byte kernel)
    (2, 8, 8, 1, "v1", (3, 3, 2), torch.float32, 0),
    (2, 8, 8, 255, "v1", (3, 3, 2), torch.bfloat16, 0),
    (1, 8, 8, 4100, "v1", (3, 3, 2), torch.float32, 3),
    (2, 16, 4, 777, "v1", (3, 3, 2), torch.float32, 0),           # grouped fp32: one query head per unit
    (1, 32, 2, 600, "v1", (3, 3, 2), torch.float32, 2),           # group 16
    (1, 6, 2, 300, "v1", (3, 3, 2), torch.float16, 0),            # grouped fp16: tensor cores
    (2, 4, 4, 600, "v1", (4, 2, 2), torch.float32, 0),
    (2, 4, 4, 600, "v1", (3, 2, 3), torch.float32, 0),
    (2, 4, 4, 600, "v1", (2, 3, 3), torch.float32, 0),            # 64 (r, theta) cells: polar kernel
    (1, 4, 4, 700, "lloyd", (3, 3, 2), torch.float32, 0),
    (2, 4, 4, 513, "learned", (3, 3, 2), torch.float32, 0),
    (1, 4, 2, 300, "v1", (4, 4, 4), torch.float32, 0),            # group 2
    (1, 16, 2, 300, "v1", (4, 4, 4), torch.float32, 0),           # group 8
    (1, 6, 2, 100, "v1", (4, 4, 4), torch.float32, 0),            # group 3 (padded to 4)
    (2, 8, 4, 2000, "v1", (4, 4, 4), torch.float32, 1),
    (2, 8, 4, 2000, "v1", (4, 4, 4), torch.float32, 2),
    (2, 8, 4, 2000, "v1", (4, 4, 4), torch.float32, 7),
    (2, 8, 4, 2000, "v1", (4, 4, 4), torch.float32, 16),
    (1, 8, 8, 5000, "v1", (4, 4, 4), torch.float32, 0),           # past 4096 tokens: one-pass 12-bit kernel
    (2, 8, 8, 4097, "v1", (4, 4, 4), torch.bfloat16, 0),
    (1, 32, 8, 9000, "v1", (4, 4, 4), torch.float32, 0),          # group 4: four heads per unit
    (2, 16, 4, 3000, "v1", (4, 4, 4), torch.bfloat16, 0),         # group 4, bf16 queries
    (1, 8, 2, 777, "v1", (4, 4, 4), torch.float16, 0),            # group 4, partial tiles
    (2, 32, 4, 5000, "v1", (4, 4, 4), torch.float32, 0),          # group 8: two units per KV head
    (1, 16, 4, 20000, "v1", (4, 4, 4), torch.float32, 3),         # group 4, forced splits
    (1, 4, 1, 1, "v1", (4, 4, 4), torch.float32, 0),              # group 4, one token
    (1, 64, 4, 600, "v1", (4, 4, 4), torch.bfloat16, 0),          # group 16
    (1, 8, 8, 12345, "v1", (4, 4, 4), torch.float16, 5),
]


@pytest.mark.parametrize("B,Hq,Hkv,S,variant,bits,qdt,splits", CASES)
def test_attention_matches_oracle(cuda_ready, B, Hq, Hkv, S, variant, bits, qdt, splits):
    q, p = _setup(variant, bits)
    kc, vc = _codes(q, B, Hkv, S, seed=S + Hq)
    qv = torch.randn(B, Hq, 96, generator=torch.Generator(device=DEV).manual_seed(7), device=DEV).to(qdt)
    out = decode_attention(q, qv, kc, vc, num_splits=splits)
    ref = oracle.attention(qv.float().cpu().numpy(), kc.cpu().numpy().astype(np.int64),
                           vc.cpu().numpy().astype(np.int64), q.R.numpy(), p)
    codec = q.codec(torch.device(DEV))
    plan = codec.describe(qv, kc, vc)
    tol = TOL_TC if plan["kernel"] == "attn_tc_kernel" else TOL
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=tol, rtol=0)
    if plan["kernel"] == "attn_gqa12_mma_kernel":          # and the same groups on the fp32 kernel
        codec.fp32_attention = True
        try:
            assert codec.describe(qv, kc, vc)["kernel"] == "attn_gqa12_kernel"
            out32 = decode_attention(q, qv, kc, vc, num_splits=splits)
        finally:
            codec.fp32_attention = False
        np.testing.assert_allclose(out32.cpu().numpy(), ref, atol=TOL, rtol=0)


@pytest.mark.parametrize("dim", [66, 192, 129])
def test_attention_other_head_dims(cuda_ready, dim):
    """d=66 (GPT-2 64 padded; 44-byte rows -> plain-load path), d=192 (two triplets per lane)."""
    q, p = _setup("v1", (4, 4, 4), dim=dim)
    kc, vc = _codes(q, 1, 4, 300, seed=dim)
    qv = torch.randn(1, 4, dim, generator=torch.Generator(device=DEV).manual_seed(1), device=DEV)
    out = decode_attention(q, qv, kc, vc)
    ref = oracle.attention(qv.cpu().numpy(), kc.cpu().numpy().astype(np.int64), vc.cpu().numpy().astype(np.int64),
                           q.R.numpy(), p)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL, rtol=0)


@pytest.mark.parametrize("bits,S,Hq", [((4, 4, 4), 512, 8), ((3, 3, 2), 512, 8), ((4, 4, 4), 6000, 8),
                                       ((4, 4, 4), 6000, 32)])
def test_attention_ragged_and_empty_rows(cuda_ready, bits, S, Hq):
    q, p = _setup("v1", bits)
    kc, vc = _codes(q, 3, 8, S, seed=2)
    qv = torch.randn(3, Hq, 96, generator=torch.Generator(device=DEV).manual_seed(2), device=DEV)
    lens = torch.tensor([S, 0, 77 if S < 1000 else 4500], dtype=torch.int32, device=DEV)
    for splits in (0, 1, 3):
        out = decode_attention(q, qv, kc, vc, seq_lens=lens, num_splits=splits)
        ref = oracle.attention(qv.cpu().numpy(), kc.cpu().numpy().astype(np.int64), vc.cpu().numpy().astype(np.int64),
                               q.R.numpy(), p, seq_lens=lens.cpu().numpy())
        np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL, rtol=0)
        assert (out[1] == 0).all()


def test_attention_capacity_strided_cache(cuda_ready):
    """Codes inside a larger preallocated cache (head stride = capacity * m)."""
    q, p = _setup("v1", (4, 4, 4))
    cap, S = 1000, 640
    kfull, vfull = _codes(q, 2, 4, cap, seed=3)
    kc, vc = kfull[:, :, :S], vfull[:, :, :S]
    qv = torch.randn(2, 4, 96, generator=torch.Generator(device=DEV).manual_seed(3), device=DEV)
    out = decode_attention(q, qv, kc, vc)
    ref = oracle.attention(qv.cpu().numpy(), kc.cpu().numpy().astype(np.int64), vc.cpu().numpy().astype(np.int64),
                           q.R.numpy(), p)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL, rtol=0)


@pytest.mark.parametrize("Hq,H", [(8, 8), (32, 8)])
def test_attention_partials_and_lse_combine(cuda_ready, Hq, H):
    """Shard the sequence (uneven, one empty shard), keep partials, merge: equals unsplit.
    MHA runs the one-head 12-bit kernel, groups of four the grouped kernel."""
    q, p = _setup("v1", (4, 4, 4))
    B, S = 2, 1500
    G = Hq // H
    kc, vc = _codes(q, B, H, S, seed=4)
    qv = torch.randn(B, Hq, 96, generator=torch.Generator(device=DEV).manual_seed(4), device=DEV)
    codec = q.codec(torch.device(DEV))
    bounds = [0, 700, 700, 1500]
    parts = []
    for a, b in zip(bounds[:-1], bounds[1:]):
        parts.append(codec.attention(qv, kc[:, :, a:b], vc[:, :, a:b], partial=True).view(B * Hq, 98))
    merged = codec.combine(torch.stack(parts)).view(B, Hq, 96)
    ref = oracle.attention(qv.cpu().numpy(), kc.cpu().numpy().astype(np.int64), vc.cpu().numpy().astype(np.int64),
                           q.R.numpy(), p)
    np.testing.assert_allclose(merged.cpu().numpy(), ref, atol=TOL, rtol=0)
    # partial contents against an fp64 restatement (natural-log max, l, o in rotated space)
    pa = parts[0].view(B, Hq, 98).cpu().numpy().astype(np.float64)
    kr = oracle.dequant_rotated(kc[:, :, :700].cpu().numpy().reshape(-1, 32), p).reshape(B, H, 700, 96)
    vr = oracle.dequant_rotated(vc[:, :, :700].cpu().numpy().reshape(-1, 32), p).reshape(B, H, 700, 96)
    kr = np.repeat(kr, G, axis=1)
    vr = np.repeat(vr, G, axis=1)
    qr = qv.cpu().numpy().astype(np.float64) @ q.R.numpy().astype(np.float64).T
    s = np.einsum("bhd,bhsd->bhs", qr, kr) * 96 ** -0.5
    mx = s.max(-1)
    w = np.exp(s - mx[..., None])
    np.testing.assert_allclose(pa[..., 0], mx, atol=1e-4)
    np.testing.assert_allclose(pa[..., 1], w.sum(-1), rtol=1e-4)
    np.testing.assert_allclose(pa[..., 2:], np.einsum("bhs,bhsd->bhd", w, vr), rtol=1e-4, atol=1e-3)
    empty = parts[1].view(B, Hq, 98)
    assert torch.isinf(empty[..., 0]).all() and (empty[..., 1:] == 0).all()


def test_attention_repeated_calls_reuse_workspace(cuda_ready):
    q, _ = _setup("v1", (4, 4, 4))
    kc, vc = _codes(q, 2, 8, 3000, seed=5)
    qv = torch.randn(2, 8, 96, generator=torch.Generator(device=DEV).manual_seed(5), device=DEV)
    outs = [decode_attention(q, qv, kc, vc, num_splits=6).clone() for _ in range(4)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    from prismkv_b200 import _lib
    assert _lib.device_error() == 0


def test_attention_shapes_in_turn_share_workspace(cuda_ready):
    """Calls of different shapes through one per-stream workspace: the arrival
    counters of each shape sit at a different offset, so every call must leave
    the whole workspace (partials included) zeroed for the next one."""
    q, p = _setup("v1", (4, 4, 4))
    cases = [(4, 8, 20000, 0), (1, 2, 5000, 5), (3, 4, 7000, 4), (4, 8, 20000, 0)]
    data = []
    for i, (B, H, S, ns) in enumerate(cases):
        kc, vc = _codes(q, B, H, S, seed=20 + i % 3)
        qv = torch.randn(B, H, 96, generator=torch.Generator(device=DEV).manual_seed(i % 3), device=DEV)
        data.append((qv, kc, vc, ns))
    for qv, kc, vc, ns in data:
        out = decode_attention(q, qv, kc, vc, num_splits=ns)
        ref = oracle.attention(qv.cpu().numpy(), kc.cpu().numpy().astype(np.int64),
                               vc.cpu().numpy().astype(np.int64), q.R.numpy(), p)
        np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL, rtol=0)


@pytest.mark.parametrize("B,Hq,Hkv,S,variant,bits,kernel", [
    (8, 32, 32, 4096, "v1", (4, 4, 4), "attn_mha12_kernel"),
    (4, 32, 8, 4096, "v1", (4, 4, 4), "attn_gqa12_mma_kernel"),    # grouped heads: four per unit
    (4, 16, 8, 4096, "v1", (4, 4, 4), "attn_mha12_kernel"),        # group 2: one query head per unit
    (1, 8, 8, 4097, "v1", (4, 4, 4), "attn_mha12_stream_kernel"),
    (4, 32, 8, 131072, "v1", (4, 4, 4), "attn_gqa12_mma_kernel"),
    (2, 8, 8, 4096, "v1", (3, 3, 2), "attn_mha8_kernel"),
    (2, 32, 8, 4096, "v1", (3, 3, 2), "attn_mha8_kernel"),        # fp32 queries of a group
    (2, 8, 8, 4096, "v1", (2, 3, 3), "attn_polar_kernel"),
    (2, 8, 8, 4096, "lloyd", (3, 3, 2), "attn_polar_kernel"),
    (2, 8, 8, 4096, "lloyd_bias", (4, 4, 4), "attn_polar_kernel"),
    (2, 32, 8, 4096, "learned_bias", (4, 4, 4), "attn_lut_kernel"),
])
def test_attention_plan_picks_kernel(cuda_ready, B, Hq, Hkv, S, variant, bits, kernel):
    q, _ = _setup(variant, bits)
    kc = torch.zeros(B, Hkv, S, q.m, dtype=q.code_dtype, device=DEV)
    plan = q.codec(torch.device(DEV)).describe(torch.zeros(B, Hq, 96, device=DEV), kc, kc)
    assert plan["kernel"] == kernel
    assert plan["num_splits"] >= 1 and plan["smem_bytes"] <= 227 * 1024


def test_fp32_flag_plans_the_fp32_grouped_kernel(cuda_ready):
    q, _ = _setup("v1", (4, 4, 4))
    kc = torch.zeros(4, 8, 4096, q.m, dtype=q.code_dtype, device=DEV)
    codec = q.codec(torch.device(DEV))
    qv = torch.zeros(4, 32, 96, device=DEV)
    codec.fp32_attention = True
    try:
        assert codec.describe(qv, kc, kc)["kernel"] == "attn_gqa12_kernel"
    finally:
        codec.fp32_attention = False
    assert codec.describe(qv, kc, kc)["kernel"] == "attn_gqa12_mma_kernel"


def _ref_attention(q, p, qv, kc, vc):
    return oracle.attention(qv.float().cpu().numpy(), kc.cpu().numpy().astype(np.int64),
                            vc.cpu().numpy().astype(np.int64), q.R.numpy(), p)


@pytest.mark.parametrize("case", ["huge_q", "tiny_q", "zero_q", "peaked", "one_token", "two_tokens", "mixed_rows"])
def test_grouped_tensor_core_numerics(cuda_ready, case):
    """The fp16-pair tensor-core kernel at the edges of its operand scaling: queries of 1e4 and of
    1e-7 (the per-item power-of-two scale), all-zero queries (uniform weights), one key far above
    the rest (weights down to exp2(-30) of the largest), one and two tokens (no averaging of
    rounding), and rows of very different scales in one call.  Max error 1e-3 against the oracle."""
    q, p = _setup("v1", (4, 4, 4))
    S = {"one_token": 1, "two_tokens": 2}.get(case, 700)
    B, Hq, Hkv = 2, 8, 2
    kc, vc = _codes(q, B, Hkv, S, seed=91)
    g = torch.Generator(device=DEV).manual_seed(92)
    qv = torch.randn(B, Hq, 96, generator=g, device=DEV)
    if case == "huge_q":
        qv *= 1e4
    elif case == "tiny_q":
        qv *= 1e-7
    elif case == "zero_q":
        qv.zero_()
    elif case == "peaked":
        # the query of every head points along key token 5 of its KV head (decoded), scaled so
        # that token's score leads the others by about 30 (log2 units)
        kd = q.decode(kc[:, :, 5].reshape(-1, q.m)).view(B, Hkv, 96)
        qv = kd.repeat_interleave(Hq // Hkv, dim=1) * 3.0
    elif case == "mixed_rows":
        qv[0] *= 1e3
        qv[1] *= 1e-3
    codec = q.codec(torch.device(DEV))
    assert codec.describe(qv, kc, vc)["kernel"] == "attn_gqa12_mma_kernel"
    out = decode_attention(q, qv, kc, vc)
    ref = _ref_attention(q, p, qv, kc, vc)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL, rtol=0)
    from prismkv_b200 import _lib
    assert _lib.device_error() == 0


def test_attention_balanced_schedule(cuda_ready):
    """Learned codebooks (one-pass kernel) over 128 KV heads x 4096 tokens: the planner gives
    every CTA an equal share of token tiles, cutting segments across (batch, kv head) ends;
    the segments merge through the workspace counters."""
    q, p = _setup("learned_bias", (4, 4, 4))
    B, Hq, Hkv, S = 16, 32, 8, 4096
    kc, vc = _codes(q, B, Hkv, S, seed=31)
    qv = torch.randn(B, Hq, 96, generator=torch.Generator(device=DEV).manual_seed(31), device=DEV)
    codec = q.codec(torch.device(DEV))
    plan = codec.describe(qv, kc, vc)
    assert plan["kernel"] == "attn_lut_kernel" and plan["balanced"] == 1
    ref = oracle.attention(qv.cpu().numpy(), kc.cpu().numpy().astype(np.int64), vc.cpu().numpy().astype(np.int64),
                           q.R.numpy(), p)
    for _ in range(2):
        out = decode_attention(q, qv, kc, vc)
        np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL, rtol=0)
    from prismkv_b200 import _lib
    assert _lib.device_error() == 0


def test_phi3_decode_full_size(cuda_ready):
    """The benchmark workload at full size (B=8, 32 heads, S=4096) against the oracle."""
    from prismkv_b200.synthetic import WORKLOADS, make_kv_codes, make_query, make_quantizer
    w = WORKLOADS["phi3-decode"]
    q = make_quantizer(w)
    kc, vc = make_kv_codes(w, q, DEV)
    qv = make_query(w, DEV)
    out = decode_attention(q, qv, kc, vc)
    p = oracle.QuantParams.default(96)
    ref = oracle.attention(qv.float().cpu().numpy(), kc.cpu().numpy().astype(np.int64),
                           vc.cpu().numpy().astype(np.int64), q.R.numpy(), p)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL, rtol=0)


def test_aggressive_decode_full_size(cuda_ready):
    """The batch-sharded 8-bit workload at full size (B=32, 32 heads, S=16384, 3+3+2) through the
    one-byte kernel; three batch rows against the oracle."""
    from prismkv_b200.synthetic import WORKLOADS, make_kv_codes, make_query, make_quantizer
    w = WORKLOADS["aggressive-332"]
    q = make_quantizer(w)
    kc, vc = make_kv_codes(w, q, DEV)
    qv = make_query(w, DEV)
    assert q.codec(torch.device(DEV)).describe(qv, kc, vc)["kernel"] == "attn_mha8_kernel"
    out = decode_attention(q, qv, kc, vc)
    p = oracle.QuantParams(dim=96, bits_z=3, bits_r=3, bits_theta=2, z_min=q.z_min, z_max=q.z_max, r_max=q.r_max)
    rows = [0, 17, 31]
    ref = oracle.attention(qv[rows].float().cpu().numpy(), kc[rows].cpu().numpy().astype(np.int64),
                           vc[rows].cpu().numpy().astype(np.int64), q.R.numpy(), p)
    np.testing.assert_allclose(out[rows].cpu().numpy(), ref, atol=TOL, rtol=0)


def test_longctx_full_size_with_outliers(cuda_ready):
    """The split-sequence workload at full size on one GPU (B=4, 32 query / 8 KV heads, S=131072,
    1 % of the channels x8 before the rotation) through the grouped 12-bit kernels (tensor-core
    and fp32); two (batch, KV head) units -- eight query heads -- against the oracle at the fp32
    bound, and all units of the two kernels against each other."""
    from prismkv_b200.synthetic import WORKLOADS, make_kv_codes, make_query, make_quantizer
    w = WORKLOADS["longctx-splitseq"]
    q = make_quantizer(w)
    kc, vc = make_kv_codes(w, q, DEV)
    qv = make_query(w, DEV)
    codec = q.codec(torch.device(DEV))
    assert codec.describe(qv, kc, vc)["kernel"] == "attn_gqa12_mma_kernel"
    out = decode_attention(q, qv, kc, vc)
    codec.fp32_attention = True
    try:
        assert codec.describe(qv, kc, vc)["kernel"] == "attn_gqa12_kernel"
        out32 = decode_attention(q, qv, kc, vc)
    finally:
        codec.fp32_attention = False
    p = oracle.QuantParams.default(96)
    for b, hk in ((0, 0), (3, 7)):
        ref = oracle.attention(qv[b:b + 1, 4 * hk:4 * hk + 4].float().cpu().numpy(),
                               kc[b:b + 1, hk:hk + 1].cpu().numpy().astype(np.int64),
                               vc[b:b + 1, hk:hk + 1].cpu().numpy().astype(np.int64), q.R.numpy(), p)
        for o in (out, out32):
            np.testing.assert_allclose(o[b:b + 1, 4 * hk:4 * hk + 4].cpu().numpy(), ref, atol=TOL, rtol=0)
    # every unit: the two kernels agree far inside the bound
    np.testing.assert_allclose(out.cpu().numpy(), out32.cpu().numpy(), atol=1e-4, rtol=0)
    from prismkv_b200 import _lib
    assert _lib.device_error() == 0


def test_learned_gqa_full_size(cuda_ready):
    """The learned-codebook workload at full size (B=16, 32 query / 8 KV heads, S=32768, 16x256
    codebooks + BiasTable, bf16 queries) on the tensor-core kernel; two units against the oracle at
    the bf16 bound."""
    from prismkv_b200.synthetic import WORKLOADS, make_kv_codes, make_query, make_quantizer
    w = WORKLOADS["learned-gqa"]
    q = make_quantizer(w)
    kc, vc = make_kv_codes(w, q, DEV)
    qv = make_query(w, DEV)
    assert q.codec(torch.device(DEV)).describe(qv, kc, vc)["kernel"] == "attn_tc_kernel"
    out = decode_attention(q, qv, kc, vc)
    p = oracle.QuantParams.default(96)
    p.codebook = q._codebooks.codebooks.numpy()
    p.bias_table = q._bias.table.numpy()
    p.bias_delta_z = q._bias.delta_z
    for b, hk in ((0, 0), (15, 5)):
        ref = oracle.attention(qv[b:b + 1, 4 * hk:4 * hk + 4].float().cpu().numpy(),
                               kc[b:b + 1, hk:hk + 1].cpu().numpy().astype(np.int64),
                               vc[b:b + 1, hk:hk + 1].cpu().numpy().astype(np.int64), q.R.numpy(), p)
        np.testing.assert_allclose(out[b:b + 1, 4 * hk:4 * hk + 4].cpu().numpy(), ref, atol=TOL_TC, rtol=0)
