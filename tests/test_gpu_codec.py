"""GPU parity of pkv_encode / pkv_decode against the oracle and the golden vectors.

Codes must equal the oracle's except at rounding ties proven by the fp64
classifier (oracle/ties.py); decoded vectors must agree to 1e-5 (fp32
output; the stated bound for fp32 is 1e-3) and bf16/fp16 outputs to their rounding.
"""

import numpy as np
import pytest
import torch

import oracle
from conftest import golden_files, load_golden, params_from, quantizer_from
from prismkv_b200 import StackedPlaneQuantizer, LearnedSliceCodebook, BiasTable, LloydMaxQuantizer1D
from prismkv_b200.synthetic import synthetic_bias, synthetic_codebook
from prismkv_b200 import tables

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIE_RATE = 1e-4          # mismatches allowed per code, all of which must be proven ties


def _mask(p):
    return (1 << (p.bits_z + p.bits_r + p.bits_theta)) - 1


@pytest.mark.parametrize("path", golden_files("enc_"), ids=lambda p: p.split("/")[-1])
def test_encode_matches_reference_golden(cuda_ready, path):
    f = load_golden(path)
    p = params_from(f)
    q = quantizer_from(f)
    codes = q.encode(torch.from_numpy(f["X"]).to(DEV)).cpu().numpy()
    rep = oracle.classify(f["X"], f["R"], p, codes, f["codes"].astype(np.int64) & _mask(p))
    assert rep.unexplained == 0, rep.examples
    assert rep.mismatches <= max(2, int(rep.total * TIE_RATE))


@pytest.mark.parametrize("path", golden_files("enc_"), ids=lambda p: p.split("/")[-1])
def test_decode_matches_reference_golden(cuda_ready, path):
    f = load_golden(path)
    q = quantizer_from(f)
    n = f["decoded"].shape[0]
    dec = q.decode(torch.from_numpy(f["codes"][:n].astype(np.int64)).to(DEV)).cpu().numpy()
    np.testing.assert_allclose(dec, f["decoded"], atol=1e-5, rtol=0)
    dall = q.decode(torch.from_numpy(f["all_codes"]).to(DEV)).cpu().numpy()   # every code value
    np.testing.assert_allclose(dall, f["decoded_all"], atol=1e-5, rtol=0)


def _quantizer(variant, bits):
    q = StackedPlaneQuantizer(96, *bits, seed=42)
    Cz, K = 1 << bits[0], 1 << (bits[1] + bits[2])
    if "learned" in variant:
        q._codebooks = LearnedSliceCodebook(synthetic_codebook(Cz, K, q.r_max, 11), Cz, K, q.z_min, q.z_max, q.r_max)
    if "bias" in variant:
        q._bias = BiasTable(synthetic_bias(Cz, 12), delta_z=(q.z_max - q.z_min) / Cz)
    if "lloyd" in variant:
        g = torch.Generator().manual_seed(5)
        q.calibrate_lloyd_max_z(torch.randn(2048, 96, generator=g).to(DEV))
    if "calib" in variant:
        g = torch.Generator().manual_seed(6)
        q.calibrate(torch.randn(4096, 96, generator=g).to(DEV), percentile_clip=0.005)
    return q


def _params(q):
    p = oracle.QuantParams(dim=q.dim, bits_z=q.bits_z, bits_r=q.bits_r, bits_theta=q.bits_theta,
                           z_min=q.z_min, z_max=q.z_max, r_max=q.r_max)
    if q._codebooks is not None:
        p.codebook = q._codebooks.codebooks.numpy()
    if q._lloyd_max_z is not None:
        p.lloyd_boundaries = q._lloyd_max_z.boundaries.numpy()
        p.lloyd_centroids = q._lloyd_max_z.centroids.numpy()
    if q._bias is not None:
        p.bias_table = q._bias.table.numpy()
        p.bias_delta_z = q._bias.delta_z
    return p


VARIANTS = [("v1", (4, 4, 4)), ("v1", (3, 3, 2)), ("v1", (2, 3, 1)), ("v1_calib", (4, 4, 4)),
            ("learned_bias", (4, 4, 4)), ("learned", (3, 3, 2)), ("lloyd", (4, 4, 4)),
            ("lloyd_learned_bias", (4, 4, 4)), ("v1", (5, 5, 6))]


@pytest.mark.parametrize("variant,bits", VARIANTS, ids=lambda v: str(v))
def test_encode_matches_oracle_seeded(cuda_ready, variant, bits):
    q = _quantizer(variant, bits)
    p = _params(q)
    g = torch.Generator().manual_seed(hash((variant, bits)) % 1000)
    X = torch.randn(40000 + 37, 96, generator=g) * (0.5 + 2.0 * torch.rand(40037, 1, generator=g))
    codes = q.encode(X.to(DEV)).cpu().numpy()
    ref = oracle.encode(X.numpy(), q.R.numpy(), p)
    rep = oracle.classify(X.numpy(), q.R.numpy(), p, codes, ref)
    assert rep.unexplained == 0, rep.examples
    assert rep.mismatches <= max(3, int(rep.total * TIE_RATE)), rep.as_dict()
    # compact storage holds the same values
    compact = q.encode_compact(X.to(DEV)).cpu().numpy().astype(np.int64) & _mask(p)
    np.testing.assert_array_equal(compact, codes)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_encode_half_inputs(cuda_ready, dtype):
    q = _quantizer("v1", (4, 4, 4))
    p = _params(q)
    g = torch.Generator().manual_seed(9)
    X = torch.randn(20000, 96, generator=g).to(dtype)
    codes = q.encode(X.to(DEV)).cpu().numpy()
    X32 = X.float().numpy()
    rep = oracle.classify(X32, q.R.numpy(), p, codes, oracle.encode(X32, q.R.numpy(), p))
    assert rep.unexplained == 0


@pytest.mark.parametrize("variant,bits", [("v1", (4, 4, 4)), ("learned_bias", (4, 4, 4)),
                                          ("lloyd", (4, 4, 4)), ("v1", (3, 3, 2))], ids=str)
@pytest.mark.parametrize("out_dtype,tol", [(torch.float32, 0.0), (torch.bfloat16, 2.0 ** -8), (torch.float16, 2.0 ** -11)])
def test_decode_matches_oracle(cuda_ready, variant, bits, out_dtype, tol):
    q = _quantizer(variant, bits)
    p = _params(q)
    g = torch.Generator().manual_seed(3)
    codes = torch.randint(0, 1 << sum(bits), (30011, 32), generator=g)
    ref = oracle.decode(codes.numpy(), q.R.numpy(), p)
    out = q.codec(torch.device(DEV)).decode(codes.to(DEV), out_dtype=out_dtype).float().cpu().numpy()
    # fp32: GEMM rounding; bf16/fp16: one rounding of the fp32 result (half an ulp, relative)
    np.testing.assert_allclose(out, ref, atol=1e-5, rtol=tol)


@pytest.mark.parametrize("n", [0, 1, 63, 64, 65, 127, 128, 129, 4097])
def test_encode_decode_edge_sizes(cuda_ready, n):
    q = _quantizer("v1", (4, 4, 4))
    p = _params(q)
    g = torch.Generator().manual_seed(n)
    X = torch.randn(n, 96, generator=g)
    codes = q.encode(X.to(DEV))
    assert codes.shape == (n, 32) and codes.dtype == torch.int64
    ref = oracle.encode(X.numpy(), q.R.numpy(), p)
    assert oracle.classify(X.numpy(), q.R.numpy(), p, codes.cpu().numpy(), ref).unexplained == 0
    dec = q.decode(codes)
    assert dec.shape == (n, 96)
    np.testing.assert_allclose(dec.cpu().numpy(), oracle.decode(codes.cpu().numpy(), q.R.numpy(), p), atol=1e-5)


def test_strided_input_and_output(cuda_ready):
    q = _quantizer("v1", (4, 4, 4))
    g = torch.Generator().manual_seed(4)
    wide = torch.randn(1000, 130, generator=g).to(DEV)
    X = wide[:, 7:103]                                     # row stride 130
    codec = q.codec(torch.device(DEV))
    out = torch.full((1000, 40), -1, dtype=torch.int16, device=DEV)
    codec.encode(X, out=out[:, :32])
    ref = codec.encode(X.contiguous())
    assert torch.equal(out[:, :32], ref)
    assert (out[:, 32:] == -1).all()                        # nothing written past the row
    dec = torch.zeros(1000, 100, device=DEV)
    codec.decode(ref, out=dec[:, 2:98])
    assert torch.allclose(dec[:, 2:98], codec.decode(ref))
    assert (dec[:, :2] == 0).all() and (dec[:, 98:] == 0).all()


def test_cpu_tensors_round_trip_through_gpu(cuda_ready):
    q = _quantizer("v1", (4, 4, 4))
    X = torch.randn(100, 96)
    codes = q.encode(X)
    assert codes.device.type == "cpu" and codes.dtype == torch.int64
    assert q.decode(codes).device.type == "cpu"


@pytest.mark.parametrize("variant", ["v1", "learned"])
def test_reencode_of_decoded_is_idempotent_full_size(cuda_ready, variant):
    """Decoded vectors sit on bin centres / grid points / centroids, far from any
    boundary, so re-encoding reproduces the codes (v1: except where i_r == 0, whose
    angle is undefined).  262144 vectors = one layer of the learned-gqa encode."""
    q = _quantizer(variant, (4, 4, 4))
    g = torch.Generator(device=DEV).manual_seed(0)
    X = torch.randn(262144, 96, generator=g, device=DEV)
    c1 = q.encode(X)
    c2 = q.encode(q.decode(c1))
    if variant == "v1":
        # angle bins 0 and 15 are the same direction (theta = -pi and +pi are both grid
        # points, stacked_plane.py:255,307): a decoded -pi may come back as +pi
        ir = (c1 >> 4) & 15
        fold = lambda c: torch.where((c & 15) == 15, c - 15, c)
        keep = ir != 0
        assert torch.equal(fold(c1[keep]), fold(c2[keep]))
    else:
        assert (c1 != c2).float().mean().item() < 1e-4      # duplicate-nearest centroids only


@pytest.mark.parametrize("bits", [(4, 4, 4), (3, 3, 2)])
def test_learned_encode_candidate_cells_equal_full_scan(cuda_ready, bits):
    """The per-cell candidate lists give exactly the full 2^(br+bt)-centroid scan's indices:
    points at all scales (inside, at the edge of and beyond the cell grid) and on cell edges."""
    q = _quantizer("learned", bits)
    codec = q.codec(torch.device(DEV))
    assert codec.struct.cell_grid == tables.CELL_GRID
    g = torch.Generator().manual_seed(77)
    parts = [torch.randn(20000, 96, generator=g) * s for s in (0.3, 1.0, 3.0, 8.0)]
    # rows whose rotated (x, y) land exactly on cell edges: rotate grid points back with R
    edge = torch.zeros(4096, 96)
    G = tables.CELL_GRID
    w = 2 * q.r_max / G
    vals = (torch.randint(-G // 2, G // 2 + 1, (4096, 64), generator=g).float() * w).reshape(4096, 64)
    rot = torch.zeros(4096, 96)
    rot[:, 1::3] = vals[:, :32]
    rot[:, 2::3] = vals[:, 32:]
    edge = rot @ q.R
    X = torch.cat(parts + [edge]).float().to(DEV)
    with_cells = codec.encode(X).cpu()
    saved = codec.struct.cell_grid
    codec.struct.cell_grid = 0
    try:
        full = codec.encode(X).cpu()
    finally:
        codec.struct.cell_grid = saved
    assert torch.equal(with_cells, full)


def _force_cuda_core(codec):
    """Context: the codec without its bf16 R parts, so encode takes the CUDA-core kernel."""
    class _Ctx:
        def __enter__(self):
            self.saved = codec.struct.R_bf16x3
            codec.struct.R_bf16x3 = None

        def __exit__(self, *exc):
            codec.struct.R_bf16x3 = self.saved
    return _Ctx()


@pytest.mark.parametrize("variant,bits", [("v1", (4, 4, 4)), ("v1", (3, 3, 2)), ("learned_bias", (4, 4, 4)),
                                          ("lloyd", (4, 4, 4))])
@pytest.mark.parametrize("n", [1, 127, 128, 129, 5000, 70001])
def test_tensor_core_encode_matches_oracle(cuda_ready, variant, bits, n):
    """bf16 rows of head_dim 96 are rotated on tcgen05 (R in three bf16 parts): codes equal the
    oracle's except proven ties, and equal the CUDA-core kernel's except proven ties; every
    partial tile and the grid-stride tail are covered by the sizes."""
    q = _quantizer(variant, bits)
    p = _params(q)
    codec = q.codec(torch.device(DEV))
    g = torch.Generator().manual_seed(n)
    X = (torch.randn(n, 96, generator=g) * 1.3).to(torch.bfloat16)
    Xd = X.to(DEV)
    tc = codec.encode(Xd).cpu().numpy().astype(np.int64)
    with _force_cuda_core(codec):
        cc = codec.encode(Xd).cpu().numpy().astype(np.int64)
    X32 = X.float().numpy()
    rep = oracle.classify(X32, q.R.numpy(), p, tc, oracle.encode(X32, q.R.numpy(), p))
    assert rep.unexplained == 0, rep.examples
    assert rep.mismatches <= max(2, int(rep.total * TIE_RATE))
    rep2 = oracle.classify(X32, q.R.numpy(), p, tc, cc)
    assert rep2.unexplained == 0, rep2.examples


def test_tensor_core_encode_strided_rows_and_cache_append(cuda_ready):
    """Row stride > 96 (16-byte multiple) and the KV-cache append form (grouped code rows)."""
    q = _quantizer("v1", (4, 4, 4))
    codec = q.codec(torch.device(DEV))
    g = torch.Generator(device=DEV).manual_seed(3)
    big = torch.randn(3000, 128, generator=g, device=DEV).to(torch.bfloat16)
    X = big[:, :96]
    a = codec.encode(X)
    b = codec.encode(X.contiguous())
    assert torch.equal(a, b)
    cache = torch.zeros(4, 1000, 32, dtype=torch.int16, device=DEV)
    xs = torch.randn(4, 300, 96, generator=g, device=DEV).to(torch.bfloat16)
    codec.encode_append(xs, cache, 77)
    ref = codec.encode(xs.reshape(-1, 96)).view(4, 300, 32)
    assert torch.equal(cache[:, 77:377], ref)
    assert (cache[:, :77] == 0).all() and (cache[:, 377:] == 0).all()


def test_tensor_core_encode_edge_rows(cuda_ready):
    """Edge rows through the tensor-core epilogue (first-guess bin counts): zeros, huge,
    tiny, +-inf and NaN components, in bf16, against the CUDA-core kernel."""
    for variant in ("v1", "lloyd", "learned"):
        q = _quantizer(variant, (4, 4, 4))
        codec = q.codec(torch.device(DEV))
        g = torch.Generator().manual_seed(9)
        rows = [torch.zeros(96), torch.randn(96, generator=g) * 1e30, torch.randn(96, generator=g) * 1e-30,
                torch.randn(96, generator=g) * 60]
        for k, val in ((3, float("inf")), (10, float("nan")), (0, -float("inf")), (40, float("inf"))):
            r = torch.randn(96, generator=g)
            r[k] = val
            rows.append(r)
        X = torch.stack(rows * 40).to(torch.bfloat16).to(DEV)
        tc = codec.encode(X)
        with _force_cuda_core(codec):
            cc = codec.encode(X)
        assert torch.equal(tc, cc), variant


@pytest.mark.parametrize("which", ["cb", "lloyd"])
def test_encode_after_loading_reference_written_files(cuda_ready, which):
    """A codebook / Lloyd-Max file written by the reference, loaded through the drop-in API, gives
    the reference's codes on the GPU (rounding ties excepted, each proven in fp64)."""
    import os
    from conftest import GOLDEN
    from prismkv_b200 import StackedPlaneQuantizer
    f = load_golden("files_codes")
    q = StackedPlaneQuantizer(96, 4, 4, 4, seed=42)
    p = oracle.QuantParams.default(96)
    if which == "cb":
        q.load_codebooks(os.path.join(GOLDEN, "ref_codebook_444.npz"))
        p.codebook = q._codebooks.codebooks.numpy()
        p.z_min, p.z_max, p.r_max = q.z_min, q.z_max, q.r_max
    else:
        q.load_lloyd_max_z(os.path.join(GOLDEN, "ref_lloyd_z.npz"))
        p.lloyd_boundaries = q._lloyd_max_z.boundaries.numpy()
        p.lloyd_centroids = q._lloyd_max_z.centroids.numpy()
    codes = q.encode(torch.from_numpy(f["x"]).to(DEV)).cpu().numpy()
    rep = oracle.classify(f["x"], f["R"], p, codes, f[f"codes_{which}"].astype(np.int64) & 0xFFF)
    assert rep.unexplained == 0, rep.examples
    assert rep.mismatches <= max(2, int(rep.total * TIE_RATE))
