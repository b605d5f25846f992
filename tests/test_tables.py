"""Host tables (thresholds, LUTs) reproduce the reference's fp32 binning exactly.

The kernels compute i = #{b : v >= t_b} on the same fp32 value the
reference bins; here that count (numpy emulation of the device rule) is
compared with the oracle's step-by-step restatement of the reference chain
over random values, values on and one ulp either side of every threshold,
and the special values (signed zeros, infinities, NaN, values overflowing
the reference's int64 conversion).
"""

import math

import numpy as np
import pytest

import oracle
from oracle import QuantParams
from prismkv_b200.tables import build_host_tables

CONFIGS = [(4, 4, 4), (3, 3, 2), (2, 3, 1), (1, 1, 1), (8, 4, 4), (5, 5, 6), (4, 6, 6)]


def _kernel_bins(ht, z, x, y):
    """numpy emulation of the encode kernel's binning (pkv_codec.cu)."""
    z = np.asarray(z, np.float32)
    iz = np.searchsorted(ht.z_thr, z, side="right")
    iz = np.where(z >= np.float32(ht.z_hi), 0, iz)
    iz = np.where(np.isnan(z), ht.z_nan_bin, iz)
    with np.errstate(over="ignore", invalid="ignore"):
        s = (x * x).astype(np.float32) + (y * y).astype(np.float32)
    ir = np.where(np.isnan(s), 0, np.searchsorted(ht.r2_thr, s, side="right"))
    th = np.arctan2(y.astype(np.float64), x.astype(np.float64)).astype(np.float32)
    it = np.where(np.isnan(th), 0, np.searchsorted(ht.th_thr, th, side="right"))
    return iz, ir, it


def _probe_values(thr, scale, rng):
    thr = thr[np.isfinite(thr)]
    around = np.concatenate([thr, np.nextafter(thr, np.float32(np.inf)), np.nextafter(thr, np.float32(-np.inf))])
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e19, -1e19, 1e30, -1e30, 1e-40, 3e38],
                        dtype=np.float32)
    rnd = (rng.standard_normal(200000) * scale).astype(np.float32)
    return np.concatenate([around.astype(np.float32), specials, rnd])


@pytest.mark.parametrize("bits", CONFIGS, ids=str)
def test_encode_thresholds_match_reference_chain(bits):
    rng = np.random.default_rng(sum(bits))
    dim = 96
    p = QuantParams.default(dim, *bits)
    ht = build_host_tables(dim, *bits, np.eye(dim, dtype=np.float32), p.z_min, p.z_max, p.r_max)
    z = _probe_values(ht.z_thr, 6.0, rng)
    iz, _, _ = _kernel_bins(ht, z, np.zeros_like(z), np.zeros_like(z))
    np.testing.assert_array_equal(iz, oracle.bin_z(z, p))
    # radius: probe along x with y = 0 and on random (x, y)
    rt = np.sqrt(ht.r2_thr.astype(np.float64)).astype(np.float32)
    xv = np.concatenate([_probe_values(rt, 5.0, rng), (rng.standard_normal(100000) * 3).astype(np.float32)])
    yv = np.concatenate([np.zeros(xv.size - 100000, np.float32), (rng.standard_normal(100000) * 3).astype(np.float32)])
    _, ir, it = _kernel_bins(ht, np.zeros_like(xv), xv, yv)
    np.testing.assert_array_equal(ir, oracle.bin_r(oracle.prismkv_oracle.radius_f32(xv, yv), p))
    th = oracle.prismkv_oracle.atan2_f32(yv, xv)
    np.testing.assert_array_equal(it, oracle.bin_theta(th, p))
    # angle thresholds probed directly as angles
    tv = np.concatenate([ht.th_thr, np.nextafter(ht.th_thr, np.float32(9)), np.nextafter(ht.th_thr, np.float32(-9)),
                         np.float32([-math.pi, math.pi, 0.0, -0.0])]).astype(np.float32)
    got = np.searchsorted(ht.th_thr, tv, side="right")
    np.testing.assert_array_equal(got, oracle.bin_theta(tv, p))


def test_lloyd_thresholds_match_bucketize():
    rng = np.random.default_rng(5)
    b = np.sort(rng.standard_normal(17).astype(np.float32))
    b[0], b[-1] = b[0] - 1, b[-1] + 1
    p = QuantParams.default(96)
    p.lloyd_boundaries = b
    p.lloyd_centroids = ((b[:-1] + b[1:]) / 2).astype(np.float32)
    ht = build_host_tables(96, 4, 4, 4, np.eye(96, dtype=np.float32), p.z_min, p.z_max, p.r_max,
                           lloyd_boundaries=b, lloyd_centroids=p.lloyd_centroids)
    z = _probe_values(b, 2.0, rng)
    iz, _, _ = _kernel_bins(ht, z, np.zeros_like(z), np.zeros_like(z))
    np.testing.assert_array_equal(iz, oracle.bin_z(z, p))


@pytest.mark.parametrize("variant", ["v1", "v1_bias", "lloyd", "learned_bias", "v1_332"])
def test_decode_tables_match_reference_dequant(variant):
    rng = np.random.default_rng(11)
    bits = (3, 3, 2) if variant == "v1_332" else (4, 4, 4)
    p = QuantParams.default(96, *bits)
    Cz, K = 1 << bits[0], 1 << (bits[1] + bits[2])
    if "bias" in variant:
        p.bias_table = (rng.standard_normal((Cz, 3)) * 0.3).astype(np.float32)   # some entries clip
        p.bias_delta_z = p.delta_z
    if variant == "lloyd":
        bnd = np.sort(rng.standard_normal(Cz + 1).astype(np.float32) * 4)
        p.lloyd_boundaries = bnd
        p.lloyd_centroids = ((bnd[:-1] + bnd[1:]) / 2).astype(np.float32)
    if variant.startswith("learned"):
        p.codebook = (rng.standard_normal((Cz, K, 2)) * 3).astype(np.float32)
    ht = build_host_tables(96, *bits, np.eye(96, dtype=np.float32), p.z_min, p.z_max, p.r_max,
                           codebook=p.codebook, lloyd_boundaries=p.lloyd_boundaries,
                           lloyd_centroids=p.lloyd_centroids, bias_table=p.bias_table,
                           bias_delta_z=p.bias_delta_z if p.bias_table is not None else None)
    total = Cz * K
    codes = np.arange(total)
    pad = (-total) % p.m
    rows = np.concatenate([codes, np.zeros(pad, np.int64)]).reshape(-1, p.m)
    ref = oracle.dequant_rotated(rows, p).reshape(-1, 3)[:total]
    bf = bits[1] + bits[2]
    z = ht.dec_z[codes >> bf]
    xy = ht.dec_xy.reshape(-1, 2)[codes if ht.xy_per_z else codes & ((1 << bf) - 1)]
    np.testing.assert_array_equal(z, ref[:, 0])
    # the tables take cos/sin from torch's vectorised CPU kernels, exactly as the
    # reference's decode does; the oracle rounds them correctly: <= 1 ulp of cos/sin apart
    tol = 2.0 ** -21 * p.r_max
    np.testing.assert_allclose(xy[:, 0], ref[:, 1], atol=tol, rtol=0)
    np.testing.assert_allclose(xy[:, 1], ref[:, 2], atol=tol, rtol=0)


def test_split_bf16x3_exact_and_sign_preserving():
    """R = R1 + R2 + R3 in bf16 parts: sum within 2^-24 |R|, every part with R's sign and
    non-zero, so an infinite input component never meets inf - inf or inf * 0."""
    from prismkv_b200.codec import split_bf16x3
    from prismkv_b200.utils import make_rotation
    for dim, seed in ((96, 42), (66, 7)):
        R = make_rotation(dim, seed).numpy()
        parts = (split_bf16x3(R).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        err = np.abs(parts.sum(0) - R.astype(np.float64))
        assert (err <= 2.0 ** -24 * np.abs(R)).all()
        assert (np.sign(parts) == np.sign(R)[None]).all() and (parts != 0).all()
    z = split_bf16x3(np.array([[0.0, 1.0, -3.0]], np.float32))
    assert (z[:, 0, 0] == 0).all()                      # an exact zero stays zero


def test_centroid_cells_contain_every_nearest_centroid():
    """Every point of a grid cell has its nearest centroid (fp64) among the cell's candidates,
    in ascending index order: the device scan over the candidates then equals the full scan.
    Points at random, at cell edges and at the grid's rim."""
    from prismkv_b200.synthetic import synthetic_codebook
    from prismkv_b200.tables import CELL_GRID, CELL_MAX, centroid_cells
    r_max = math.sqrt(96.0)
    cb = synthetic_codebook(4, 256, r_max, 11).numpy()
    idx, cnt = centroid_cells(cb, r_max)
    assert idx.shape == (4, CELL_GRID, CELL_GRID, CELL_MAX) and cnt.shape == (4, CELL_GRID, CELL_GRID)
    w = 2 * r_max / CELL_GRID
    rng = np.random.default_rng(3)
    pts = [rng.standard_normal((20000, 2)) * s for s in (0.5, 1.5, 4.0)]
    edges = (rng.integers(0, CELL_GRID + 1, (20000, 2)) * w - r_max)          # on cell edges
    rim = np.stack([np.full(2000, -r_max), rng.uniform(-r_max, r_max, 2000)], 1)
    P = np.concatenate(pts + [edges, rim]).astype(np.float32)
    P = P[(np.abs(P) < r_max).all(1)]                                       # inside the grid
    iz = rng.integers(0, 4, len(P))
    fx = np.floor((P[:, 0] + np.float32(r_max)) * np.float32(CELL_GRID / (2 * r_max))).astype(int)
    fy = np.floor((P[:, 1] + np.float32(r_max)) * np.float32(CELL_GRID / (2 * r_max))).astype(int)
    fx, fy = np.clip(fx, 0, CELL_GRID - 1), np.clip(fy, 0, CELL_GRID - 1)
    d = ((P[:, None, :].astype(np.float64) - cb[iz].astype(np.float64)) ** 2).sum(-1)
    nearest = d.argmin(1)
    n = cnt[iz, fy, fx]
    assert (n != 255).mean() > 0.999 and n[n != 255].mean() < 4
    ok = n != 255
    cand = idx[iz, fy, fx].astype(int)[ok]                                  # (points, CELL_MAX)
    valid = np.arange(CELL_MAX)[None, :] < n[ok][:, None]
    assert (((np.diff(cand, axis=1) > 0) | ~valid[:, 1:]).all())             # ascending indices
    hit = ((cand == nearest[ok][:, None]) & valid).any(1)
    assert hit.all(), P[ok][~hit][:5]
