"""Rounding-tie classifier for PrismKV codes -- TEST INFRASTRUCTURE ONLY.

Two correct implementations of ``StackedPlaneQuantizer.encode``
(stacked_plane.py:210-262) can disagree on a code only where the exact
(fp64) value of a binned quantity lies within the rounding error of a bin
boundary: the rotation GEMM rounds differently on every machine, and the
reference's vectorised ``sqrt``/``atan2`` are within 1 ulp.  This module
decides, for each mismatching code, whether it is such a tie.

For each component with differing indices, the exact value ``v`` and a
bound ``e`` on any fp32 evaluation's error are computed; the mismatch is a
tie when both indices are reachable by binning some value in ``[v-e, v+e]``
with the reference's own (monotone) fp32 binning chain.  The nearest
centroid of the learned path is a tie when the two centroids' exact squared
distances differ by less than their evaluation error.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List

import numpy as np

from .prismkv_oracle import (F32, QuantParams, bin_r, bin_theta, bin_z)

U32 = 2.0 ** -24


@dataclass
class TieReport:
    total: int
    mismatches: int
    ties: int
    unexplained: int
    examples: List[tuple] = field(default_factory=list)

    def as_dict(self):
        return {"codes": self.total, "mismatches": self.mismatches, "ties": self.ties,
                "unexplained": self.unexplained}


def _down(v):
    v32 = np.asarray(v, dtype=np.float64).astype(F32)
    return np.where(v32.astype(np.float64) > v, np.nextafter(v32, F32(-np.inf)), v32).astype(F32)


def _up(v):
    v32 = np.asarray(v, dtype=np.float64).astype(F32)
    return np.where(v32.astype(np.float64) < v, np.nextafter(v32, F32(np.inf)), v32).astype(F32)


def _in_range(i, lo, hi):
    return (i >= np.minimum(lo, hi)) & (i <= np.maximum(lo, hi))


def classify(X: np.ndarray, R: np.ndarray, p: QuantParams, codes_a: np.ndarray,
             codes_b: np.ndarray, slack: float = 1.5) -> TieReport:
    """Classify every position where ``codes_a != codes_b``.

    X: (N, dim) inputs (any float dtype, taken exactly); R: (dim, dim).
    ``slack`` scales the worst-case fp32 dot-product bound ``dim * u * sum|x R|``.
    """
    codes_a = np.asarray(codes_a).astype(np.int64)
    codes_b = np.asarray(codes_b).astype(np.int64)
    mask = codes_a != codes_b
    n_mis = int(mask.sum())
    rep = TieReport(total=int(codes_a.size), mismatches=n_mis, ties=0, unexplained=0)
    if n_mis == 0:
        return rep
    rows, cols = np.nonzero(mask)
    X64 = np.asarray(X, dtype=np.float32).astype(np.float64)[rows]       # (k, dim)
    R64 = np.asarray(R, dtype=np.float32).astype(np.float64)
    kz, kx, ky = 3 * cols, 3 * cols + 1, 3 * cols + 2
    v = {}
    e = {}
    for name, k in (("z", kz), ("x", kx), ("y", ky)):
        rr = R64[k]                                                        # (k, dim)
        v[name] = np.einsum("nd,nd->n", X64, rr)
        mag = np.einsum("nd,nd->n", np.abs(X64), np.abs(rr))
        e[name] = slack * p.dim * U32 * mag + 4 * U32 * np.abs(v[name]) + 1e-30

    bits_flat = p.bits_r + p.bits_theta
    a, b = codes_a[rows, cols], codes_b[rows, cols]
    iz_a, iz_b = a >> bits_flat, b >> bits_flat
    fl_a, fl_b = a & ((1 << bits_flat) - 1), b & ((1 << bits_flat) - 1)

    ok = np.ones(n_mis, dtype=bool)
    # --- z component
    dz = iz_a != iz_b
    if dz.any():
        lo = bin_z(_down(v["z"] - e["z"]), p)
        hi = bin_z(_up(v["z"] + e["z"]), p)
        ok &= ~dz | (_in_range(iz_a, lo, hi) & _in_range(iz_b, lo, hi))
    dfl = fl_a != fl_b
    if dfl.any():
        x, y = v["x"], v["y"]
        ex, ey = e["x"], e["y"]
        if p.codebook is None:
            mt = (1 << p.bits_theta) - 1
            ir_a, ir_b = fl_a >> p.bits_theta, fl_b >> p.bits_theta
            it_a, it_b = fl_a & mt, fl_b & mt
            r = np.hypot(x, y)
            er = ex + ey + 4 * U32 * r + 1e-30
            lo = bin_r(_down(np.maximum(r - er, 0.0)), p)
            hi = bin_r(_up(r + er), p)
            dr = ir_a != ir_b
            ok &= ~dr | (_in_range(ir_a, lo, hi) & _in_range(ir_b, lo, hi))
            dt = it_a != it_b
            if dt.any():
                th = np.arctan2(y, x)
                with np.errstate(divide="ignore", invalid="ignore"):
                    et = (ex + ey) / r + 4 * U32 * np.maximum(np.abs(th), 1e-30) + 1e-30
                et = np.where(np.isfinite(et), et, np.inf)
                undefined = et >= math.pi                    # radius within error of zero
                tlo, thi = th - et, th + et
                lo = bin_theta(_down(np.maximum(tlo, -math.pi)), p)
                hi = bin_theta(_up(np.minimum(thi, math.pi)), p)
                inside = _in_range(it_a, lo, hi) & _in_range(it_b, lo, hi)
                # wrap-around at the +-pi branch cut: bins near -pi and near +pi both valid
                wlo = bin_theta(_down(np.maximum(tlo + 2 * math.pi, -math.pi)), p)
                wlo_top = bin_theta(F32(math.pi), p)
                whi = bin_theta(_up(np.minimum(thi - 2 * math.pi, math.pi)), p)
                wbot = bin_theta(F32(-math.pi), p)
                in_a = (_in_range(it_a, lo, hi) | ((thi > math.pi) & _in_range(it_a, wbot, whi))
                        | ((tlo < -math.pi) & _in_range(it_a, wlo, wlo_top)))
                in_b = (_in_range(it_b, lo, hi) | ((thi > math.pi) & _in_range(it_b, wbot, whi))
                        | ((tlo < -math.pi) & _in_range(it_b, wlo, wlo_top)))
                ok &= ~dt | undefined | inside | (in_a & in_b)
        else:
            cb = p.codebook.astype(np.float64)
            ca = cb[np.clip(iz_a, 0, p.Cz - 1), fl_a]
            cbb = cb[np.clip(iz_b, 0, p.Cz - 1), fl_b]
            da = (x - ca[:, 0]) ** 2 + (y - ca[:, 1]) ** 2
            db = (x - cbb[:, 0]) ** 2 + (y - cbb[:, 1]) ** 2
            pn = x * x + y * y
            cn = np.maximum((ca ** 2).sum(1), (cbb ** 2).sum(1))
            tol = (2 * (np.sqrt(da) + np.sqrt(db) + 1e-30) * (ex + ey)
                   + 32 * U32 * (pn + cn) + 1e-30)
            same_bin = iz_a == iz_b
            # within one z-bin: both centroids nearly equidistant and nearest
            bins = np.clip(iz_a, 0, p.Cz - 1)
            allc = cb[bins]                                         # (k, K, 2)
            dmin = ((x[:, None] - allc[..., 0]) ** 2 + (y[:, None] - allc[..., 1]) ** 2).min(1)
            near = (np.abs(da - db) <= tol) & (da <= dmin + tol) & (db <= dmin + tol)
            # across a z tie each side picked the nearest of its own bin
            bins_b = np.clip(iz_b, 0, p.Cz - 1)
            allb = cb[bins_b]
            dminb = ((x[:, None] - allb[..., 0]) ** 2 + (y[:, None] - allb[..., 1]) ** 2).min(1)
            cross = (~same_bin) & (da <= dmin + tol) & (db <= dminb + tol)
            ok &= ~dfl | np.where(same_bin, near, cross)
    # non-finite inputs have no rounding ties: their codes must agree exactly
    ok &= np.isfinite(X64).all(axis=1)
    rep.ties = int(ok.sum())
    rep.unexplained = int((~ok).sum())
    bad = np.nonzero(~ok)[0][:10]
    rep.examples = [(int(rows[i]), int(cols[i]), int(a[i]), int(b[i])) for i in bad]
    return rep
