"""Host-side construction of the quantizer tables the kernels consume.

The tables are the quantizer's parameters (a few KB), built once per
quantizer state on the host and uploaded.  They let the device reproduce the
reference's fp32 arithmetic exactly:

* Encode thresholds.  Each index the reference computes after the rotation
  is a monotone step function of one fp32 value:
    - ``i_z  = clamp(floor((z - z_min) / delta_z), 0, C_z - 1)``
      (stacked_plane.py:239-241), or ``bucketize(z, boundaries[1:-1])``
      (lloyd_max.py:123);
    - ``i_r  = clamp(round(clamp(sqrt(s), 0, r_max) / r_max * (C_r - 1)), ...)``
      with ``s = x*x + y*y`` (stacked_plane.py:249, 252-253);
    - ``i_th = clamp(round((theta + pi) / (2 pi) * (C_th - 1)), ...)``
      (stacked_plane.py:250, 255-256).
  For every bin ``b`` the smallest fp32 input reaching ``b`` is found by
  bisection over the ordered fp32 values, evaluating the chain with the
  reference's own op sequence in fp32.  On the device ``i = #{b : v >= t_b}``
  then equals the reference's index for the same fp32 input.
* Decode tables.  The dequantized z per bin and (x, y) per code, computed
  with the reference's fp32 expressions (stacked_plane.py:288-310,
  learned_codebook.py:268) and with the BiasTable subtraction folded in
  (bias_correction.py:81-89).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import numpy as np
import torch

F32 = np.float32


# ---------------------------------------------------------------------------
# fp32 ordering helpers
# ---------------------------------------------------------------------------

def _f32_to_key(v: np.ndarray) -> np.ndarray:
    """Map fp32 values to int64 keys whose order matches the float order."""
    b = np.asarray(v, dtype=F32).view(np.int32).astype(np.int64)
    return np.where(b < 0, -(b & 0x7FFFFFFF) - 1, b)


def _key_to_f32(k: np.ndarray) -> np.ndarray:
    k = np.asarray(k, dtype=np.int64)
    b = np.where(k < 0, (-(k + 1)) | 0x80000000, k)
    return b.astype(np.uint32).view(F32)


def smallest_reaching(f: Callable[[np.ndarray], np.ndarray], targets: np.ndarray,
                      lo: float, hi: float) -> np.ndarray:
    """For each target b: the smallest fp32 v in [lo, hi] with f(v) >= b.

    ``f`` must be non-decreasing on [lo, hi] (fp32 order).  Targets not
    reached at ``hi`` get +inf.
    """
    targets = np.asarray(targets, dtype=np.int64)
    klo = np.full(targets.shape, _f32_to_key(F32(lo)), dtype=np.int64)
    khi = np.full(targets.shape, _f32_to_key(F32(hi)), dtype=np.int64)
    reach_hi = f(_key_to_f32(khi)) >= targets
    # invariant: f(lo_key) < target (or lo itself reaches), f(hi_key) >= target
    lo_ok = f(_key_to_f32(klo)) >= targets
    for _ in range(40):
        mid = (klo + khi) // 2
        fm = f(_key_to_f32(mid)) >= targets
        khi = np.where(fm, mid, khi)
        klo = np.where(fm, klo, mid)
    res = np.where(lo_ok, _key_to_f32(klo), _key_to_f32(khi))
    return np.where(reach_hi, res, F32(np.inf)).astype(F32)


def _to_long_raw(v: np.ndarray) -> np.ndarray:
    """Monotone fp32 -> integer map used while searching thresholds (+-inf saturate)."""
    v = np.nan_to_num(np.asarray(v, dtype=np.float64), nan=-2.0 ** 62, posinf=2.0 ** 62, neginf=-2.0 ** 62)
    return np.clip(v, -2.0 ** 62, 2.0 ** 62).astype(np.int64)


# ---------------------------------------------------------------------------
# encode thresholds
# ---------------------------------------------------------------------------

def z_uniform_thresholds(z_min: float, z_max: float, bits_z: int):
    """Thresholds for ``floor((z - z_min) / delta_z)`` (stacked_plane.py:239-241).

    Returns (thresholds (C_z-1,), z_hi): ``z >= z_hi`` overflows the
    reference's int64 conversion (the result INT64_MIN clamps to bin 0).
    """
    Cz = 1 << bits_z
    zmin = F32(z_min)
    dz = F32((z_max - z_min) / Cz)

    def pre(z):
        with np.errstate(over="ignore", invalid="ignore"):
            return ((np.asarray(z, F32) - zmin).astype(F32) / dz).astype(F32)

    def idx(z):
        return _to_long_raw(np.floor(pre(z)))

    big = F32(3.0e38)
    thr = smallest_reaching(idx, np.arange(1, Cz), -big, big)
    # z_hi: smallest z whose pre-floor value is >= 2**63
    def over(z):
        with np.errstate(invalid="ignore"):
            return (pre(z).astype(np.float64) >= 2.0 ** 63).astype(np.int64)
    z_hi = smallest_reaching(over, np.array([1]), -big, big)[0]
    return thr, F32(z_hi)


def z_lloyd_thresholds(boundaries: np.ndarray):
    """``bucketize(z, boundaries[1:-1])`` counts inner boundaries strictly below z."""
    inner = np.asarray(boundaries, dtype=F32)[1:-1]
    return np.nextafter(inner, F32(np.inf)).astype(F32)


def r2_thresholds(r_max: float, bits_r: int) -> np.ndarray:
    """Thresholds on ``s = x*x + y*y`` for the radius bin (stacked_plane.py:249,252-253)."""
    Cr = 1 << bits_r
    rmax = F32(r_max)

    def idx(s):
        with np.errstate(invalid="ignore"):
            r = np.sqrt(np.asarray(s, F32)).astype(F32)
            r = np.minimum(np.maximum(r, F32(0)), rmax)
            t = ((r / rmax).astype(F32) * F32(Cr - 1)).astype(F32)
            return _to_long_raw(np.rint(t))

    return smallest_reaching(idx, np.arange(1, Cr), 0.0, 3.0e38)


def theta_thresholds(bits_theta: int) -> np.ndarray:
    """Thresholds on ``theta = atan2(y, x)`` (stacked_plane.py:250, 255-256)."""
    Ct = 1 << bits_theta

    def idx(th):
        t = (np.asarray(th, F32) + F32(math.pi)).astype(F32)
        t = (t / F32(2 * math.pi)).astype(F32)
        t = (t * F32(Ct - 1)).astype(F32)
        return _to_long_raw(np.rint(t))

    return smallest_reaching(idx, np.arange(1, Ct), -4.0, 4.0)


# ---------------------------------------------------------------------------
# decode tables
# ---------------------------------------------------------------------------

def _torch_vec_f32(fn, x: np.ndarray) -> np.ndarray:
    """Evaluate a torch CPU elementwise op through its vectorised path."""
    n = x.size
    reps = max(1, -(-256 // max(n, 1)))
    t = torch.from_numpy(np.tile(x.astype(F32), reps))
    return fn(t).numpy()[:n].astype(F32)


def dec_z_table(z_min: float, z_max: float, bits_z: int,
                lloyd_centroids: Optional[np.ndarray] = None) -> np.ndarray:
    Cz = 1 << bits_z
    if lloyd_centroids is not None:                         # lloyd_max.py:126-140
        return np.asarray(lloyd_centroids, dtype=F32)[:Cz].copy()
    iz = np.arange(Cz).astype(F32)                          # stacked_plane.py:292-293
    t = ((iz + F32(0.5)).astype(F32) * F32((z_max - z_min) / Cz)).astype(F32)
    return (F32(z_min) + t).astype(F32)


def dec_xy_polar(r_max: float, bits_r: int, bits_theta: int) -> np.ndarray:
    """(K, 2) uniform polar grid (stacked_plane.py:297-310), K = C_r * C_th."""
    Cr, Ct = 1 << bits_r, 1 << bits_theta
    flat = np.arange(Cr * Ct)
    i_t = (flat & (Ct - 1)).astype(F32)
    i_r = ((flat >> bits_theta) & (Cr - 1)).astype(F32)
    r_q = ((i_r / F32(Cr - 1)).astype(F32) * F32(r_max)).astype(F32)
    th = (i_t / F32(Ct - 1)).astype(F32)
    th = (th * F32(2.0)).astype(F32)
    th = (th * F32(math.pi)).astype(F32)
    th = (th - F32(math.pi)).astype(F32)
    c = _torch_vec_f32(torch.cos, th)
    s = _torch_vec_f32(torch.sin, th)
    return np.stack([(r_q * c).astype(F32), (r_q * s).astype(F32)], axis=-1)


CELL_GRID = 128         # cells per axis of the nearest-centroid candidate grid
CELL_MAX = 16           # candidates kept per cell; fuller cells fall back to the full scan


def centroid_cells(codebook: np.ndarray, half_width: float, grid: int = CELL_GRID, max_cand: int = CELL_MAX):
    """Candidate centroids per cell of a grid over [-half_width, half_width]^2, per z-bin.

    Centroid k is a candidate of cell Q when its least squared distance to Q is
    within a rounding margin of min_j (greatest squared distance from Q to c_j):
    for any point p of Q the nearest centroid (and every centroid whose fp32
    distance could tie with it) satisfies that bound, so scanning the candidates
    in index order gives the full scan's first-minimal index.  Cells are widened
    by 1e-4 of their width to absorb the fp32 rounding of the point-to-cell map.
    Returns (idx uint8 [Cz, grid, grid, max_cand], cnt uint8 [Cz, grid, grid]);
    cnt 255 marks a cell with more than max_cand candidates.
    """
    cb = np.asarray(codebook, dtype=np.float64)
    Cz, K, _ = cb.shape
    if K > 256:
        raise ValueError("candidate cells index at most 256 centroids")
    w = 2.0 * half_width / grid
    edges = -half_width + w * np.arange(grid + 1)
    lo, hi = edges[:-1] - 1e-4 * w, edges[1:] + 1e-4 * w
    idx = np.zeros((Cz, grid, grid, max_cand), dtype=np.uint8)
    cnt = np.zeros((Cz, grid, grid), dtype=np.uint8)
    for b in range(Cz):
        cx, cy = cb[b, :, 0], cb[b, :, 1]
        dxn = np.maximum(np.maximum(lo[:, None] - cx[None, :], 0.0), cx[None, :] - hi[:, None])
        dxf = np.maximum(np.abs(lo[:, None] - cx[None, :]), np.abs(hi[:, None] - cx[None, :]))
        dyn = np.maximum(np.maximum(lo[:, None] - cy[None, :], 0.0), cy[None, :] - hi[:, None])
        dyf = np.maximum(np.abs(lo[:, None] - cy[None, :]), np.abs(hi[:, None] - cy[None, :]))
        near = dyn[:, None, :] ** 2 + dxn[None, :, :] ** 2           # [y cell, x cell, k]
        far = dyf[:, None, :] ** 2 + dxf[None, :, :] ** 2
        bound = far.min(axis=2) * (1.0 + 1e-5) + 1e-6
        cand = near <= bound[..., None]
        n = cand.sum(axis=2)
        cnt[b] = np.where(n > max_cand, 255, n).astype(np.uint8)
        order = np.argsort(~cand, axis=2, kind="stable")[..., :max_cand]   # candidate indices first, ascending
        idx[b] = np.where(np.arange(max_cand)[None, None, :] < n[..., None], order, 0).astype(np.uint8)
    return idx, cnt


@dataclass
class HostTables:
    dim: int
    bits: tuple
    xy_mode: int
    xy_per_z: int
    z_nan_bin: int
    z_hi: float
    r_max: float
    R: np.ndarray
    z_thr: np.ndarray
    r2_thr: np.ndarray
    th_thr: np.ndarray
    codebook: np.ndarray
    dec_z: np.ndarray
    dec_xy: np.ndarray
    bias_xy: Optional[np.ndarray] = None     # (C_z, 2) clamped BiasTable (x, y) terms
    z_uniform: bool = False                  # dec_z[i] = z_min + (i + 0.5) * delta_z (no Lloyd-Max, no bias)
    cell_idx: Optional[np.ndarray] = None    # learned codebooks: candidate centroids per grid cell
    cell_cnt: Optional[np.ndarray] = None
    cell_half_width: float = 0.0


def build_host_tables(dim: int, bits_z: int, bits_r: int, bits_theta: int, R: np.ndarray,
                      z_min: float, z_max: float, r_max: float,
                      codebook: Optional[np.ndarray] = None,
                      lloyd_boundaries: Optional[np.ndarray] = None,
                      lloyd_centroids: Optional[np.ndarray] = None,
                      bias_table: Optional[np.ndarray] = None,
                      bias_delta_z: Optional[float] = None) -> HostTables:
    Cz = 1 << bits_z
    K = 1 << (bits_r + bits_theta)
    if lloyd_boundaries is not None:
        z_thr = z_lloyd_thresholds(lloyd_boundaries)
        z_hi = F32(np.nan)
        z_nan_bin = Cz - 1                                   # bucketize(NaN) lands past the end
    else:
        z_thr, z_hi = z_uniform_thresholds(z_min, z_max, bits_z)
        z_nan_bin = 0                                        # NaN -> INT64_MIN -> clamp -> 0
    r2 = r2_thresholds(r_max, bits_r)
    th = theta_thresholds(bits_theta)
    dz = dec_z_table(z_min, z_max, bits_z, lloyd_centroids)
    if codebook is not None:
        cb = np.ascontiguousarray(codebook, dtype=F32).reshape(Cz, K, 2)
        xy = cb.copy()
        xy_mode = 1
    else:
        cb = np.zeros((1, 1, 2), dtype=F32)
        xy = np.broadcast_to(dec_xy_polar(r_max, bits_r, bits_theta), (Cz, K, 2)).copy()
        xy_mode = 0
    xy_per_z = int(codebook is not None or bias_table is not None)
    bias_xy = None
    if bias_table is not None:
        clip = F32(bias_delta_z / 2.0)
        b = np.clip(np.asarray(bias_table, dtype=F32), -clip, clip).astype(F32)   # (Cz, 3)
        dz = (dz - b[:, 0]).astype(F32)
        xy = (xy - b[:, None, 1:3]).astype(F32)
        bias_xy = np.ascontiguousarray(b[:, 1:3])
    if not xy_per_z:
        xy = xy[0]
    cells = (None, None)
    if codebook is not None and K <= 256:
        cells = centroid_cells(cb, float(r_max))
    return HostTables(dim=dim, bits=(bits_z, bits_r, bits_theta), xy_mode=xy_mode, xy_per_z=xy_per_z,
                      z_nan_bin=z_nan_bin, z_hi=float(z_hi), r_max=float(r_max),
                      R=np.ascontiguousarray(R, dtype=F32), z_thr=z_thr.astype(F32),
                      r2_thr=r2.astype(F32), th_thr=th.astype(F32), codebook=cb,
                      dec_z=dz.astype(F32), dec_xy=np.ascontiguousarray(xy, dtype=F32), bias_xy=bias_xy,
                      z_uniform=(lloyd_boundaries is None and lloyd_centroids is None and bias_table is None),
                      cell_idx=cells[0], cell_cnt=cells[1], cell_half_width=float(r_max) if cells[0] is not None else 0.0)
