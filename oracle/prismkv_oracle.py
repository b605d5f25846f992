"""CPU oracle for the PrismKV quantized-KV hot path.

TEST INFRASTRUCTURE ONLY.  This module is the oracle the CUDA path is
compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it,
and only to check results or as the timed CPU reference -- never as part of
the product path in ``prismkv_b200``.

It restates, in NumPy, the reference's CPU algorithm (PrismKV v1.4.1, whose
arithmetic is PyTorch CPU kernels: torch>=2.1, pinned here by the installed
2.11.0).  Every function cites the reference file:line it follows.  The
fp32 op sequence is mirrored operation by operation:

* a division by a Python scalar is a true fp32 division by the scalar cast
  to fp32 (not a multiply by a reciprocal);
* ``x ** 2`` is ``x * x``; no fused multiply-add is formed between ops;
* ``torch.round`` rounds half to even (``np.rint``);
* ``.long()`` of NaN, +-inf or a value of magnitude >= 2**63 yields
  INT64_MIN, which the following ``clamp(0, C-1)`` turns into bin 0;
* ``torch.bucketize(right=False)`` counts boundaries strictly below the
  value, and a NaN lands past the last boundary.

Two reference kernels are not reproducible bit for bit on another machine:
the fp32 GEMM of the rotation (MKL, blocking unknown) and the vectorised
``sqrt`` / ``atan2`` (each within 1 ulp).  The oracle uses NumPy's fp32 GEMM
and correctly rounded ``sqrt``/``atan2``.  Codes produced either way agree
except where the exact value lies within the rounding error of a bin
boundary; ``oracle.ties`` classifies every such mismatch in fp64.

Parity of this restatement is pinned against golden vectors produced by
running the reference itself (``tests/golden/gen_golden.py`` →
``tests/golden/*.npz``; checked by ``tests/test_oracle_golden.py``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np

F32 = np.float32
I64_MIN = np.iinfo(np.int64).min


# ---------------------------------------------------------------------------
# Parameters
# ---------------------------------------------------------------------------

@dataclass
class QuantParams:
    """State of one ``StackedPlaneQuantizer`` (stacked_plane.py:58-108).

    ``z_min``/``z_max``/``r_max`` are Python floats exactly as the reference
    holds them; they are cast to fp32 inside each op, as torch does.
    """

    dim: int
    bits_z: int = 4
    bits_r: int = 4
    bits_theta: int = 4
    z_min: float = 0.0
    z_max: float = 0.0
    r_max: float = 0.0
    codebook: Optional[np.ndarray] = None          # (C_z, K, 2) fp32, learned_codebook.py:150
    lloyd_boundaries: Optional[np.ndarray] = None  # (C_z+1,) fp32, lloyd_max.py:57
    lloyd_centroids: Optional[np.ndarray] = None   # (C_z,) fp32
    bias_table: Optional[np.ndarray] = None        # (C_z, 3) fp32, bias_correction.py:51
    bias_delta_z: float = 0.0                      # BiasTable.delta_z, bias_correction.py:53

    @property
    def m(self) -> int:
        return self.dim // 3

    @property
    def Cz(self) -> int:
        return 1 << self.bits_z

    @property
    def Cr(self) -> int:
        return 1 << self.bits_r

    @property
    def Ct(self) -> int:
        return 1 << self.bits_theta

    @property
    def delta_z(self) -> float:
        # stacked_plane.py:239 (Python double)
        return (self.z_max - self.z_min) / self.Cz

    @classmethod
    def default(cls, dim: int, bits_z=4, bits_r=4, bits_theta=4) -> "QuantParams":
        # stacked_plane.py:97-101: conservative ranges +-sqrt(dim)
        c = math.sqrt(dim)
        return cls(dim=dim, bits_z=bits_z, bits_r=bits_r, bits_theta=bits_theta,
                   z_min=-c, z_max=c, r_max=c)


# ---------------------------------------------------------------------------
# fp32 helpers mirroring torch CPU semantics
# ---------------------------------------------------------------------------

def to_long(v: np.ndarray) -> np.ndarray:
    """``Tensor.long()`` of an fp32 tensor on x86: NaN/inf/out-of-range → INT64_MIN."""
    v = np.asarray(v)
    out = np.full(v.shape, I64_MIN, dtype=np.int64)
    with np.errstate(invalid="ignore"):
        ok = np.isfinite(v) & (np.abs(v.astype(np.float64)) < 2.0 ** 63)
    out[ok] = v[ok].astype(np.int64)
    return out


def atan2_f32(y: np.ndarray, x: np.ndarray) -> np.ndarray:
    """Correctly rounded fp32 atan2 (the reference's vectorised atan2 is within 1 ulp)."""
    return np.arctan2(y.astype(np.float64), x.astype(np.float64)).astype(F32)


def cos_f32(t: np.ndarray) -> np.ndarray:
    return np.cos(t.astype(np.float64)).astype(F32)


def sin_f32(t: np.ndarray) -> np.ndarray:
    return np.sin(t.astype(np.float64)).astype(F32)


# ---------------------------------------------------------------------------
# Per-component binning (elementwise, fp32) -- used by encode and by ties.py
# ---------------------------------------------------------------------------

def bin_z_uniform(z: np.ndarray, p: QuantParams) -> np.ndarray:
    """stacked_plane.py:237-241: clamp(floor((z - z_min) / delta_z), 0, C_z-1)."""
    z = np.asarray(z, dtype=F32)
    with np.errstate(invalid="ignore", over="ignore"):
        t = (z - F32(p.z_min)).astype(F32)
        t = (t / F32(p.delta_z)).astype(F32)
        i = to_long(np.floor(t))
    return np.clip(i, 0, p.Cz - 1)


def bin_z_lloyd(z: np.ndarray, p: QuantParams) -> np.ndarray:
    """lloyd_max.py:106-124: bucketize(z, boundaries[1:-1]) then clamp(0, K-1)."""
    z = np.asarray(z, dtype=F32)
    inner = p.lloyd_boundaries[1:-1].astype(F32)
    # searchsorted(side='left') == torch.bucketize(right=False); NaN sorts last.
    i = np.searchsorted(inner, z, side="left").astype(np.int64)
    return np.clip(i, 0, p.Cz - 1)


def bin_z(z: np.ndarray, p: QuantParams) -> np.ndarray:
    """stacked_plane.py:233-241."""
    if p.lloyd_boundaries is not None:
        return bin_z_lloyd(z, p)
    return bin_z_uniform(z, p)


def bin_r(r: np.ndarray, p: QuantParams) -> np.ndarray:
    """stacked_plane.py:249,252-253 applied to an fp32 radius."""
    r = np.asarray(r, dtype=F32)
    with np.errstate(invalid="ignore"):
        r = np.minimum(np.maximum(r, F32(0.0)), F32(p.r_max))  # clamp(0, r_max), NaN kept
        t = (r / F32(p.r_max)).astype(F32)
        t = (t * F32(p.Cr - 1)).astype(F32)
        i = to_long(np.rint(t))
    return np.clip(i, 0, p.Cr - 1)


def bin_theta(theta: np.ndarray, p: QuantParams) -> np.ndarray:
    """stacked_plane.py:250,255-256 applied to an fp32 angle."""
    theta = np.asarray(theta, dtype=F32)
    with np.errstate(invalid="ignore"):
        t = (theta + F32(math.pi)).astype(F32)
        t = (t / F32(2 * math.pi)).astype(F32)
        t = (t * F32(p.Ct - 1)).astype(F32)
        i = to_long(np.rint(t))
    return np.clip(i, 0, p.Ct - 1)


def radius_f32(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    """stacked_plane.py:249: sqrt(x**2 + y**2) in fp32, no fused multiply-add."""
    x = np.asarray(x, dtype=F32)
    y = np.asarray(y, dtype=F32)
    with np.errstate(over="ignore", invalid="ignore"):
        s = ((x * x).astype(F32) + (y * y).astype(F32)).astype(F32)
        return np.sqrt(s).astype(F32)


def nearest_centroid(x: np.ndarray, y: np.ndarray, i_z: np.ndarray, p: QuantParams) -> np.ndarray:
    """learned_codebook.py:217-248: index of the nearest centroid of bin ``i_z``.

    The reference measures Euclidean distance with ``torch.cdist`` and takes
    the first minimal index (``argmin``, which treats NaN as minimal).  For
    a finite point, distances are evaluated here in fp64 from the fp32
    point, so the result is the exact nearest centroid; cdist's own rounding
    can only reorder centroids whose distances agree to within its error
    (classified by ``ties.py``).

    For more than 25 points or centroids, cdist evaluates the squared
    distance as ``-2 p.c + |p|^2 + |c|^2`` (one matrix product), so a point
    with an infinite coordinate gets NaN for every centroid where an
    ``inf - inf`` or ``inf * 0`` arises and +inf elsewhere; ``argmin`` then
    returns the first NaN, or 0.  That category is independent of summation
    order and is reproduced exactly.  A NaN point gives index 0.
    """
    cb = p.codebook.astype(np.float64)
    cb32 = p.codebook.astype(F32)
    x32 = np.asarray(x, dtype=F32).reshape(-1)
    y32 = np.asarray(y, dtype=F32).reshape(-1)
    px = x32.astype(np.float64)
    py = y32.astype(np.float64)
    iz = np.asarray(i_z).reshape(-1)
    out = np.zeros(px.shape[0], dtype=np.int64)
    finite = np.isfinite(px) & np.isfinite(py)
    chunk = 65536
    for b in range(p.Cz):
        idx = np.nonzero((iz == b) & finite)[0]
        c = cb[b]                                              # (K, 2)
        for s in range(0, idx.size, chunk):
            sel = idx[s:s + chunk]
            d2 = (px[sel, None] - c[None, :, 0]) ** 2 + (py[sel, None] - c[None, :, 1]) ** 2
            out[sel] = np.argmin(d2, axis=1)
    inf_pts = np.nonzero(~finite & ~np.isnan(px) & ~np.isnan(py))[0]
    for i in inf_pts:
        c = cb32[int(iz[i])]
        with np.errstate(invalid="ignore", over="ignore"):
            t = ((F32(-2.0) * x32[i]) * c[:, 0]).astype(F32) + ((F32(-2.0) * y32[i]) * c[:, 1]).astype(F32)
            t = t + (x32[i] * x32[i] + y32[i] * y32[i]) + (c[:, 0] * c[:, 0] + c[:, 1] * c[:, 1])
        nan = np.nonzero(np.isnan(t))[0]
        out[i] = int(nan[0]) if nan.size else int(np.argmin(t))
    return out.reshape(np.shape(x))


# ---------------------------------------------------------------------------
# Encode / decode
# ---------------------------------------------------------------------------

def rotate(X: np.ndarray, R: np.ndarray) -> np.ndarray:
    """stacked_plane.py:226: ``vectors @ R.T`` (fp32 GEMM)."""
    return (np.asarray(X, dtype=F32) @ np.asarray(R, dtype=F32).T).astype(F32)


def encode_rotated(rot: np.ndarray, p: QuantParams) -> np.ndarray:
    """stacked_plane.py:228-262 applied to already rotated fp32 vectors."""
    z = rot[:, 0::3]
    x = rot[:, 1::3]
    y = rot[:, 2::3]
    i_z = bin_z(z, p)
    if p.codebook is not None:
        i_flat = nearest_centroid(x, y, i_z, p)
    else:
        r = radius_f32(x, y)
        th = atan2_f32(y, x)
        i_r = bin_r(r, p)
        i_t = bin_theta(th, p)
        i_flat = (i_r << p.bits_theta) | i_t
    return (i_z << (p.bits_r + p.bits_theta)) | i_flat


def encode(X: np.ndarray, R: np.ndarray, p: QuantParams) -> np.ndarray:
    """``StackedPlaneQuantizer.encode`` (stacked_plane.py:210-262) → (N, m) int64."""
    X = np.asarray(X, dtype=F32)
    if X.shape[0] == 0:
        return np.zeros((0, p.m), dtype=np.int64)
    return encode_rotated(rotate(X, R), p)


def dequant_rotated(codes: np.ndarray, p: QuantParams) -> np.ndarray:
    """stacked_plane.py:278-324: codes → rotated-space triplets (N, dim) fp32.

    Includes the BiasTable subtraction (bias_correction.py:58-91).
    """
    codes = np.asarray(codes).astype(np.int64)
    bits_flat = p.bits_r + p.bits_theta
    i_flat = codes & ((1 << bits_flat) - 1)
    i_z = codes >> bits_flat
    if p.lloyd_centroids is not None:
        # lloyd_max.py:126-140
        z_q = p.lloyd_centroids.astype(F32)[np.clip(i_z, 0, p.Cz - 1)]
    else:
        # stacked_plane.py:292-293: z_min + (i_z + 0.5) * delta_z
        t = (i_z.astype(F32) + F32(0.5)).astype(F32)
        t = (t * F32(p.delta_z)).astype(F32)
        z_q = (F32(p.z_min) + t).astype(F32)
    if p.codebook is not None:
        # learned_codebook.py:250-269
        xy = p.codebook.astype(F32)[i_z, i_flat]
        x_q, y_q = xy[..., 0], xy[..., 1]
    else:
        # stacked_plane.py:297-310
        i_t = (i_flat & ((1 << p.bits_theta) - 1)).astype(F32)
        i_r = ((i_flat >> p.bits_theta) & ((1 << p.bits_r) - 1)).astype(F32)
        r_q = ((i_r / F32(p.Cr - 1)).astype(F32) * F32(p.r_max)).astype(F32)
        th = (i_t / F32(p.Ct - 1)).astype(F32)
        th = (th * F32(2.0)).astype(F32)
        th = (th * F32(math.pi)).astype(F32)
        th = (th - F32(math.pi)).astype(F32)
        x_q = (r_q * cos_f32(th)).astype(F32)
        y_q = (r_q * sin_f32(th)).astype(F32)
    N = codes.shape[0]
    out = np.zeros((N, p.dim), dtype=F32)
    out[:, 0::3] = z_q
    out[:, 1::3] = x_q
    out[:, 2::3] = y_q
    if p.bias_table is not None:
        # bias_correction.py:81-89: subtract clamp(table[i_z], +-delta_z/2)
        clip = F32(p.bias_delta_z / 2.0)
        b = np.clip(p.bias_table.astype(F32)[i_z], -clip, clip).astype(F32)
        out[:, 0::3] = (out[:, 0::3] - b[..., 0]).astype(F32)
        out[:, 1::3] = (out[:, 1::3] - b[..., 1]).astype(F32)
        out[:, 2::3] = (out[:, 2::3] - b[..., 2]).astype(F32)
    return out


def decode(codes: np.ndarray, R: np.ndarray, p: QuantParams) -> np.ndarray:
    """``StackedPlaneQuantizer.decode`` (stacked_plane.py:268-327) → (N, dim) fp32."""
    rq = dequant_rotated(codes, p)
    return (rq @ np.asarray(R, dtype=F32)).astype(F32)   # stacked_plane.py:327: @ R_inv.T == @ R


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------

def attention(q: np.ndarray, k_codes: np.ndarray, v_codes: np.ndarray, R: np.ndarray,
              p: QuantParams, scale: Optional[float] = None,
              seq_lens: Optional[np.ndarray] = None) -> np.ndarray:
    """Decode attention over packed K/V codes, evaluated in fp64.

    Computes ``softmax(q · decode(K)^T · scale) · decode(V)`` per query head
    -- the reference's ``PolarAttentionApprox.forward`` with decoded values
    (polar_attention.py:277-309; the polar score identity of
    polar_attention.py:113-212 equals the decoded dot product exactly) and,
    for learned codebooks / BiasTable / Lloyd-Max, the decode-then-attend
    composite (stacked_plane.py:268-327).

    q: (B, Hq, D) or (B, Hq, 1, D); k/v codes: (B, Hkv, S, m); Hq % Hkv == 0
    (grouped heads share KV head ``h // (Hq // Hkv)``).  ``seq_lens`` (B,)
    limits the valid tokens per batch row; an empty row yields zeros
    (softmax over nothing times an empty V).  Returns (B, Hq, D) float64.
    """
    q = np.asarray(q)
    if q.ndim == 4:
        q = q[:, :, 0, :]
    B, Hq, D = q.shape
    _, Hkv, S, m = k_codes.shape
    G = Hq // Hkv
    d = p.dim
    if scale is None:
        scale = d ** -0.5                                  # polar_attention.py:299-300
    R64 = np.asarray(R, dtype=np.float64)
    qr = q.astype(np.float64) @ R64.T                      # rotate the query once
    out = np.zeros((B, Hq, D), dtype=np.float64)
    for b in range(B):
        L = S if seq_lens is None else int(seq_lens[b])
        if L == 0:
            continue
        for hk in range(Hkv):
            kr = dequant_rotated(k_codes[b, hk, :L].reshape(L, m), p).astype(np.float64)
            vr = dequant_rotated(v_codes[b, hk, :L].reshape(L, m), p).astype(np.float64)
            for g in range(G):
                h = hk * G + g
                s = (kr @ qr[b, h]) * scale
                s = s - s.max()
                w = np.exp(s)
                w /= w.sum()
                out[b, h] = (w @ vr) @ R64
    return out


def polar_attention_forward_f32(q: np.ndarray, k_codes: np.ndarray, v: np.ndarray,
                                R: np.ndarray, p: QuantParams,
                                scale: Optional[float] = None) -> Tuple[np.ndarray, np.ndarray]:
    """fp32 restatement of ``PolarAttentionApprox.forward`` (polar_attention.py:277-309).

    Follows the reference step by step (rotate q, unpack codes, uniform
    dequant, polar -> cartesian query, three contractions, scale, softmax,
    weights @ v).  This is the CPU path the benchmark times as the
    reference; results are checked against :func:`attention`.  ``v`` is the decoded
    value tensor (B, H, Sk, d).  Returns (output, weights).
    """
    q = np.asarray(q, dtype=F32)
    B, H, Sq, d = q.shape
    if scale is None:
        scale = d ** -0.5
    qr = (q.reshape(-1, d) @ np.asarray(R, dtype=F32).T).astype(F32).reshape(B, H, Sq, d)
    scores = polar_dot_product_from_codes_f32(qr, k_codes, p)
    scores = (scores * F32(scale)).astype(F32)
    scores = scores - scores.max(axis=-1, keepdims=True)
    w = np.exp(scores).astype(F32)
    w = (w / w.sum(axis=-1, keepdims=True)).astype(F32)
    out = np.matmul(w, np.asarray(v, dtype=F32)).astype(F32)
    return out, w


def polar_dot_product_from_codes_f32(q_rot: np.ndarray, k_codes: np.ndarray, p: QuantParams,
                                     z_max: Optional[float] = None) -> np.ndarray:
    """polar_attention.py:153-212 for a query that is already rotated (R=None)."""
    codes = np.asarray(k_codes).astype(np.int64)
    Cz, Cr, Ct = p.Cz, p.Cr, p.Ct
    i_t = codes & ((1 << p.bits_theta) - 1)
    i_r = (codes >> p.bits_theta) & ((1 << p.bits_r) - 1)
    i_z = (codes >> (p.bits_theta + p.bits_r)) & ((1 << p.bits_z) - 1)
    zmax = p.z_max if z_max is None else z_max
    delta_z = (zmax - p.z_min) / Cz
    kz = (F32(p.z_min) + ((i_z.astype(F32) + F32(0.5)).astype(F32) * F32(delta_z)).astype(F32)).astype(F32)
    kr = ((i_r.astype(F32) / F32(max(Cr - 1, 1))).astype(F32) * F32(p.r_max)).astype(F32)
    kt = ((i_t.astype(F32) / F32(max(Ct - 1, 1))).astype(F32) * F32(2 * math.pi)).astype(F32)
    kt = (kt - F32(math.pi)).astype(F32)
    m = codes.shape[-1]
    qt = q_rot[..., : 3 * m].reshape(*q_rot.shape[:-1], m, 3).astype(F32)
    qz, qx, qy = qt[..., 0], qt[..., 1], qt[..., 2]
    q_r = np.sqrt(((qx * qx).astype(F32) + (qy * qy).astype(F32) + F32(1e-12)).astype(F32)).astype(F32)
    q_t = atan2_f32(qy, qx)
    qrx = (q_r * cos_f32(q_t)).astype(F32)
    qry = (q_r * sin_f32(q_t)).astype(F32)
    krx = (kr * cos_f32(kt)).astype(F32)
    kry = (kr * sin_f32(kt)).astype(F32)
    s = np.matmul(qz, np.swapaxes(kz, -1, -2))
    s = s + np.matmul(qrx, np.swapaxes(krx, -1, -2)) + np.matmul(qry, np.swapaxes(kry, -1, -2))
    return s.astype(F32)


def polar_scores(Q_rot: np.ndarray, K_codes: np.ndarray, z_min: float, delta_z: float,
                 r_max: float, scale: float, bits_z: int, bits_r: int, bits_theta: int) -> np.ndarray:
    """``prismkv.cuda.polar_attn_fwd`` contract (cuda/__init__.py:23-92), fp64.

    Scores ``scale * <Q_rot, dequant(K)>`` for a pre-rotated query, with the
    uniform v1 dequant and ``z_max = z_min + delta_z * 2**bits_z``
    (cuda/__init__.py:82-83).  Returns (B, H, Sq, Sk) float64.
    """
    Cz = 1 << bits_z
    dim = 3 * K_codes.shape[-1]
    p = QuantParams(dim=dim, bits_z=bits_z, bits_r=bits_r, bits_theta=bits_theta,
                    z_min=z_min, z_max=z_min + delta_z * Cz, r_max=r_max)
    B, H, Sk, m = K_codes.shape
    kr = dequant_rotated(K_codes.reshape(-1, m), p).astype(np.float64).reshape(B, H, Sk, dim)
    Q = np.asarray(Q_rot, dtype=np.float64)[..., :dim]
    return np.einsum("bhqd,bhkd->bhqk", Q, kr) * scale


# ---------------------------------------------------------------------------
# Split-sequence log-sum-exp combine
# ---------------------------------------------------------------------------

def lse_combine(m: np.ndarray, l: np.ndarray, o: np.ndarray) -> np.ndarray:
    """Combine per-shard softmax partials, in fp64.

    Shard ``i`` holds ``m_i = max_t s_t`` (natural-log domain),
    ``l_i = sum_t exp(s_t - m_i)`` and ``o_i = sum_t exp(s_t - m_i) v_t``
    over its tokens.  The combined output is
    ``sum_i exp(m_i - M) o_i / sum_i exp(m_i - M) l_i`` with ``M = max m_i``.
    Shards with no tokens carry ``m_i = -inf, l_i = 0`` and drop out.
    Shapes: m, l (n, ...); o (n, ..., D).  Returns (..., D).
    """
    m = np.asarray(m, dtype=np.float64)
    l = np.asarray(l, dtype=np.float64)
    o = np.asarray(o, dtype=np.float64)
    M = m.max(axis=0)
    Msafe = np.where(np.isfinite(M), M, 0.0)
    w = np.where(np.isfinite(m), np.exp(m - Msafe), 0.0)
    L = (w * l).sum(axis=0)
    O = (w[..., None] * o).sum(axis=0)
    with np.errstate(invalid="ignore", divide="ignore"):
        res = np.where(L[..., None] > 0, O / np.where(L > 0, L, 1.0)[..., None], 0.0)
    return res
