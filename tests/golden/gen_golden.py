"""Generate golden vectors by running the PrismKV reference implementation.

Run with the reference's ``src/`` directory on ``PYTHONPATH`` (the reference
is needed only to regenerate the fixtures; the tests read the committed
files):

    PYTHONPATH=<PrismKV checkout>/src python tests/golden/gen_golden.py

Each case runs the reference's own public API on seeded inputs and stores
inputs and outputs in ``tests/golden/<case>.npz``.  The rotation ``R`` is
stored explicitly, because a QR factorisation may round differently on a
machine with another BLAS code path.
"""

from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref():
    from prismkv.quantizer.stacked_plane import StackedPlaneQuantizer
    from prismkv.quantizer.learned_codebook import LearnedSliceCodebook
    from prismkv.quantizer.bias_correction import BiasTable
    from prismkv.quantizer.lloyd_max import LloydMaxQuantizer1D
    from prismkv.quantizer.polar_attention import PolarAttentionApprox
    from prismkv.cache.backend import PrismKVBackend
    from prismkv.cache.cache_config import PrismKVConfig
    from prismkv.cuda import polar_attn_fwd, CUDA_AVAILABLE
    assert not CUDA_AVAILABLE
    return dict(SPQ=StackedPlaneQuantizer, LSC=LearnedSliceCodebook, BT=BiasTable,
                LM=LloydMaxQuantizer1D, PAA=PolarAttentionApprox, Backend=PrismKVBackend,
                Config=PrismKVConfig, polar_attn_fwd=polar_attn_fwd)


def edge_rows(R: torch.Tensor, g: torch.Generator) -> torch.Tensor:
    """Rows that stress the binning: zeros, near-axis, huge, tiny, inf, NaN."""
    d = R.shape[0]
    rows = [torch.zeros(d), torch.zeros(d)]
    rows += [R[k].clone() for k in (0, 1, 2, 5)]            # rotate to ~e_k: near-zero triplets
    rows += [-R[4].clone(), 3.0 * R[7].clone()]
    rows.append(torch.randn(d, generator=g) * 1e3)
    rows.append(torch.randn(d, generator=g) * 1e-30)
    r = torch.randn(d, generator=g); r[3] = float("inf"); rows.append(r)
    r = torch.randn(d, generator=g); r[10] = float("nan"); rows.append(r)
    r = torch.randn(d, generator=g); r[0] = -float("inf"); rows.append(r)
    return torch.stack(rows).float()


def synthetic_codebook(Cz: int, K: int, r_max: float, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    ang = (torch.rand(Cz, K, generator=g) * 2 - 1) * math.pi
    rad = torch.sqrt(torch.rand(Cz, K, generator=g)) * r_max * 0.6
    return torch.stack([rad * torch.cos(ang), rad * torch.sin(ang)], dim=-1).float()


def synthetic_bias(Cz: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(Cz, 3, generator=g) * 0.05).float()


def quant_state(q):
    out = dict(dim=q.dim, bits=np.array([q.bits_z, q.bits_r, q.bits_theta], np.int32),
               ranges=np.array([q.z_min, q.z_max, q.r_max], np.float64),
               R=q.R.numpy().astype(np.float32))
    if q._codebooks is not None:
        out["codebook"] = q._codebooks.codebooks.numpy().astype(np.float32)
    if q._lloyd_max_z is not None:
        out["lloyd_boundaries"] = q._lloyd_max_z.boundaries.numpy().astype(np.float32)
        out["lloyd_centroids"] = q._lloyd_max_z.centroids.numpy().astype(np.float32)
    if q._bias is not None:
        out["bias_table"] = q._bias.table.numpy().astype(np.float32)
        out["bias_delta_z"] = np.float64(q._bias.delta_z)
    return out


def save(name, **arrays):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **arrays)
    print(f"{name}: {os.path.getsize(path) / 1024:.1f} KB")


def enc_case(ref, name, bits, n, seed, scale_rows=False, codebook=False, bias=False,
             lloyd=False, dim=96):
    q = ref["SPQ"](dim=dim, bits_z=bits[0], bits_r=bits[1], bits_theta=bits[2], seed=42)
    g = torch.Generator().manual_seed(seed)
    if lloyd:
        calib = torch.randn(512, dim, generator=g)
        q.calibrate_lloyd_max_z(calib)
    if codebook:
        Cz, K = 1 << bits[0], 1 << (bits[1] + bits[2])
        cb = synthetic_codebook(Cz, K, q.r_max, seed + 1)
        q._codebooks = ref["LSC"](cb, Cz, K, q.z_min, q.z_max, q.r_max)
    if bias:
        q._bias = ref["BT"](synthetic_bias(1 << bits[0], seed + 2),
                            delta_z=(q.z_max - q.z_min) / (1 << bits[0]))
    X = torch.randn(n, dim, generator=g)
    if scale_rows:
        X = X * (0.5 + 1.5 * torch.rand(n, 1, generator=g))
    X = torch.cat([X, edge_rows(q.R, g)], dim=0).float()
    codes = q.encode(X)
    ok = torch.isfinite(X).all(dim=1)
    dec = q.decode(codes[:64])
    # every code value once, packed m per row
    total = 1 << sum(bits)
    allc = torch.arange(total, dtype=torch.int64)
    pad = (-total) % q.m
    allc = torch.cat([allc, torch.zeros(pad, dtype=torch.int64)]).reshape(-1, q.m)
    dec_all = q.decode(allc)
    save(name, X=X.numpy(), codes=codes.numpy().astype(np.int16), finite_rows=ok.numpy(),
         decoded=dec.numpy(), all_codes=allc.numpy().astype(np.int16),
         decoded_all=dec_all.numpy(), **quant_state(q))


def backend_case(ref):
    be = ref["Backend"](ref["Config"](), head_dim=64)
    g = torch.Generator().manual_seed(7)
    k = torch.randn(256, 64, generator=g)
    v = torch.randn(256, 64, generator=g) * 2.0
    kc, vc = be.compress(k, v)
    kd, vd = be.decompress(kc, vc)
    q = be._quantizer
    save("backend_d64", k=k.numpy(), v=v.numpy(), k_codes=kc.numpy(), v_codes=vc.numpy(),
         k_dec=kd.numpy(), v_dec=vd.numpy(), head_dim=np.int32(64), **quant_state(q))


def attn_v1_case(ref):
    # Config-1 shape with a shorter context: B=1, H=8, d=96, 4+4+4, seed 42 rotation.
    d, B, H, S = 96, 1, 8, 64
    q = ref["SPQ"](dim=d, seed=42)
    g = torch.Generator().manual_seed(0)
    K = torch.randn(B, H, S, d, generator=g)
    V = torch.randn(B, H, S, d, generator=g)
    Q = torch.randn(B, H, 1, d, generator=g)
    kc = q.encode(K.reshape(-1, d)).reshape(B, H, S, -1).to(torch.int16)
    vc = q.encode(V.reshape(-1, d)).reshape(B, H, S, -1).to(torch.int16)
    vdec = q.decode(vc.reshape(-1, q.m).long()).reshape(B, H, S, d)
    paa = ref["PAA"](bits_z=4, bits_r=4, bits_theta=4, z_min=q.z_min, z_max=q.z_max,
                     r_max=q.r_max, scale=d ** -0.5, R=q.R)
    out, w = paa.forward(Q, kc, vdec)
    save("attn_v1", q=Q.numpy(), k_codes=kc.numpy(), v_codes=vc.numpy(), out=out.numpy(),
         weights=w.numpy(), **quant_state(q))


def attn_v2_gqa_case(ref):
    # Learned codebook + BiasTable, GQA 8 query / 2 KV heads; composite oracle.
    d, B, Hkv, Hq, S = 96, 2, 2, 8, 40
    q = ref["SPQ"](dim=d, seed=42)
    cb = synthetic_codebook(16, 256, q.r_max, 11)
    q._codebooks = ref["LSC"](cb, 16, 256, q.z_min, q.z_max, q.r_max)
    q._bias = ref["BT"](synthetic_bias(16, 12), delta_z=(q.z_max - q.z_min) / 16)
    g = torch.Generator().manual_seed(3)
    K = torch.randn(B, Hkv, S, d, generator=g)
    V = torch.randn(B, Hkv, S, d, generator=g)
    Q = torch.randn(B, Hq, 1, d, generator=g).to(torch.bfloat16).float()
    kc = q.encode(K.reshape(-1, d)).reshape(B, Hkv, S, -1)
    vc = q.encode(V.reshape(-1, d)).reshape(B, Hkv, S, -1)
    kd = q.decode(kc.reshape(-1, q.m)).reshape(B, Hkv, S, d)
    vd = q.decode(vc.reshape(-1, q.m)).reshape(B, Hkv, S, d)
    G = Hq // Hkv
    kd = kd.repeat_interleave(G, dim=1)
    vd = vd.repeat_interleave(G, dim=1)
    w = torch.softmax((Q @ kd.transpose(-1, -2)) * d ** -0.5, dim=-1)
    out = w @ vd
    save("attn_v2_gqa", q=Q.numpy(), k_codes=kc.numpy().astype(np.int16),
         v_codes=vc.numpy().astype(np.int16), out=out.numpy(), **quant_state(q))


def scores_case(ref, name, B, H, Sq, Sk, d, bits, seed):
    q = ref["SPQ"](dim=d, bits_z=bits[0], bits_r=bits[1], bits_theta=bits[2], seed=0)
    g = torch.Generator().manual_seed(seed)
    Q = torch.randn(B, H, Sq, d, generator=g)
    K = torch.randn(B, H, Sk, d, generator=g)
    kc = q.encode(K.reshape(-1, d)).reshape(B, H, Sk, -1).to(torch.int16)
    Qr = (Q.reshape(-1, d) @ q.R.T).reshape(B, H, Sq, d)
    Cz = 1 << bits[0]
    kw = dict(z_min=q.z_min, delta_z=(q.z_max - q.z_min) / Cz, r_max=q.r_max,
              delta_r=q.r_max / max((1 << bits[1]) - 1, 1),
              delta_theta=2.0 * math.pi / max((1 << bits[2]) - 1, 1),
              scale=1.0 / math.sqrt(d), bits_z=bits[0], bits_r=bits[1], bits_theta=bits[2])
    s = ref["polar_attn_fwd"](Qr, kc, **kw)
    save(name, Q_rot=Qr.numpy(), k_codes=kc.numpy(), scores=s.numpy(),
         params=np.array([kw["z_min"], kw["delta_z"], kw["r_max"], kw["delta_r"],
                          kw["delta_theta"], kw["scale"]], np.float64),
         bits=np.array(bits, np.int32))


def raw_cache_case(ref):
    """RawKVCache over one (batch, head) group, two updates, and a 2x3-group single update."""
    from prismkv.cache.raw_cache import RawKVCache
    be = ref["Backend"](ref["Config"](), head_dim=64)
    g = torch.Generator().manual_seed(21)
    k1, v1 = torch.randn(1, 1, 5, 64, generator=g), torch.randn(1, 1, 5, 64, generator=g)
    k2, v2 = torch.randn(1, 1, 3, 64, generator=g), torch.randn(1, 1, 3, 64, generator=g)
    cache = RawKVCache(be)
    cache.update(0, k1, v1)
    kf, vf = cache.update(0, k2, v2)
    kc, vc = cache.get_codes(0)
    k3, v3 = torch.randn(2, 3, 4, 64, generator=g), torch.randn(2, 3, 4, 64, generator=g)
    kf3, vf3 = RawKVCache(be).update(1, k3, v3)
    save("raw_cache_d64", k1=k1.numpy(), v1=v1.numpy(), k2=k2.numpy(), v2=v2.numpy(),
         k_full=kf.numpy(), v_full=vf.numpy(), k_codes=kc.numpy(), v_codes=vc.numpy(),
         seq_len=np.int32(cache.get_seq_length(0)), k3=k3.numpy(), v3=v3.numpy(),
         k3_full=kf3.numpy(), v3_full=vf3.numpy(), **quant_state(be._quantizer))


def kv_cache_case(ref):
    """PrismKVCache (HF DynamicCache) over two updates, and the file its save_cache writes."""
    from prismkv.cache.kv_cache import PrismKVCache
    from prismkv.cache.cache_store import save_cache
    g = torch.Generator().manual_seed(22)
    k1, v1 = torch.randn(1, 2, 4, 96, generator=g), torch.randn(1, 2, 4, 96, generator=g)
    k2, v2 = torch.randn(1, 2, 1, 96, generator=g), torch.randn(1, 2, 1, 96, generator=g)
    cache = PrismKVCache(ref["Config"]())
    cache.update(k1, v1, 0)
    kf, vf = cache.update(k2, v2, 0)
    save("kv_cache_d96", k1=k1.numpy(), v1=v1.numpy(), k2=k2.numpy(), v2=v2.numpy(),
         k_full=kf.numpy(), v_full=vf.numpy(), **quant_state(cache._quantizers[0]))
    one = PrismKVCache(ref["Config"]())
    one.update(k1, v1, 0)
    save_cache(one, os.path.join(HERE, "ref_cache_store.npz"))
    print(f"ref_cache_store: {os.path.getsize(os.path.join(HERE, 'ref_cache_store.npz')) / 1024:.1f} KB")


def vllm_block_case(ref):
    """VLLMSwapCompressor block round trip: fp16 (heads, block, 64) -> int16 codes -> fp16."""
    from prismkv.cache.vllm_adapter import VLLMSwapCompressor
    comp = VLLMSwapCompressor(ref["Config"](), head_dim=64, n_layers=2)
    g = torch.Generator().manual_seed(23)
    kb = torch.randn(2, 16, 64, generator=g).half()
    vb = torch.randn(2, 16, 64, generator=g).half()
    kc, vc = comp.compress_block(1, 7, kb, vb)
    kd, vd = comp.decompress_block(1, 7, 2, 16, dtype=torch.float16, device="cpu")
    save("vllm_block_d64", k_block=kb.numpy(), v_block=vb.numpy(), k_codes=kc.numpy(), v_codes=vc.numpy(),
         k_dec=kd.numpy(), v_dec=vd.numpy(), **quant_state(comp._backends[1]._quantizer))


def files_case(ref):
    """The reference writes a prismkv-cb-v1 codebook file and a Lloyd-Max z file with its own save
    methods (learned_codebook.py:275-323, lloyd_max.py:156-185), then encodes seeded vectors after
    loading each file into a fresh quantizer (stacked_plane.py:183-204, :349-356)."""
    g = torch.Generator().manual_seed(21)
    q = ref["SPQ"](dim=96, bits_z=4, bits_r=4, bits_theta=4, seed=42)
    cb = ref["LSC"](synthetic_codebook(16, 256, q.r_max, 13), bins_z=16, K=256, z_min=q.z_min, z_max=q.z_max,
                    r_max=q.r_max)
    cb_path = os.path.join(HERE, "ref_codebook_444.npz")
    cb.save(cb_path)
    lq = ref["SPQ"](dim=96, bits_z=4, bits_r=4, bits_theta=4, seed=42)
    lq.calibrate_lloyd_max_z(torch.randn(4096, 96, generator=g))
    lm_path = os.path.join(HERE, "ref_lloyd_z.npz")
    lq.save_lloyd_max_z(lm_path)
    x = torch.cat([torch.randn(512, 96, generator=g) * 1.3, edge_rows(q.R, g)])
    qc = ref["SPQ"](dim=96, bits_z=4, bits_r=4, bits_theta=4, seed=42)
    qc.load_codebooks(cb_path)
    ql = ref["SPQ"](dim=96, bits_z=4, bits_r=4, bits_theta=4, seed=42)
    ql.load_lloyd_max_z(lm_path)
    save("files_codes", x=x.numpy(), codes_cb=qc.encode(x).numpy().astype(np.int16),
         codes_lloyd=ql.encode(x).numpy().astype(np.int16),
         R=q.R.numpy().astype(np.float32))


CASES = {"files": files_case, "enc": None, "backend_d64": backend_case, "attn_v1": attn_v1_case, "attn_v2_gqa": attn_v2_gqa_case,
         "raw_cache_d64": raw_cache_case, "kv_cache_d96": kv_cache_case, "vllm_block_d64": vllm_block_case}


def main():
    if not any("reference" in p for p in sys.path + os.environ.get("PYTHONPATH", "").split(":")):
        print("set PYTHONPATH to the reference's src directory", file=sys.stderr)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = _ref()
    only = sys.argv[1:]                      # case names to (re)generate; none = all
    if only:
        for name in only:
            CASES[name](ref)
        return
    enc_case(ref, "enc_v1_444", (4, 4, 4), 768, seed=0)
    enc_case(ref, "enc_v1_332", (3, 3, 2), 384, seed=1, scale_rows=True)
    enc_case(ref, "enc_v2_cb_bias", (4, 4, 4), 384, seed=2, codebook=True, bias=True)
    enc_case(ref, "enc_lloyd", (4, 4, 4), 384, seed=3, lloyd=True)
    enc_case(ref, "enc_v2_lloyd_bias", (4, 4, 4), 384, seed=4, codebook=True, bias=True,
             lloyd=True)
    enc_case(ref, "enc_v2_332", (3, 3, 2), 256, seed=5, codebook=True)
    backend_case(ref)
    attn_v1_case(ref)
    attn_v2_gqa_case(ref)
    scores_case(ref, "scores_d66", 1, 2, 4, 6, 66, (4, 4, 4), 42)
    scores_case(ref, "scores_d96_332", 2, 3, 3, 37, 96, (3, 3, 2), 5)
    raw_cache_case(ref)
    kv_cache_case(ref)
    vllm_block_case(ref)
    files_case(ref)


if __name__ == "__main__":
    main()
