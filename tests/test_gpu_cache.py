"""GPU parity of the KV-cache adapters (prismkv_b200.cache) with the reference's.

Fixtures come from running the reference's own RawKVCache, PrismKVCache,
save_cache and VLLMSwapCompressor on seeded inputs (tests/golden/gen_golden.py).
Codes must match except at proven rounding ties (oracle.classify); decoded
tensors within 1e-5 (fp32) or one fp16 ulp.
"""

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden, params_from
from prismkv_b200 import decode_attention
from prismkv_b200.cache import (PrismKVBackend, PrismKVCache, PrismKVConfig, RawKVCache, VLLMSwapCompressor,
                                load_cache, save_cache)

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _pad(x, d):
    x = np.asarray(x, dtype=np.float32).reshape(-1, x.shape[-1])
    return np.concatenate([x, np.zeros((x.shape[0], d - x.shape[1]), np.float32)], axis=1)


def _codes_match(f, X, ours, theirs):
    p = params_from(f)
    rep = oracle.classify(X, f["R"], p, np.asarray(ours, np.int64), np.asarray(theirs, np.int64) & 0xFFF)
    assert rep.unexplained == 0, rep.examples
    return rep


def test_backend_matches_reference(cuda_ready):
    f = load_golden("backend_d64")
    be = PrismKVBackend(PrismKVConfig(), head_dim=64)
    assert np.array_equal(be.quantizer.R.numpy(), f["R"])
    kc, vc = be.compress(torch.from_numpy(f["k"]).to(DEV), torch.from_numpy(f["v"]).to(DEV))
    assert kc.dtype == torch.int16 and kc.shape == (256, 22)
    _codes_match(f, _pad(f["k"], 66), kc.cpu().numpy(), f["k_codes"])
    _codes_match(f, _pad(f["v"], 66), vc.cpu().numpy(), f["v_codes"])
    kd, vd = be.decompress(torch.from_numpy(f["k_codes"]).to(DEV), torch.from_numpy(f["v_codes"]).to(DEV))
    np.testing.assert_allclose(kd.cpu().numpy(), f["k_dec"], atol=1e-5, rtol=0)
    np.testing.assert_allclose(vd.cpu().numpy(), f["v_dec"], atol=1e-5, rtol=0)
    kc2, _ = be.compress(torch.from_numpy(f["k"]), torch.from_numpy(f["v"]))      # CPU tensors in and out
    assert kc2.device.type == "cpu" and torch.equal(kc2, kc.cpu())


def test_raw_cache_matches_reference(cuda_ready):
    f = load_golden("raw_cache_d64")
    cache = RawKVCache(PrismKVBackend(PrismKVConfig(), head_dim=64), initial_capacity=4)   # forces a regrow
    t = lambda a: torch.from_numpy(f[a]).to(DEV)
    cache.update(0, t("k1"), t("v1"))
    kf, vf = cache.update(0, t("k2"), t("v2"))
    assert kf.shape == (1, 1, 8, 64) and cache.get_seq_length(0) == int(f["seq_len"]) == 8
    np.testing.assert_allclose(kf.cpu().numpy(), f["k_full"], atol=1e-5, rtol=0)
    np.testing.assert_allclose(vf.cpu().numpy(), f["v_full"], atol=1e-5, rtol=0)
    kc, vc = cache.get_codes(0)
    assert kc.dtype == torch.int16 and kc.shape == f["k_codes"].shape
    Xk = _pad(np.concatenate([f["k1"].reshape(-1, 64), f["k2"].reshape(-1, 64)]), 66)
    _codes_match(f, Xk, kc.cpu().numpy(), f["k_codes"])
    k3f, v3f = RawKVCache(PrismKVBackend(PrismKVConfig(), head_dim=64)).update(1, t("k3"), t("v3"))
    assert k3f.shape == (2, 3, 4, 64)
    np.testing.assert_allclose(k3f.cpu().numpy(), f["k3_full"], atol=1e-5, rtol=0)
    np.testing.assert_allclose(v3f.cpu().numpy(), f["v3_full"], atol=1e-5, rtol=0)
    fp = cache.memory_footprint()
    assert fp["n_layers"] == 1 and fp["codes_bytes"] == 2 * 8 * 22 * 2 and "RawKVCache" in repr(cache)


def test_raw_cache_groups_keep_their_tokens_in_order(cuda_ready):
    """(batch, heads) groups over several updates: each group's context equals encode->decode
    of its own tokens in order (the reference's flat concatenation interleaves groups here)."""
    be = PrismKVBackend(PrismKVConfig(), head_dim=96)
    cache = RawKVCache(be, initial_capacity=3)
    g = torch.Generator(device=DEV).manual_seed(5)
    chunks = [torch.randn(2, 4, s, 96, generator=g, device=DEV) for s in (5, 1, 1, 7, 2)]
    for c in chunks:
        kf, vf = cache.update(0, c, -c)
    full = torch.cat(chunks, dim=2)
    ref = be.quantizer.decode(be.quantizer.encode(full.reshape(-1, 96))).reshape(full.shape)
    torch.testing.assert_close(kf, ref, atol=1e-5, rtol=0)
    assert cache.get_seq_length(0) == 16 and cache.cached_layers == [0]
    # the fused kernel on the cache buffers in place (head stride = capacity)
    q = torch.randn(2, 8, 96, generator=g, device=DEV)
    out = cache.attention(0, q)
    kc = be.quantizer.encode_compact(full.reshape(-1, 96)).view(2, 4, 16, 32)
    vc = be.quantizer.encode_compact(-full.reshape(-1, 96)).view(2, 4, 16, 32)
    torch.testing.assert_close(out, decode_attention(be.quantizer, q, kc, vc), atol=1e-5, rtol=0)
    cache.clear(0)
    assert cache.get_seq_length(0) == 0 and cache.cached_layers == []


def test_prismkv_cache_matches_reference(cuda_ready):
    from transformers import DynamicCache
    f = load_golden("kv_cache_d96")
    t = lambda a: torch.from_numpy(f[a]).to(DEV)
    cache = PrismKVCache(PrismKVConfig(), initial_capacity=2)
    assert isinstance(cache, DynamicCache)
    cache.update(t("k1"), t("v1"), 0)
    kf, vf = cache.update(t("k2"), t("v2"), 0)
    assert kf.shape == (1, 2, 5, 96)
    np.testing.assert_allclose(kf.cpu().numpy(), f["k_full"], atol=1e-5, rtol=0)
    np.testing.assert_allclose(vf.cpu().numpy(), f["v_full"], atol=1e-5, rtol=0)
    assert cache.get_seq_length(0) == 5
    kc, _ = cache.get_codes(0)
    assert kc.shape == (1, 2, 5, 32)
    assert cache.compression_ratio() == pytest.approx(96 * 2 / (32 * 2))
    cache.crop(3)
    assert cache.get_seq_length(0) == 3 and cache.get_codes(0)[0].shape[2] == 3
    assert "PrismKVCache" in repr(cache)


def test_prismkv_cache_reorder_and_store_round_trip(cuda_ready, tmp_path):
    g = torch.Generator(device=DEV).manual_seed(8)
    cache = PrismKVCache(PrismKVConfig())
    k = torch.randn(3, 2, 6, 64, generator=g, device=DEV)
    cache.update(k, 2 * k, 0)
    cache.update(k[:, :, :1], k[:, :, :1], 1)
    cache.reorder_cache(torch.tensor([2, 0, 1], device=DEV))
    kc, _ = cache.get_codes(0)
    path = tmp_path / "c.npz"
    save_cache(cache, path)
    back = load_cache(path, device=DEV)
    kc2, vc2 = back.get_codes(0)
    assert torch.equal(kc2, kc) and back.get_seq_length(0) == 6
    torch.testing.assert_close(back.layers[0].keys, cache.layers[0].keys, atol=1e-5, rtol=0)


def test_load_cache_reads_reference_file(cuda_ready):
    """A file written by the reference's save_cache loads here (flat layout, inferred head_dim)."""
    from conftest import GOLDEN
    import os
    f = load_golden("kv_cache_d96")
    back = load_cache(os.path.join(GOLDEN, "ref_cache_store.npz"), device=DEV)
    keys = back.layers[0].keys                           # (1, 1, batch*heads*seq, 96)
    assert keys.shape == (1, 1, 8, 96)
    # the reference's cache after its first update returns the same decoded rows
    np.testing.assert_allclose(keys.reshape(1, 2, 4, 96).cpu().numpy(), f["k_full"][:, :, :4], atol=1e-5, rtol=0)


def test_vllm_block_codec_matches_reference(cuda_ready):
    f = load_golden("vllm_block_d64")
    comp = VLLMSwapCompressor(PrismKVConfig(), head_dim=64, n_layers=2)
    kb, vb = torch.from_numpy(f["k_block"]).to(DEV), torch.from_numpy(f["v_block"]).to(DEV)
    kc, vc = comp.compress_block(1, 7, kb, vb)
    assert kc.device.type == "cpu" and kc.dtype == torch.int16 and kc.shape == (32, 22)
    _codes_match(f, _pad(f["k_block"].astype(np.float32), 66), kc.numpy(), f["k_codes"])
    _codes_match(f, _pad(f["v_block"].astype(np.float32), 66), vc.numpy(), f["v_codes"])
    kd, vd = comp.decompress_block(1, 7, 2, 16, dtype=torch.float16, device=DEV)
    assert kd.shape == (2, 16, 64) and kd.dtype == torch.float16 and kd.is_cuda
    np.testing.assert_allclose(kd.float().cpu().numpy(), f["k_dec"].astype(np.float32), atol=2e-3, rtol=1e-3)
    comp.evict_block(1, 7)
    with pytest.raises(KeyError):
        comp.decompress_block(1, 7, 2, 16)


def test_vllm_swap_loop_reuses_pinned_buffers(cuda_ready):
    """A swap loop without a per-block host wait: blocks compressed with sync=False decompress
    correctly (stream order), synchronize() makes their host codes complete, and an evicted
    block's pinned buffers serve the next block of the same shape."""
    comp = VLLMSwapCompressor(PrismKVConfig(), head_dim=96, n_layers=1)
    g = torch.Generator(device=DEV).manual_seed(3)
    blocks = [(torch.randn(4, 16, 96, generator=g, device=DEV).half(),
               torch.randn(4, 16, 96, generator=g, device=DEV).half()) for _ in range(3)]
    kept = [comp.compress_block(0, i, kb, vb, sync=False) for i, (kb, vb) in enumerate(blocks)]
    for i, (kb, vb) in enumerate(blocks):
        kd, vd = comp.decompress_block(0, i, 4, 16, dtype=torch.float32, device=DEV)
        ref_k = comp._backends[0].codec(torch.device(DEV)).decode(
            comp._backends[0].codec(torch.device(DEV)).encode(kb.reshape(64, 96), code_dtype=torch.int16))
        np.testing.assert_allclose(kd.reshape(64, 96).cpu().numpy(), ref_k.cpu().numpy(), atol=1e-6)
    comp.synchronize()
    first_k = kept[0][0]
    comp.evict_block(0, 0)
    kc, _ = comp.compress_block(0, 9, *blocks[1])
    assert kc.data_ptr() == first_k.data_ptr() or kept[0][1].data_ptr() == kc.data_ptr()
    assert comp.n_compressed_blocks == 3


def test_sidecar_json_and_binary_agree_with_the_reference(cuda_ready):
    """The sidecar's JSON API gives the reference backend's codes (golden backend_d64, through
    PrismKVBackend.compress); the binary transport gives the same codes and the same decoded
    vectors with raw arrays instead of decimal lists."""
    import json as _json
    import urllib.request
    from prismkv_b200 import sidecar
    f = load_golden("backend_d64")
    k, v = f["k"].astype(np.float32), f["v"].astype(np.float32)
    srv = sidecar.PrismKVSidecar(port=0)
    srv.start_background()
    url = f"http://127.0.0.1:{srv.port}"
    try:
        req = urllib.request.Request(url + "/compress", method="POST", headers={"Content-Type": "application/json"},
                                     data=_json.dumps({"k": k.tolist(), "v": v.tolist()}).encode())
        with urllib.request.urlopen(req, timeout=60) as r:
            js = _json.loads(r.read())
        kc_json = np.array(js["k_codes"], dtype=np.int16)
        assert js["n_groups"] == 22 and js["head_dim"] == 64
        _codes_match(f, _pad(k, 66), kc_json, f["k_codes"])
        req = urllib.request.Request(url + "/compress", method="POST", data=k.tobytes() + v.tobytes(),
                                     headers={"Content-Type": sidecar.BINARY, "X-PrismKV-Shape": f"{k.shape[0]},64"})
        with urllib.request.urlopen(req, timeout=60) as r:
            raw = r.read()
            assert r.headers["X-PrismKV-Shape"] == f"{k.shape[0]},22"
        codes = np.frombuffer(raw, dtype=np.int16).reshape(2, k.shape[0], 22)
        np.testing.assert_array_equal(codes[0], kc_json)
        np.testing.assert_array_equal(codes[1], np.array(js["v_codes"], dtype=np.int16))
        req = urllib.request.Request(url + "/decompress", method="POST", data=raw,
                                     headers={"Content-Type": sidecar.BINARY, "X-PrismKV-Shape": f"{k.shape[0]},22",
                                              "X-PrismKV-Head-Dim": "64"})
        with urllib.request.urlopen(req, timeout=60) as r:
            dec = np.frombuffer(r.read(), dtype=np.float32).reshape(2, k.shape[0], 64)
        req = urllib.request.Request(url + "/decompress", method="POST", headers={"Content-Type": "application/json"},
                                     data=_json.dumps({"k_codes": js["k_codes"], "v_codes": js["v_codes"],
                                                       "head_dim": 64}).encode())
        with urllib.request.urlopen(req, timeout=60) as r:
            jd = _json.loads(r.read())
        np.testing.assert_array_equal(dec[0], np.array(jd["k"], dtype=np.float32))
        np.testing.assert_array_equal(dec[1], np.array(jd["v"], dtype=np.float32))
    finally:
        srv.stop()
