"""Pin the CPU oracle to golden vectors produced by the reference itself.

The fixtures under tests/golden were written by tests/golden/gen_golden.py
running PrismKV v1.4.1's own API (StackedPlaneQuantizer.encode/decode,
PrismKVBackend, PolarAttentionApprox.forward, prismkv.cuda.polar_attn_fwd's
torch path).  Code mismatches are allowed only where the tie classifier
proves a rounding tie; float outputs must agree to fp32 rounding.
"""

import numpy as np
import pytest

import oracle
from conftest import golden_files, load_golden, params_from

ENC = [f for f in golden_files("enc_")]


@pytest.mark.parametrize("path", ENC, ids=lambda p: p.split("/")[-1])
def test_encode_matches_reference(path):
    f = load_golden(path)
    p = params_from(f)
    codes = oracle.encode(f["X"], f["R"], p)
    ref = f["codes"].astype(np.int64) & ((1 << (p.bits_z + p.bits_r + p.bits_theta)) - 1)
    rep = oracle.classify(f["X"], f["R"], p, codes, ref)
    assert rep.unexplained == 0, rep.examples
    assert rep.mismatches <= max(2, rep.total // 10000)


@pytest.mark.parametrize("path", ENC, ids=lambda p: p.split("/")[-1])
def test_decode_matches_reference(path):
    f = load_golden(path)
    p = params_from(f)
    dec = oracle.decode(f["codes"][: f["decoded"].shape[0]].astype(np.int64), f["R"], p)
    np.testing.assert_allclose(dec, f["decoded"], atol=2e-5, rtol=0)
    dall = oracle.decode(f["all_codes"].astype(np.int64), f["R"], p)
    np.testing.assert_allclose(dall, f["decoded_all"], atol=2e-5, rtol=0)


def test_backend_d64_padding():
    f = load_golden("backend_d64")
    p = params_from(f)
    k = np.pad(f["k"], ((0, 0), (0, 2)))                 # DimAligner zero-pads 64 -> 66
    codes = oracle.encode(k, f["R"], p)
    rep = oracle.classify(k, f["R"], p, codes, f["k_codes"].astype(np.int64))
    assert rep.unexplained == 0
    dec = oracle.decode(f["k_codes"].astype(np.int64), f["R"], p)[:, :64]
    np.testing.assert_allclose(dec, f["k_dec"], atol=2e-5)


def test_attention_v1_matches_polar_attention_approx():
    f = load_golden("attn_v1")
    p = params_from(f)
    out = oracle.attention(f["q"], f["k_codes"].astype(np.int64), f["v_codes"].astype(np.int64), f["R"], p)
    np.testing.assert_allclose(out, f["out"][:, :, 0], atol=1e-5)
    B, H, S, m = f["k_codes"].shape
    v = oracle.decode(f["v_codes"].reshape(-1, m).astype(np.int64), f["R"], p).reshape(B, H, S, 3 * m)
    o32, w = oracle.polar_attention_forward_f32(f["q"], f["k_codes"], v, f["R"], p)
    np.testing.assert_allclose(o32, f["out"], atol=1e-5)
    np.testing.assert_allclose(w, f["weights"], atol=1e-6)


def test_attention_learned_gqa_matches_composite():
    f = load_golden("attn_v2_gqa")
    p = params_from(f)
    out = oracle.attention(f["q"], f["k_codes"].astype(np.int64), f["v_codes"].astype(np.int64), f["R"], p)
    np.testing.assert_allclose(out, f["out"][:, :, 0], atol=1e-5)


@pytest.mark.parametrize("name", ["scores_d66", "scores_d96_332"])
def test_polar_scores_match_polar_attn_fwd(name):
    f = load_golden(name)
    pr, b = f["params"], [int(x) for x in f["bits"]]
    s = oracle.polar_scores(f["Q_rot"], f["k_codes"].astype(np.int64), pr[0], pr[1], pr[2], pr[5], *b)
    np.testing.assert_allclose(s, f["scores"], atol=1e-5)


def test_packing_known_answer():
    # tests/test_quantizer.py:146-162 of the reference: (i_z, i_r, i_theta) = (3, 7, 11)
    code = (3 << 8) | (7 << 4) | 11
    p = oracle.QuantParams.default(96)
    rot = oracle.dequant_rotated(np.full((1, 32), code), p)
    assert rot[0, 0] == np.float32(np.float32(-np.sqrt(96.0)) + np.float32(3.5 * (2 * np.sqrt(96.0) / 16)))


def test_tie_classifier_flags_planted_error():
    rng = np.random.default_rng(1)
    f = load_golden("enc_v1_444")
    p = params_from(f)
    X = rng.standard_normal((20000, 96)).astype(np.float32)
    rot = (X.astype(np.float64) @ f["R"].astype(np.float64).T).astype(np.float32)
    good = oracle.encode_rotated(rot, p)
    assert oracle.classify(X, f["R"], p, oracle.encode(X, f["R"], p), good).unexplained == 0
    bad = rot.copy()
    bad[:, 0::3] += np.float32(2e-3)                      # a planted bias far above rounding
    rep = oracle.classify(X, f["R"], p, good, oracle.encode_rotated(bad, p))
    assert rep.unexplained > 100


def test_lse_combine_equals_unsplit():
    rng = np.random.default_rng(2)
    s = rng.standard_normal(300) * 3
    v = rng.standard_normal((300, 8))
    full = (np.exp(s - s.max()) @ v) / np.exp(s - s.max()).sum()
    parts = [slice(0, 100), slice(100, 100), slice(100, 300)]
    ms, ls, os = [], [], []
    for sl in parts:
        ss = s[sl]
        if ss.size == 0:
            ms.append(-np.inf); ls.append(0.0); os.append(np.zeros(8)); continue
        mm = ss.max()
        ms.append(mm); ls.append(np.exp(ss - mm).sum()); os.append(np.exp(ss - mm) @ v[sl])
    np.testing.assert_allclose(oracle.lse_combine(np.array(ms), np.array(ls), np.array(os)), full, atol=1e-12)
