"""Host parts of prismkv_b200.cache (no GPU): config, padding, and the cache
golden fixtures pinned against the oracle."""

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden, params_from
from prismkv_b200.cache import DimAligner, PrismKVConfig


def test_config_matches_reference_formulas():
    c = PrismKVConfig()
    assert (c.bits_z, c.bits_r, c.bits_theta, c.rotation_seed, c.codebook_path) == (4, 4, 4, 42, None)
    assert c.bits_per_dim == 4.0 and c.compression_vs_fp16 == 4.0
    c2 = PrismKVConfig(3, 3, 2)
    assert c2.bits_per_dim == pytest.approx(8 / 3) and "2.67 bits/dim" in repr(c2)


@pytest.mark.parametrize("d,padded", [(64, 66), (96, 96), (128, 129), (65, 66)])
def test_dim_aligner(d, padded):
    a = DimAligner(d)
    x = torch.randn(5, d)
    y = a.pad(x)
    assert y.shape == (5, padded) and torch.equal(y[:, :d], x) and (y[:, d:] == 0).all()
    assert torch.equal(a.unpad(y), x)


def test_cache_fixtures_against_oracle():
    """The reference's cache outputs equal the oracle's encode/decode of the padded rows."""
    f = load_golden("raw_cache_d64")
    p = params_from(f)
    X = np.concatenate([f["k1"].reshape(-1, 64), f["k2"].reshape(-1, 64)])
    X = np.concatenate([X, np.zeros((X.shape[0], 2), np.float32)], axis=1)
    codes = oracle.encode(X, f["R"], p)
    rep = oracle.classify(X, f["R"], p, codes, f["k_codes"].astype(np.int64))
    assert rep.unexplained == 0
    dec = oracle.decode(f["k_codes"].astype(np.int64), f["R"], p)[:, :64]
    np.testing.assert_allclose(dec, f["k_full"].reshape(-1, 64), atol=1e-5)
    g = load_golden("vllm_block_d64")
    dec = oracle.decode(g["k_codes"].astype(np.int64), g["R"], params_from(g))[:, :64]
    np.testing.assert_allclose(dec.reshape(2, 16, 64), g["k_dec"].astype(np.float32), atol=2e-3, rtol=1e-3)
