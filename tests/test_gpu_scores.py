"""GPU parity of pkv_polar_scores behind prismkv_b200.cuda.polar_attn_fwd.

Mirrors the reference's tests/test_cuda_kernel.py contract (:116-221):
scores equal PolarAttentionApprox.attention_scores * scale to 1e-4, scale is
linear, 3+3+2 bit budgets are accepted, batches are independent.
"""

import math

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden
from prismkv_b200 import PolarAttentionApprox, StackedPlaneQuantizer
from prismkv_b200.cuda import CUDA_AVAILABLE, polar_attn_fwd

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("name", ["scores_d66", "scores_d96_332"])
def test_scores_match_reference_golden(cuda_ready, name):
    f = load_golden(name)
    pr, b = f["params"], [int(x) for x in f["bits"]]
    s = polar_attn_fwd(torch.from_numpy(f["Q_rot"]).to(DEV), torch.from_numpy(f["k_codes"]).to(DEV),
                       float(pr[0]), float(pr[1]), float(pr[2]), float(pr[3]), float(pr[4]), float(pr[5]), *b)
    np.testing.assert_allclose(s.cpu().numpy(), f["scores"], atol=1e-4, rtol=1e-4)


def _args(d=66, bits=4, B=1, H=2, Sq=4, Sk=6, seed=0):
    qz = StackedPlaneQuantizer(dim=d, bits_z=bits, bits_r=bits, bits_theta=bits, seed=0)
    g = torch.Generator().manual_seed(seed)
    Q = torch.randn(B, H, Sq, d, generator=g)
    K = torch.randn(B, H, Sk, d, generator=g)
    kc = qz.encode(K.reshape(-1, d).to(DEV)).reshape(B, H, Sk, -1).to(torch.int16)
    Cz = 1 << bits
    kw = dict(z_min=qz.z_min, delta_z=(qz.z_max - qz.z_min) / Cz, r_max=qz.r_max,
              delta_r=qz.r_max / (Cz - 1), delta_theta=2 * math.pi / (Cz - 1), scale=1 / math.sqrt(d),
              bits_z=bits, bits_r=bits, bits_theta=bits)
    return Q, kc, kw, qz


def test_cuda_available(cuda_ready):
    assert CUDA_AVAILABLE is True


def test_scores_match_polar_attention_approx(cuda_ready):
    Q, kc, kw, qz = _args(B=2, H=4, Sq=8, Sk=100)
    Qr = (Q.reshape(-1, 66) @ qz.R.T).reshape(Q.shape).to(DEV)
    s = polar_attn_fwd(Qr, kc, **kw)
    approx = PolarAttentionApprox(4, 4, 4, qz.z_min, qz.z_max, qz.r_max, scale=kw["scale"], R=qz.R)
    ref = approx.attention_scores(Q.to(DEV), kc) * kw["scale"]
    torch.testing.assert_close(s, ref, atol=1e-4, rtol=1e-4)
    p = oracle.QuantParams(dim=66, z_min=qz.z_min, z_max=qz.z_max, r_max=qz.r_max)
    o = oracle.polar_scores(Qr.cpu().numpy(), kc.cpu().numpy().astype(np.int64), qz.z_min, kw["delta_z"],
                            qz.r_max, kw["scale"], 4, 4, 4)
    np.testing.assert_allclose(s.cpu().numpy(), o, atol=1e-4)
    del p


def test_scale_linear_and_cpu_io(cuda_ready):
    Q, kc, kw, _ = _args(seed=1)
    s1 = polar_attn_fwd(Q, kc.cpu(), **{**kw, "scale": 1.0})
    s2 = polar_attn_fwd(Q, kc.cpu(), **{**kw, "scale": 2.0})
    assert s1.device.type == "cpu" and s1.dtype == torch.float32 and s1.shape == (1, 2, 4, 6)
    torch.testing.assert_close(s2, 2.0 * s1, atol=1e-5, rtol=1e-5)


def test_332_bits_and_uint8_codes(cuda_ready):
    Q, kc, kw, qz = _args(d=96, bits=4, Sk=77)
    qz = StackedPlaneQuantizer(dim=96, bits_z=3, bits_r=3, bits_theta=2, seed=0)
    K = torch.randn(1, 2, 77, 96)
    kc8 = qz.encode_compact(K.reshape(-1, 96).to(DEV)).reshape(1, 2, 77, 32)
    kw = dict(z_min=qz.z_min, delta_z=(qz.z_max - qz.z_min) / 8, r_max=qz.r_max, delta_r=qz.r_max / 7,
              delta_theta=2 * math.pi / 3, scale=0.1, bits_z=3, bits_r=3, bits_theta=2)
    Q = torch.randn(1, 2, 4, 96).to(DEV)
    a = polar_attn_fwd(Q, kc8, **kw)
    b = polar_attn_fwd(Q, kc8.to(torch.int16), **kw)
    torch.testing.assert_close(a, b)
    o = oracle.polar_scores(Q.cpu().numpy(), kc8.cpu().numpy().astype(np.int64), kw["z_min"], kw["delta_z"],
                            kw["r_max"], 0.1, 3, 3, 2)
    np.testing.assert_allclose(a.cpu().numpy(), o, atol=1e-4)


def test_batch_independence(cuda_ready):
    Q, kc, kw, _ = _args(B=3, H=2, Sq=5, Sk=130, seed=4)
    full = polar_attn_fwd(Q.to(DEV), kc, **kw)
    for b in range(3):
        one = polar_attn_fwd(Q[b:b + 1].to(DEV), kc[b:b + 1], **kw)
        torch.testing.assert_close(one[0], full[b])


def test_shape_errors(cuda_ready):
    Q, kc, kw, _ = _args()
    with pytest.raises(RuntimeError):
        polar_attn_fwd(Q[..., :63].to(DEV), kc, **kw)
    with pytest.raises(RuntimeError):
        polar_attn_fwd(Q.to(DEV), kc[:, :1], **kw)
