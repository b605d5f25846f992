"""GPU parity of the tensor-core decode-attention kernel (attn_tc_kernel).

It serves bf16 / fp16 queries of head_dim 96 for grouped heads (up to 16 per KV
head) and per-z-bin tables (learned codebooks, BiasTable), with any codec the
one-head 12-bit kernel does not take (Lloyd-Max z, 8-bit codes, learned).  Operands are bf16 (or fp16)
on the tensor cores with fp32 accumulation, so the bound is the stated one for
bf16 queries, 2e-2 max abs against the oracle's fp64 attention; the observed
error is also kept below 1e-2 so that a drift is noticed well before the bound.
"""

import numpy as np
import pytest
import torch

import oracle
from prismkv_b200 import decode_attention
from test_gpu_attention import _codes, _setup

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-2
WARN = 1e-2

CASES = [
    # B, Hq, Hkv, S, variant, bits, qdtype, splits
    (2, 32, 8, 1000, "learned_bias", (4, 4, 4), torch.bfloat16, 0),
    (1, 32, 8, 5000, "learned_bias", (4, 4, 4), torch.bfloat16, 0),
    (2, 8, 4, 513, "v1", (3, 3, 2), torch.bfloat16, 0),            # 8-bit uniform codes, group of 2
    (2, 8, 8, 513, "learned", (3, 3, 2), torch.float16, 0),         # 8-bit learned, MHA
    (1, 8, 4, 700, "lloyd", (4, 4, 4), torch.bfloat16, 0),
    (1, 16, 1, 300, "learned", (4, 4, 4), torch.bfloat16, 0),        # group of 16
    (1, 6, 2, 129, "learned_bias", (4, 4, 4), torch.float16, 0),      # group of 3
    (2, 8, 4, 2000, "learned_bias", (4, 4, 4), torch.bfloat16, 3),   # forced splits
    (1, 8, 2, 1, "learned", (4, 4, 4), torch.bfloat16, 0),           # one token
]


@pytest.mark.parametrize("B,Hq,Hkv,S,variant,bits,qdt,splits", CASES)
def test_tc_attention_matches_oracle(cuda_ready, B, Hq, Hkv, S, variant, bits, qdt, splits):
    q, p = _setup(variant, bits)
    kc, vc = _codes(q, B, Hkv, S, seed=S + 3 * Hq)
    qv = torch.randn(B, Hq, 96, generator=torch.Generator(device=DEV).manual_seed(11), device=DEV).to(qdt)
    plan = q.codec(torch.device(DEV)).describe(qv, kc, vc, num_splits=splits)
    assert plan["kernel"] == "attn_tc_kernel"
    out = decode_attention(q, qv, kc, vc, num_splits=splits)
    ref = oracle.attention(qv.float().cpu().numpy(), kc.cpu().numpy().astype(np.int64),
                           vc.cpu().numpy().astype(np.int64), q.R.numpy(), p)
    err = np.abs(out.cpu().numpy() - ref).max()
    assert err < WARN, err
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL, rtol=0)
    from prismkv_b200 import _lib
    assert _lib.device_error() == 0


def test_tc_attention_ragged_rows_and_partials(cuda_ready):
    """seq_lens with an empty row, and the partial (split-sequence) output merged with
    pkv_lse_combine, on the tensor-core kernel."""
    q, p = _setup("learned_bias", (4, 4, 4))
    B, Hq, Hkv, S = 3, 16, 4, 900
    kc, vc = _codes(q, B, Hkv, S, seed=77)
    qv = torch.randn(B, Hq, 96, generator=torch.Generator(device=DEV).manual_seed(5), device=DEV).to(torch.bfloat16)
    lens = torch.tensor([900, 0, 131], dtype=torch.int32, device=DEV)
    out = decode_attention(q, qv, kc, vc, seq_lens=lens)
    ref = oracle.attention(qv.float().cpu().numpy(), kc.cpu().numpy().astype(np.int64),
                           vc.cpu().numpy().astype(np.int64), q.R.numpy(), p, seq_lens=lens.cpu().numpy())
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=TOL, rtol=0)
    assert (out[1] == 0).all()
    codec = q.codec(torch.device(DEV))
    parts = [codec.attention(qv, kc[:, :, a:b], vc[:, :, a:b], partial=True).view(B * Hq, 98)
             for a, b in ((0, 400), (400, 900))]
    merged = codec.combine(torch.stack(parts)).view(B, Hq, 96)
    ref_full = oracle.attention(qv.float().cpu().numpy(), kc.cpu().numpy().astype(np.int64),
                                vc.cpu().numpy().astype(np.int64), q.R.numpy(), p)
    np.testing.assert_allclose(merged.cpu().numpy(), ref_full, atol=TOL, rtol=0)
