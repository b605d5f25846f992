"""The in-kernel split-sequence exchange (pkv_attn_decode_xr) on one GPU.

With one rank the whole protocol runs -- partial rows stored into the exchange buffer as
flagged words, every CTA's share of the units merged once their flags are in, R, the output
rows, the call count advanced -- and must give the unsplit kernel's output, call after call (the
flags of one call never match the next's).  With two ranks in one process nothing plays the
second rank: its partials never arrive, so the merge's wait must run out after its short bound,
set the device error word (4) and return; after pkv_xr_reset the exchange works again.  No
second kernel is involved in either case: the wait that runs out waits on words nothing writes.
"""

import numpy as np
import pytest
import torch

import oracle
from prismkv_b200 import BiasTable, LearnedSliceCodebook, StackedPlaneQuantizer, _lib
from prismkv_b200.dist import SequenceExchange
from prismkv_b200.synthetic import synthetic_bias, synthetic_codebook

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _quantizer(bits, variant):
    q = StackedPlaneQuantizer(96, *bits, seed=42)
    Cz, K = 1 << bits[0], 1 << (bits[1] + bits[2])
    if "learned" in variant:
        q._codebooks = LearnedSliceCodebook(synthetic_codebook(Cz, K, q.r_max, 11), Cz, K, q.z_min, q.z_max, q.r_max)
    if "bias" in variant:
        q._bias = BiasTable(synthetic_bias(Cz, 12), delta_z=(q.z_max - q.z_min) / Cz)
    return q


def _data(q, B, Hq, Hkv, S, qdt, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    kc = q.encode_compact(torch.randn(B * Hkv * S, 96, generator=g, device=DEV)).view(B, Hkv, S, 32)
    vc = q.encode_compact(torch.randn(B * Hkv * S, 96, generator=g, device=DEV)).view(B, Hkv, S, 32)
    qv = torch.randn(B, Hq, 96, generator=g, device=DEV).to(qdt)
    return qv, kc, vc


@pytest.mark.parametrize("B,Hq,Hkv,S,bits,variant,qdt,kernel", [
    (2, 16, 4, 3000, (4, 4, 4), "v1", torch.bfloat16, "attn_gqa12_mma_kernel"),
    (1, 32, 8, 20000, (4, 4, 4), "v1", torch.float32, "attn_gqa12_mma_kernel"),   # balanced segments
    (1, 32, 8, 20000, (4, 4, 4), "fp32", torch.float32, "attn_gqa12_kernel"),
    (2, 8, 8, 3000, (4, 4, 4), "v1", torch.float32, "attn_mha12_kernel"),
    (2, 8, 8, 6000, (4, 4, 4), "v1", torch.bfloat16, "attn_mha12_stream_kernel"),
    (2, 8, 8, 3000, (3, 3, 2), "v1", torch.float32, "attn_mha8_kernel"),
    (2, 16, 4, 2000, (4, 4, 4), "learned_bias", torch.bfloat16, "attn_tc_kernel"),
    (1, 8, 4, 1500, (4, 4, 4), "learned_bias", torch.float32, "attn_lut_kernel"),
    (2, 8, 8, 0, (4, 4, 4), "v1", torch.float32, None),                           # an empty shard
])
def test_one_rank_exchange_matches_unsplit(cuda_ready, B, Hq, Hkv, S, bits, variant, qdt, kernel):
    q = _quantizer(bits, variant)
    qv, kc, vc = _data(q, B, Hq, Hkv, S, qdt, seed=S + Hq)
    codec = q.codec(torch.device(DEV))
    codec.fp32_attention = variant == "fp32"                 # this test's own quantizer: no restore
    if kernel is not None:
        assert codec.describe(qv, kc, vc)["kernel"] == kernel
    ref = codec.attention(qv, kc, vc)
    ex = SequenceExchange.single_process(q, qv, kc, world=1, wait_ms=2000)
    try:
        for _ in range(3):                                  # the counters reset themselves
            out = ex.run(qv, kc, vc).clone()
            torch.cuda.synchronize()
            ex.check()
            np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), atol=1e-5, rtol=0)
    finally:
        ex.close()


def test_one_rank_exchange_matches_oracle(cuda_ready):
    q = _quantizer((4, 4, 4), "v1")
    qv, kc, vc = _data(q, 1, 8, 2, 2500, torch.float32, seed=3)
    ex = SequenceExchange.single_process(q, qv, kc, world=1)
    try:
        out = ex.run(qv, kc, vc).clone()
        ex.check()
    finally:
        ex.close()
    ref = oracle.attention(qv.cpu().numpy(), kc.cpu().numpy().astype(np.int64), vc.cpu().numpy().astype(np.int64),
                           q.R.numpy(), oracle.QuantParams.default(96))
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=1e-3, rtol=0)


def test_completion_wait_runs_out_and_reset_recovers(cuda_ready):
    """Two ranks, one of them absent: the wait expires after ~20 ms of device time, the device
    error word reads 4, the GPU stays usable; reset, and a one-rank exchange then succeeds."""
    q = _quantizer((4, 4, 4), "v1")
    qv, kc, vc = _data(q, 2, 16, 4, 3000, torch.bfloat16, seed=7)
    assert _lib.device_error() == 0
    ex2 = SequenceExchange.single_process(q, qv, kc, world=2, wait_ms=20)
    try:
        ex2.run(qv, kc, vc)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="device error 4"):
            ex2.check()
        assert _lib.device_error() == 0                     # check() cleared it
        ex2.reset(qv, kc)
        torch.cuda.synchronize()
    finally:
        ex2.close()
    ex1 = SequenceExchange.single_process(q, qv, kc, world=1)
    try:
        out = ex1.run(qv, kc, vc).clone()
        ex1.check()
    finally:
        ex1.close()
    ref = q.codec(torch.device(DEV)).attention(qv, kc, vc)
    np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), atol=1e-5, rtol=0)


def test_exchange_rejects_mismatched_calls(cuda_ready):
    q = _quantizer((4, 4, 4), "v1")
    qv, kc, vc = _data(q, 2, 16, 4, 500, torch.float32, seed=1)
    ex = SequenceExchange.single_process(q, qv, kc, world=1)
    try:
        with pytest.raises(ValueError):
            ex.run(qv[:1], kc[:1], vc[:1])
    finally:
        ex.close()
