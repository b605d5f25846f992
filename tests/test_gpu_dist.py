"""Split-sequence (NCCL all-gather, and the in-kernel exchange over CUDA-IPC peer memory) and
batch-sharded decode on 2 GPUs, against the oracle.

Runs only where at least two GPUs are visible; the exchange logic itself is
also covered on CPU with gloo (test_dist_cpu.py).  NVLS is off in these child
processes (NCCL_NVLS_ENABLE=0), as for every multi-rank test here.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        import oracle
        from prismkv_b200 import StackedPlaneQuantizer
        from prismkv_b200.dist import SequenceExchange, batch_shard_decode, shard_range, split_sequence_decode
        err_seq = err_batch = 0.0
        # shards on the grouped 12-bit kernel, the two-pass and one-pass one-head 12-bit kernels
        # (MHA shards below and past 4096 tokens) and the one-byte kernel
        for bits, S, Hq, Hkv in (((4, 4, 4), 3001, 16, 4), ((4, 4, 4), 5001, 8, 8), ((4, 4, 4), 9001, 8, 8),
                                 ((3, 3, 2), 5001, 16, 4)):
            q = StackedPlaneQuantizer(96, *bits, seed=42)
            B = 2
            g = torch.Generator().manual_seed(9)
            k = torch.randn(B * Hkv * S, 96, generator=g)
            v = torch.randn(B * Hkv * S, 96, generator=g)
            kc = q.encode_compact(k.to(dev)).view(B, Hkv, S, 32)
            vc = q.encode_compact(v.to(dev)).view(B, Hkv, S, 32)
            qv = torch.randn(B, Hq, 96, generator=g).to(dev)
            a, b = shard_range(S, world, rank)
            out = split_sequence_decode(q, qv, kc[:, :, a:b].contiguous(), vc[:, :, a:b].contiguous())
            p = oracle.QuantParams.default(96, *bits)
            ref = oracle.attention(qv.cpu().numpy(), kc.cpu().numpy().astype(np.int64),
                                   vc.cpu().numpy().astype(np.int64), q.R.numpy(), p)
            err_seq = max(err_seq, float(np.abs(out.cpu().numpy() - ref).max()))
            ks, vs = kc[:, :, a:b].contiguous(), vc[:, :, a:b].contiguous()
            ex = SequenceExchange(q, qv, ks, wait_ms=5000)
            for _ in range(3):                       # the counters reset themselves between steps
                outp = split_sequence_decode(q, qv, ks, vs, exchange=ex)
                ex.check()
                err_seq = max(err_seq, float(np.abs(outp.cpu().numpy() - ref).max()))
            ex.close()
            ba, bb = shard_range(B, world, rank)
            outb = batch_shard_decode(q, qv[ba:bb].contiguous(), kc[ba:bb].contiguous(), vc[ba:bb].contiguous())
            err_batch = max(err_batch, float(np.abs(outb.cpu().numpy() - ref[ba:bb]).max()))
        torch.cuda.synchronize()
        torch.distributed.barrier()                  # no rank frees a buffer a peer still reads
        torch.cuda.synchronize()
        results.put((rank, err_seq, err_batch))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_split_sequence_and_batch_shards_two_gpus(cuda_ready):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=240)
    for pr in procs:
        if pr.is_alive():
            pr.kill()
    assert all(pr.exitcode == 0 for pr in procs), [pr.exitcode for pr in procs]
    for _ in range(2):
        rank, e_seq, e_batch = results.get(timeout=5)
        assert e_seq < 1e-3 and e_batch < 1e-3, (rank, e_seq, e_batch)
