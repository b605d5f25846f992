"""Host side of the multi-GPU decode (prismkv_b200.dist), on CPU with gloo.

The exchange step of split-sequence decode is tested with two gloo ranks: each
rank computes fp64 softmax partials of its token shard with the oracle,
``gather_partials`` exchanges them, and the log-sum-exp merge of the gathered
partials must equal the oracle's attention over the whole sequence.  The CUDA
side of the same step (partial kernel + pkv_lse_combine) is covered by the
GPU tests.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from prismkv_b200.dist import gather_partials, shard_range


@pytest.mark.parametrize("n,world", [(0, 1), (1, 2), (7, 2), (131072, 8), (5, 8), (100, 3)])
def test_shard_range_covers_contiguously(n, world):
    bounds = [shard_range(n, world, r) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == n
    for (a, b), (c, _) in zip(bounds, bounds[1:]):
        assert b == c
    sizes = [b - a for a, b in bounds]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _problem():
    rng = np.random.default_rng(3)
    p = oracle.QuantParams.default(96)
    R = np.linalg.qr(rng.standard_normal((96, 96)))[0].astype(np.float32)
    B, H, S = 2, 4, 301
    kc = oracle.encode(rng.standard_normal((B * H * S, 96)).astype(np.float32), R, p).reshape(B, H, S, 32)
    vc = oracle.encode(rng.standard_normal((B * H * S, 96)).astype(np.float32), R, p).reshape(B, H, S, 32)
    q = rng.standard_normal((B, H, 96)).astype(np.float32)
    return p, R, q, kc, vc


def _partials(q, kc, vc, R, p):
    """(B*H, 98) fp64 [m, l, o_rot] of one token shard (natural-log max)."""
    B, H, S, m = kc.shape
    out = np.zeros((B * H, 98))
    out[:, 0] = -np.inf
    if S == 0:
        return out
    qr = q.astype(np.float64) @ R.astype(np.float64).T
    kr = oracle.dequant_rotated(kc.reshape(-1, m), p).reshape(B, H, S, 96).astype(np.float64)
    vr = oracle.dequant_rotated(vc.reshape(-1, m), p).reshape(B, H, S, 96).astype(np.float64)
    s = np.einsum("bhd,bhsd->bhs", qr, kr) * 96 ** -0.5
    mx = s.max(-1)
    w = np.exp(s - mx[..., None])
    out[:, 0] = mx.reshape(-1)
    out[:, 1] = w.sum(-1).reshape(-1)
    out[:, 2:] = np.einsum("bhs,bhsd->bhd", w, vr).reshape(B * H, 96)
    return out


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p, R, q, kc, vc = _problem()
        a, b = shard_range(kc.shape[2], world, rank)
        mine = torch.from_numpy(_partials(q, kc[:, :, a:b], vc[:, :, a:b], R, p))
        allp = gather_partials(mine).numpy()
        assert allp.shape == (world, 8, 98)
        merged = oracle.lse_combine(allp[:, :, 0], allp[:, :, 1], allp[:, :, 2:]) @ R.astype(np.float64)
        ref = oracle.attention(q, kc, vc, R, p).reshape(8, 96)
        results.put((rank, float(np.abs(merged - ref).max())))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_split_sequence_exchange_gloo(world):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=180)
    for pr in procs:
        if pr.is_alive():
            pr.kill()
    assert all(pr.exitcode == 0 for pr in procs), [pr.exitcode for pr in procs]
    errs = dict(results.get(timeout=5) for _ in range(world))
    assert max(errs.values()) < 1e-9, errs


# ---------------------------------------------------------------------------
# failures on the host side of the exchange: made on the host, never on a GPU
# ---------------------------------------------------------------------------

def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(target, world, timeout=120, **kw):
    port = _port()
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, port, results), kwargs=kw) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=timeout)
    for pr in procs:
        if pr.is_alive():
            pr.kill()
    out = {}
    while not results.empty():
        k, v = results.get(timeout=5)
        out[k] = v
    return [pr.exitcode for pr in procs], out


def _leaver(rank, world, port, results):
    """Step 1 with every rank; then the last rank leaves (between steps, nothing in flight).
    The others' step-2 exchange must end with an error within the group's short timeout."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=5))
    p, R, q, kc, vc = _problem()
    a, b = shard_range(kc.shape[2], world, rank)
    mine = torch.from_numpy(_partials(q, kc[:, :, a:b], vc[:, :, a:b], R, p))
    gather_partials(mine)                                 # step 1: everyone
    if rank == world - 1:
        results.put((rank, "left"))
        results.close()
        results.join_thread()                             # the message is out before the process is
        os._exit(0)                                       # leaves without a goodbye
    t0 = time.monotonic()
    try:
        gather_partials(mine)                             # step 2: a rank is missing
        results.put((rank, "no error"))
    except Exception as e:                                # noqa: BLE001 -- any transport error counts
        results.put((rank, ("error", time.monotonic() - t0, type(e).__name__)))
    results.close()
    results.join_thread()
    os._exit(0)


def test_rank_leaving_between_steps_is_detected():
    codes, res = _run(_leaver, 3, timeout=90)
    assert res.get(2) == "left"
    for r in (0, 1):
        assert isinstance(res.get(r), tuple) and res[r][0] == "error", res
        assert res[r][1] < 60, res                        # ended by the group timeout, not hung


def _late(rank, world, port, results, delay=2.0):
    """Rank 1 contributes its shard late; the merged result is still exact."""
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p, R, q, kc, vc = _problem()
        a, b = shard_range(kc.shape[2], world, rank)
        mine = torch.from_numpy(_partials(q, kc[:, :, a:b], vc[:, :, a:b], R, p))
        if rank == 1:
            time.sleep(delay)
        allp = gather_partials(mine).numpy()
        merged = oracle.lse_combine(allp[:, :, 0], allp[:, :, 1], allp[:, :, 2:]) @ R.astype(np.float64)
        ref = oracle.attention(q, kc, vc, R, p).reshape(8, 96)
        results.put((rank, float(np.abs(merged - ref).max())))
    finally:
        torch.distributed.destroy_process_group()


def test_late_rank_still_merges_exactly():
    codes, res = _run(_late, 3)
    assert codes == [0, 0, 0], codes
    assert max(res.values()) < 1e-9, res


def _odd_partials(rank, world, port, results):
    """Rank 1's shard is empty (m = -inf, l = 0, o = 0) and rank 2 sends one NaN m row: every rank
    receives both exactly as sent, the empty shard drops out of the merge, and every row but the
    NaN one merges exactly.  (What the device merge makes of a NaN row -- NaN, as a NaN score
    makes the unsplit softmax -- is a GPU test of pkv_lse_combine.)"""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p, R, q, kc, vc = _problem()
        S = kc.shape[2]
        bounds = [(0, 150), (150, 150), (150, S)]
        a, b = bounds[rank]
        mine = _partials(q, kc[:, :, a:b], vc[:, :, a:b], R, p)
        if rank == 2:
            mine[3, 0] = np.nan
        allp = gather_partials(torch.from_numpy(mine)).numpy()
        assert np.isinf(allp[1, :, 0]).all() and (allp[1, :, 1:] == 0).all()
        delivered = bool(np.isnan(allp[2, 3, 0])) and int(np.isnan(allp).sum()) == 1
        merged = oracle.lse_combine(allp[:, :, 0], allp[:, :, 1], allp[:, :, 2:]) @ R.astype(np.float64)
        ref = oracle.attention(q, kc, vc, R, p).reshape(8, 96)
        good = [i for i in range(8) if i != 3]
        results.put((rank, (float(np.abs(merged[good] - ref[good]).max()), delivered)))
    finally:
        torch.distributed.destroy_process_group()


def test_empty_and_nan_partials():
    codes, res = _run(_odd_partials, 3)
    assert codes == [0, 0, 0], codes
    for r, (err, delivered) in res.items():
        assert err < 1e-9 and delivered, (r, err, delivered)
