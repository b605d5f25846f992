"""Benchmark of the PrismKV B200 hot path: decode attention over packed KV codes.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl prismkv|reference]
                    [--workload phi3-decode|aggressive-332|learned-gqa|longctx-splitseq|cpu-roundtrip]
                    [--mode decode|encode]

One step = one fused dequant + flash-decoding attention over the whole
workload's packed K/V (inputs resident in HBM, larger than L2, L2 scrubbed
between steps).  The metric is effective HBM bandwidth: algorithmic bytes
(packed codes read once + query + fp32 output) / device time.  Under
torchrun with N > 1 every rank runs its own replica of the workload (no
data-path collective; weak scaling).  ``--mode encode`` times the fused
rotate + bin + pack kernel on the learned-gqa encode workload (Mtok/s).

``--impl reference`` times the reference algorithm's CPU path (the oracle's
NumPy restatement of PolarAttentionApprox.forward + decode) on the host
cores, one bounded slice of the workload per step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "decode attn over packed KV: effective HBM GB/s & % of peak; encode Mtok/s; 1-8 GPU"
FALLBACK_HBM_GBS = 6650.0


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def _committed_traffic(kernel: str, workload: str):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d.get(kernel, {}).get(workload)
    except (OSError, ValueError):
        return None


class L2Scrub:
    """Evicts the previous step's data from the 126 MB L2 between timed steps.

    Reads a 256 MB buffer (a sum): the lines it leaves in L2 are clean, so the
    next timed kernel pays no write-back of scrub data.  A write-based scrub
    (memset) leaves ~126 MB of dirty lines whose eviction competes with the
    kernel's own reads.
    """

    DESCRIPTION = "L2 scrubbed between steps by reading a 256 MB buffer (inputs also > L2)"

    def __init__(self, device):
        self.buf = torch.ones(64 << 20, dtype=torch.float32, device=device)

    def __call__(self):
        self.buf.sum()


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML on a background thread."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle"}

    def __init__(self, index: int, period: float = 0.01):
        self.index, self.period = index, period
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:                       # no NVML: the line carries nulls
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


def _dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _barrier(ws):
    if ws > 1:
        torch.distributed.barrier()


def _max_over_ranks(x: float, ws: int, device) -> float:
    if ws == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU reference (oracle port of the reference's CPU path)
# ---------------------------------------------------------------------------

def _cpu_reference_step(w, q_np, kc_np, vc_np, R_np, tokens):
    """One bounded slice: one (batch, kv-head) pair, `tokens` positions, its query heads."""
    import numpy as np
    import oracle
    p = oracle.QuantParams.default(w.dim, *w.bits)
    G = w.q_heads // w.kv_heads
    kc = kc_np[:tokens]
    vc = vc_np[:tokens]
    vdec = oracle.decode(vc.astype(np.int64), R_np, p).reshape(1, 1, tokens, w.dim)
    q4 = q_np[:G].reshape(G, 1, 1, w.dim).transpose(1, 0, 2, 3)      # (1, G, 1, d)
    out, _ = oracle.polar_attention_forward_f32(q4, np.broadcast_to(kc[None, None], (1, G, tokens, w.m)),
                                                np.broadcast_to(vdec, (1, G, tokens, w.dim)), R_np, p)
    return out


def cpu_reference_bandwidth(w, kc, vc, q, R, budget_s=12.0, tokens=None):
    """GB/s of the CPU reference on a slice, same byte accounting as the GPU metric."""
    import numpy as np
    G = w.q_heads // w.kv_heads
    kc_np = kc[0, 0].cpu().numpy()
    vc_np = vc[0, 0].cpu().numpy()
    q_np = q[0, :G].float().cpu().numpy()
    R_np = R.numpy()
    tokens = tokens or min(w.seq_len, 4096)
    _cpu_reference_step(w, q_np, kc_np, vc_np, R_np, min(tokens, 256))          # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        _cpu_reference_step(w, q_np, kc_np, vc_np, R_np, tokens)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 50:
            break
    per = el / reps
    qb = torch.finfo(w.q_dtype).bits // 8
    nbytes = 2 * tokens * w.m * w.code_bytes + G * w.dim * (qb + 4)
    return nbytes / per / 1e9, per, tokens, reps


# ---------------------------------------------------------------------------
# GPU decode benchmark
# ---------------------------------------------------------------------------

def _partition(w, ws, rank):
    """How N ranks share the workload: replicas, batch shards or sequence shards."""
    from prismkv_b200.dist import shard_range
    if ws > 1 and w.name == "longctx-splitseq":
        a, b = shard_range(w.seq_len, ws, rank)
        return "sequence", w.scaled(seq_len=b - a), (a, b)
    if ws > 1 and w.name == "aggressive-332":
        a, b = shard_range(w.batch, ws, rank)
        return "batch", w.scaled(batch=b - a), (a, b)
    return "replicas", w, None


def bench_decode(args, ws, rank, device):
    from prismkv_b200 import _lib, decode_attention
    from prismkv_b200.dist import gather_partials, split_sequence_decode
    from prismkv_b200.synthetic import WORKLOADS, make_kv_codes, make_query, make_quantizer

    w = WORKLOADS[args.workload]
    if args.batch:
        w = w.scaled(batch=args.batch)         # a smaller case of the same kernel, for profilers
    mode, lw, span = _partition(w, ws, rank)
    quant = make_quantizer(w)
    codec = quant.codec(device)
    kc, vc = make_kv_codes(lw, quant, device, seed=rank)
    if mode == "replicas":
        q = make_query(w, device, seed=100 + rank)
    elif mode == "batch":
        q = make_query(w, device, seed=100)[span[0]:span[1]].contiguous()
    else:
        q = make_query(w, device, seed=100)
    B, Hq, D = q.shape
    out = torch.empty(B, Hq, D, dtype=torch.float32, device=device)
    scrub = L2Scrub(device)
    stream = torch.cuda.current_stream(device)
    plan = codec.describe(q, kc, vc)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    mids = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]

    graphs = []
    exchange = None
    if mode == "sequence" and args.exchange == "peer":
        from prismkv_b200.dist import PeerExchange
        exchange = PeerExchange(B * Hq, D, device)

    def seq_step():
        split_sequence_decode(quant, q, kc, vc, out=out, exchange=exchange)

    def step(i=None):
        if i is not None:
            starts[i].record(stream)
        if mode == "sequence":
            if graphs:
                graphs[(i or 0) % len(graphs)].replay()
            else:
                seq_step()
        else:
            codec.attention(q, kc, vc, out=out)
        if i is not None:
            ends[i].record(stream)

    for _ in range(args.warmup):
        scrub()
        step()
    torch.cuda.synchronize(device)
    attn_only_ms = None
    if mode == "sequence":
        # the attention kernel alone (roofline), then the three launches of a step captured in one
        # CUDA graph, so the host's launch gaps between them leave the timed step
        ks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(20)]
        for a_, b_ in ks:
            scrub()
            a_.record(stream)
            codec.attention(q, kc, vc, partial=True)
            b_.record(stream)
        torch.cuda.synchronize(device)
        attn_only_ms = sum(a_.elapsed_time(b_) for a_, b_ in ks) / len(ks)
        _barrier(ws)
        # two graphs: the peer exchange alternates between two buffer halves from call to call
        for _ in range(2 if exchange is not None else 1):
            g_ = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_):
                seq_step()
            graphs.append(g_)
        torch.cuda.synchronize(device)
        _barrier(ws)
        for j in range(4):
            scrub()
            graphs[j % len(graphs)].replay()
    torch.cuda.synchronize(device)
    _barrier(ws)
    torch.cuda.synchronize(device)
    with ClockSampler(device.index) as clk:
        wall0 = time.perf_counter()
        for i in range(args.steps):
            scrub()
            step(i)
        torch.cuda.synchronize(device)
        wall = time.perf_counter() - wall0
    _barrier(ws)
    step_ms = [s_.elapsed_time(e) for s_, e in zip(starts, ends)]
    kern_ms = [attn_only_ms] if mode == "sequence" else step_ms            # the attention kernel alone
    local_ms = sum(step_ms) / len(step_ms)
    local_kern_ms = sum(kern_ms) / len(kern_ms)
    ms = _max_over_ranks(local_ms, ws, device)
    if _lib.device_error() != 0:
        raise RuntimeError("device error flag set during the benchmark")

    local_bytes = lw.decode_bytes()
    if mode == "replicas":
        total_bytes = local_bytes * ws
    elif mode == "batch":
        total_bytes = w.decode_bytes()
    else:                                  # every rank reads its codes and the query, writes the output
        total_bytes = w.kv_code_bytes() + ws * (local_bytes - lw.kv_code_bytes())
    value = total_bytes / (ms * 1e-3) / 1e9
    achieved = local_bytes / (local_kern_ms * 1e-3) / 1e9
    peak, peak_kind = _peaks()

    # end to end through the public API: pinned host inputs -> device -> kernel(s) -> host output
    e2e_steps = max(3, min(args.steps, 20))
    h_kc = kc.cpu().pin_memory()
    h_vc = vc.cpu().pin_memory()
    h_q = q.cpu().pin_memory()
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    d_kc, d_vc, d_q = torch.empty_like(kc), torch.empty_like(vc), torch.empty_like(q)

    def e2e_step():
        d_kc.copy_(h_kc, non_blocking=True)
        d_vc.copy_(h_vc, non_blocking=True)
        d_q.copy_(h_q, non_blocking=True)
        if mode == "sequence":
            o = split_sequence_decode(quant, d_q, d_kc, d_vc, exchange=exchange)
        else:
            o = decode_attention(quant, d_q, d_kc, d_vc)
        h_out.copy_(o, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(device)
    _barrier(ws)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1) / e2e_steps, ws, device)
    h2d = h_kc.numel() * h_kc.element_size() + h_vc.numel() * h_vc.element_size() + h_q.numel() * h_q.element_size()
    d2h = h_out.numel() * h_out.element_size()

    parallelism = {"replicas": f"replicas x{ws}", "batch": f"batch-sharded x{ws} (no collective)",
                   "sequence": f"sequence-sharded x{ws} (" + ("symmetric-memory peer reads" if exchange is not None
                                                                else "NCCL all-gather") +
                               " of partials + LSE combine)"}[mode]
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak" if mode == "replicas" else "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.name, "batch": w.batch, "q_heads": w.q_heads, "kv_heads": w.kv_heads,
                   "seq_len": w.seq_len, "head_dim": w.dim, "bits": "+".join(map(str, w.bits)),
                   "codes": "uint8" if w.code_bytes == 1 else "uint16",
                   "codebook": "learned+bias" if w.learned else "uniform-polar",
                   "q_dtype": str(w.q_dtype).replace("torch.", ""),
                   "bytes_per_step": total_bytes, "l2": L2Scrub.DESCRIPTION,
                   "parallelism": parallelism},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": (_committed_traffic(plan["kernel"], w.name)
                                 if mode == "replicas" and not args.batch else None),
                     "kernel": plan["kernel"], "num_splits": plan["num_splits"],
                     "balanced": bool(plan["balanced"])},
        "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": args.steps * (2 if mode == "sequence" else 1),
        "clocks": clk.summary(),
        "wall_s_timed": round(wall, 4),
    }
    if mode == "sequence":
        line["attn_ms_per_step"] = round(local_kern_ms, 5)
        line["config"]["step"] = ("partial attention + " + ("symmetric-memory barrier + peer-read LSE combine"
                                  if exchange is not None else "NCCL all-gather + LSE combine") +
                                  ", one CUDA graph per step")
    graphs.clear()                              # release the graphs holding collectives before teardown
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        gbs, per, tokens, reps = cpu_reference_bandwidth(w, kc, vc, q, quant.R)
        line["cpu_baseline"] = {"value": round(gbs, 4), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                                "sample": f"one (batch, kv-head) slice of {tokens} tokens x {w.q_heads // w.kv_heads} "
                                          f"query heads, {reps} reps, {per * 1e3:.1f} ms each; NumPy restatement of "
                                          "PolarAttentionApprox.forward with decoded V"}
    return line


def bench_encode(args, ws, rank, device):
    """Encode of one layer's new tokens: 32768 tokens x kv heads, K and V, bf16 in -> packed codes
    (learned-gqa: learned codebooks + BiasTable, 8 KV heads; phi3-decode: uniform polar, 32 heads)."""
    import numpy as np
    from prismkv_b200 import _lib
    from prismkv_b200.synthetic import WORKLOADS, make_encode_input, make_quantizer

    w = WORKLOADS[args.encode_workload]
    quant = make_quantizer(w)
    codec = quant.codec(device)
    tokens = 32768
    x = make_encode_input(w, device, tokens=tokens, seed=rank)
    codes = torch.empty(x.shape[0], w.m, dtype=torch.int16, device=device)
    scrub = L2Scrub(device)
    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        scrub()
        codec.encode(x, out=codes)
    torch.cuda.synchronize(device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    _barrier(ws)
    with ClockSampler(device.index) as clk:
        for s, e in ev:
            scrub()
            s.record(stream)
            codec.encode(x, out=codes)
            e.record(stream)
        torch.cuda.synchronize(device)
    _barrier(ws)
    local_ms = sum(s.elapsed_time(e) for s, e in ev) / len(ev)
    ms = _max_over_ranks(local_ms, ws, device)
    assert _lib.device_error() == 0
    nbytes = x.numel() * x.element_size() + codes.numel() * 2
    peak, peak_kind = _peaks()
    kernel = "encode_tc_kernel" if (w.dim == 96 and x.dtype == torch.bfloat16) else "encode_kernel"

    # end to end through the public API: pinned bf16 rows -> device -> encode -> codes back to the host
    h_x = x.cpu().pin_memory()
    h_codes = torch.empty(codes.shape, dtype=codes.dtype).pin_memory()
    d_x = torch.empty_like(x)

    def e2e_step():
        d_x.copy_(h_x, non_blocking=True)
        h_codes.copy_(quant.encode_compact(d_x), non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(3, min(args.steps, 20))
    e0.record(stream)
    for _ in range(n_e2e):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1) / n_e2e, ws, device)
    line = {
        "metric": METRIC, "value": round(tokens * ws / (ms * 1e-3) / 1e6, 3), "unit": "Mtok/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 in, f32 rotation", "data": "synthetic",
        "config": {"workload": f"{w.name}-encode", "tokens": tokens, "kv_heads": w.kv_heads, "head_dim": w.dim,
                   "input": "bf16", "codes": "uint16", "bytes_per_step": nbytes, "l2": L2Scrub.DESCRIPTION},
        "roofline": {"bound": "hbm", "achieved": round(nbytes / (local_ms * 1e-3) / 1e9, 2), "peak": peak,
                     "unit": "GB/s", "frac": round(nbytes / (local_ms * 1e-3) / 1e9 / peak, 4), "peak_kind": peak_kind,
                     "traffic": _committed_traffic(kernel, w.name), "kernel": kernel},
        "e2e": {"value": round(tokens * ws / (e2e_ms * 1e-3) / 1e6, 3), "unit": "Mtok/s",
                "h2d_bytes_per_step": h_x.numel() * h_x.element_size(),
                "d2h_bytes_per_step": h_codes.numel() * h_codes.element_size(), "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": args.steps, "clocks": clk.summary(),
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        import oracle
        p = oracle.QuantParams.default(w.dim, *w.bits)
        host = quant.codec(device).host
        if host.xy_mode == 1:
            p.codebook = host.codebook
        rows = 2 * w.kv_heads * 256                      # 256 tokens of the layer, K and V of every head
        xs = x[:rows].float().cpu().numpy()
        R = quant.R.numpy()
        oracle.encode(xs[:64], R, p)
        t0 = time.perf_counter()
        reps = 0
        while True:
            oracle.encode(xs, R, p)
            reps += 1
            if time.perf_counter() - t0 > 10.0 or reps >= 20:
                break
        per = (time.perf_counter() - t0) / reps
        line["cpu_baseline"] = {"value": round(256 / per / 1e6, 5), "unit": "Mtok/s", "cores": os.cpu_count(),
                                "kind": "port", "sample": f"{rows} rows (256 tokens x {w.kv_heads} heads x K, V), "
                                f"{reps} reps, {per * 1e3:.1f} ms each; NumPy restatement of "
                                "StackedPlaneQuantizer.encode"}
    return line


def bench_reference(args, ws, rank):
    """The reference's CPU path on the host cores, one bounded slice per step."""
    if rank != 0:
        return None
    import numpy as np
    from prismkv_b200.synthetic import WORKLOADS
    from prismkv_b200.utils import make_rotation
    import oracle
    w = WORKLOADS[args.workload]
    R = make_rotation(w.dim, 42).numpy()
    p = oracle.QuantParams.default(w.dim, *w.bits)
    g = np.random.default_rng(0)
    G = w.q_heads // w.kv_heads
    tokens = min(w.seq_len, 4096)
    K = g.standard_normal((tokens, w.dim)).astype(np.float32)
    V = g.standard_normal((tokens, w.dim)).astype(np.float32)
    kc = oracle.encode(K, R, p).astype(np.int16)
    vc = oracle.encode(V, R, p).astype(np.int16)
    q = g.standard_normal((G, w.dim)).astype(np.float32)
    # size the slice so that warmup + steps stay within ~2 minutes
    t0 = time.perf_counter()
    _cpu_reference_step(w, q, kc, vc, R, tokens)
    one = time.perf_counter() - t0
    budget = 120.0
    n_calls = args.steps + args.warmup
    if one * n_calls > budget:
        tokens = max(64, int(tokens * budget / (one * n_calls)))
    for _ in range(args.warmup):
        _cpu_reference_step(w, q, kc, vc, R, tokens)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _cpu_reference_step(w, q, kc, vc, R, tokens)
    el = time.perf_counter() - t0
    qb = torch.finfo(w.q_dtype).bits // 8
    nbytes = 2 * tokens * w.m * w.code_bytes + G * w.dim * (qb + 4)
    gbs = nbytes * args.steps / el / 1e9
    cores = os.cpu_count()
    sample = (f"{tokens} tokens of one (batch, kv-head) slice x {G} query heads per step; NumPy restatement of "
              "PolarAttentionApprox.forward (polar_attention.py:277-309) with decoded V")
    return {"metric": METRIC, "value": round(gbs, 5), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": w.name, "batch": w.batch, "q_heads": w.q_heads, "kv_heads": w.kv_heads,
                       "seq_len": w.seq_len, "head_dim": w.dim, "bits": "+".join(map(str, w.bits))},
            "cpu_baseline": {"value": round(gbs, 5), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(gbs, 5), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="prismkv", choices=["prismkv", "reference"])
    ap.add_argument("--workload", default="phi3-decode")
    ap.add_argument("--mode", default="decode", choices=["decode", "encode"])
    ap.add_argument("--encode-workload", default="learned-gqa", choices=["learned-gqa", "phi3-decode"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0,
                    help="decode: override the workload's batch (small cases for ncu captures)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="split-sequence exchange: symmetric-memory peer reads or an NCCL all-gather")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = _dist_env()
    if args.impl == "reference":
        line = bench_reference(args, ws, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if ws > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    try:
        line = bench_decode(args, ws, rank, device) if args.mode == "decode" else bench_encode(args, ws, rank, device)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if ws > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.path.insert(0, ROOT)
    sys.exit(main())
