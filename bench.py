"""Benchmark of the PrismKV B200 hot path: decode attention over packed KV codes.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl prismkv|reference]
                    [--workload longctx-splitseq|phi3-decode|aggressive-332|learned-gqa|cpu-roundtrip]
                    [--mode decode|encode]

One step = one fused dequant + flash-decoding attention over the whole
workload's packed K/V (inputs resident in HBM, larger than L2, L2 scrubbed
between steps).  The metric is effective HBM bandwidth: algorithmic bytes
(packed codes read once + query + fp32 output) / device time.  The default
workload is the long-context decode (B=4, 32 query / 8 KV heads, 131072
tokens).  Under torchrun with N > 1 its sequence is sharded over the ranks
(each rank attends over its contiguous token range, the partial softmax
states are exchanged and merged); aggressive-332 is batch-sharded; the
other workloads run one replica per rank.  Before timing, the step's output
is checked against the unsplit single-GPU kernel and against the oracle;
the errors are keys of the JSON line and a mismatch exits non-zero.  The
default line also carries an ``encode`` object: the fused rotate + bin +
pack kernel on one layer's new tokens (Mtok/s).

``--impl reference`` times the reference's own CPU implementation
(PrismKV v1.4.1 installed in baseline/_ref: StackedPlaneQuantizer.decode +
PolarAttentionApprox.forward) on the host cores, one bounded slice of the
workload per step; without that install it times the oracle's NumPy
restatement of the same path.
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
# The reference's CPU path: PrismKV v1.4.1 from baseline/_ref, else the oracle port
# ---------------------------------------------------------------------------

REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _reference_modules():
    """The installed reference's classes (quantizer, attention, codebook, bias), or None."""
    if not os.path.isdir(os.path.join(REF_DIR, "prismkv")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        from prismkv.quantizer.bias_correction import BiasTable
        from prismkv.quantizer.learned_codebook import LearnedSliceCodebook
        from prismkv.quantizer.polar_attention import PolarAttentionApprox
        from prismkv.quantizer.stacked_plane import StackedPlaneQuantizer
    except Exception:                                   # an incomplete install: use the port
        return None
    return StackedPlaneQuantizer, PolarAttentionApprox, LearnedSliceCodebook, BiasTable


def _unit_vectors(w, tokens: int, device):
    """K and V rows of the workload's first unit (batch 0, KV head 0), tokens [0, tokens): the
    same floats make_kv_codes draws for the GPU arm (seed 0), when `device` is the CUDA device
    it drew them on (the draws are replayed call for call); on a CPU device, the same
    distribution from a CPU generator."""
    from prismkv_b200.synthetic import _kv_rows, _workload_layout
    device = torch.device(device)
    g = torch.Generator(device=device).manual_seed(0)
    scales, outlier = _workload_layout(w, device)
    total = w.batch * w.kv_heads * w.seq_len
    chunk = 1 << 21
    out = []
    for _ in range(2):                                  # K, then V, in make_kv_codes' call order
        first = None
        for s in range(0, total, chunk):
            n = min(chunk, total - s)
            head = (torch.arange(s, s + n, device=device) // w.seq_len) % w.kv_heads
            x = _kv_rows(w, g, device, n, head, scales, outlier)
            if first is None:
                first = x[:tokens].float().cpu()
        out.append(first)
    return out[0], out[1]


class ReferenceUnit:
    """One unit (batch 0, KV head 0, its G query heads) through the reference's own CPU code.

    v1 uniform tables: StackedPlaneQuantizer.decode of V, then PolarAttentionApprox.forward over
    the K codes (polar_attention.py:277-309).  Learned codebooks + BiasTable: the reference
    quantizer with both attached decodes K and V, then softmax(q . K^T * d^-1/2) . V, the
    composite the reference's attention implies for that codec.  Without the reference install
    the oracle's NumPy restatement of the same path runs instead (kind "port").
    """

    def __init__(self, w, k_codes, v_codes, q):
        """k_codes, v_codes: (T, m) integer CPU tensors; q: (G, dim) float CPU tensor."""
        import numpy as np
        self.w, self.G = w, w.q_heads // w.kv_heads
        self.kc, self.vc, self.q = k_codes.to(torch.int16), v_codes.to(torch.int16), q.float()
        mods = _reference_modules()
        self.kind = "reference" if mods is not None else "port"
        if mods is not None:
            RefQ, RefAttn, RefCB, RefBias = mods
            torch.set_num_threads(os.cpu_count())
            self.rq = RefQ(dim=w.dim, bits_z=w.bits[0], bits_r=w.bits[1], bits_theta=w.bits[2], seed=42)
            if w.learned:
                from prismkv_b200.synthetic import synthetic_bias, synthetic_codebook
                Cz, K = 1 << w.bits[0], 1 << (w.bits[1] + w.bits[2])
                self.rq._codebooks = RefCB(synthetic_codebook(Cz, K, self.rq.r_max, 11), Cz, K, self.rq.z_min,
                                           self.rq.z_max, self.rq.r_max)
                self.rq._bias = RefBias(synthetic_bias(Cz, 12), delta_z=(self.rq.z_max - self.rq.z_min) / Cz)
            self.attn = RefAttn(*w.bits, z_min=self.rq.z_min, z_max=self.rq.z_max, r_max=self.rq.r_max,
                                R=self.rq.R)
        else:
            import oracle
            from prismkv_b200.utils import make_rotation
            self.p = oracle.QuantParams.default(w.dim, *w.bits)
            if w.learned:
                from prismkv_b200.synthetic import synthetic_bias, synthetic_codebook
                Cz, K = 1 << w.bits[0], 1 << (w.bits[1] + w.bits[2])
                self.p.codebook = synthetic_codebook(Cz, K, self.p.r_max, 11).numpy()
                self.p.bias_table = synthetic_bias(Cz, 12).numpy()
                self.p.bias_delta_z = (self.p.z_max - self.p.z_min) / Cz
            self.R = make_rotation(w.dim, 42).numpy()
            self.kc_np = self.kc.numpy().astype(np.int64)
            self.vc_np = self.vc.numpy().astype(np.int64)
            self.q_np = self.q.numpy()

    def run(self, tokens: int):
        """Attention of the G query heads over the unit's first `tokens` tokens: (G, dim)."""
        w, G = self.w, self.G
        if self.kind == "reference":
            v = self.rq.decode(self.vc[:tokens].long())                     # (T, dim)
            q4 = self.q.view(1, G, 1, w.dim)
            if w.learned:
                k = self.rq.decode(self.kc[:tokens].long())
                s = (q4 @ k.T.unsqueeze(0).unsqueeze(0)) * (w.dim ** -0.5)
                out = torch.softmax(s, dim=-1) @ v
            else:
                kc4 = self.kc[:tokens].view(1, 1, tokens, w.m).expand(1, G, tokens, w.m)
                out, _ = self.attn.forward(q4, kc4, v.view(1, 1, tokens, w.dim).expand(1, G, tokens, w.dim))
            return out.reshape(G, w.dim)
        import numpy as np
        import oracle
        if w.learned:
            return oracle.attention(self.q_np[None], self.kc_np[None, None, :tokens], self.vc_np[None, None, :tokens],
                                    self.R, self.p)[0]
        vdec = oracle.decode(self.vc_np[:tokens], self.R, self.p).reshape(1, 1, tokens, w.dim)
        q4 = self.q_np.reshape(G, 1, 1, w.dim).transpose(1, 0, 2, 3)
        out, _ = oracle.polar_attention_forward_f32(q4, np.broadcast_to(self.kc_np[None, None, :tokens],
                                                                        (1, G, tokens, w.m)),
                                                    np.broadcast_to(vdec, (1, G, tokens, w.dim)), self.R, self.p)
        return torch.from_numpy(np.ascontiguousarray(out)).reshape(G, w.dim)

    def nbytes(self, tokens: int) -> int:
        """Algorithmic bytes of a slice, as the GPU metric counts them: K and V codes once, the
        query in its dtype, the fp32 output."""
        qb = torch.finfo(self.w.q_dtype).bits // 8
        return 2 * tokens * self.w.m * self.w.code_bytes + self.G * self.w.dim * (qb + 4)

    def describe(self, tokens: int, reps: int, per_s: float) -> str:
        what = ("PrismKV v1.4.1 (baseline/_ref) " + ("StackedPlaneQuantizer.decode + softmax(q decode(K)^T) decode(V), "
                                                    "learned codebooks + BiasTable" if self.w.learned else
                                                    "StackedPlaneQuantizer.decode + PolarAttentionApprox.forward")
                if self.kind == "reference" else "oracle NumPy restatement of PolarAttentionApprox.forward + decode")
        return (f"unit (batch 0, KV head 0): {tokens} tokens x {self.G} query heads, {reps} reps of "
                f"{per_s * 1e3:.1f} ms; {what}; torch threads {torch.get_num_threads()}")


def time_reference(unit: ReferenceUnit, budget_s: float, tokens: int, max_reps: int = 50):
    """(GB/s, seconds per call, reps) of the reference slice, timed with perf_counter."""
    unit.run(min(tokens, 256))                                   # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        unit.run(tokens)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= max_reps:
            break
    per = el / reps
    return unit.nbytes(tokens) / per / 1e9, per, reps


# ---------------------------------------------------------------------------
# GPU decode benchmark
# ---------------------------------------------------------------------------

TOL_UNSPLIT = 1e-4          # sharded output vs the unsplit single-GPU kernel (fp32 both ways)


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


def _oracle_tolerance(kernel: str) -> float:
    """The north-star bounds: 1e-3 on the fp32 kernels, 2e-2 on the tensor-core kernel (bf16 operands)."""
    return 2e-2 if kernel == "attn_tc_kernel" else 1e-3


def _oracle_params(w, quant):
    import oracle
    p = oracle.QuantParams(dim=w.dim, bits_z=w.bits[0], bits_r=w.bits[1], bits_theta=w.bits[2],
                           z_min=quant.z_min, z_max=quant.z_max, r_max=quant.r_max)
    if quant._codebooks is not None:
        p.codebook = quant._codebooks.codebooks.numpy()
    if quant._bias is not None:
        p.bias_table = quant._bias.table.numpy()
        p.bias_delta_z = quant._bias.delta_z
    return p


def parity_check(w, lw, mode, span, quant, q, kc, vc, out, ws, rank, device, kernel):
    """The step's output, before timing, against (a) the unsplit single-GPU kernel over the whole
    sequence (sequence shards; every row) and (b) the oracle for two (batch, KV head) units.
    Runs on rank 0; every rank learns the verdict.  Returns the keys for the JSON line."""
    import numpy as np
    import oracle
    from prismkv_b200.dist import shard_range
    from prismkv_b200.synthetic import make_kv_codes
    res = {}
    ok = True
    if rank == 0:
        G = w.q_heads // w.kv_heads
        codec = quant.codec(device)
        kfull, vfull, qfull, ofull = kc, vc, q, out
        if mode == "sequence":
            # every rank's shard, drawn as that rank drew it, in rank order
            parts = [make_kv_codes(w.scaled(seq_len=shard_range(w.seq_len, ws, r)[1] - shard_range(w.seq_len, ws, r)[0]),
                                   quant, device, seed=r) for r in range(ws)]
            kfull = torch.cat([p_[0] for p_ in parts], dim=2)
            vfull = torch.cat([p_[1] for p_ in parts], dim=2)
            unsplit = codec.attention(q, kfull, vfull)
            res["vs_unsplit_max_abs"] = float((out - unsplit).abs().max())
            res["tol_unsplit"] = TOL_UNSPLIT
            ok &= res["vs_unsplit_max_abs"] <= TOL_UNSPLIT
        B, Hkv = kfull.shape[0], kfull.shape[1]
        units = sorted({(0, 0), (B - 1, Hkv - 1)})
        p = _oracle_params(w, quant)
        err = 0.0
        for b, hk in units:
            ref = oracle.attention(qfull[b:b + 1, G * hk:G * hk + G].float().cpu().numpy(),
                                   kfull[b:b + 1, hk:hk + 1].cpu().numpy().astype(np.int64),
                                   vfull[b:b + 1, hk:hk + 1].cpu().numpy().astype(np.int64), quant.R.numpy(), p)
            err = max(err, float(np.abs(ofull[b:b + 1, G * hk:G * hk + G].cpu().numpy() - ref).max()))
        res["vs_oracle_max_abs"] = err
        res["tol_oracle"] = _oracle_tolerance(kernel)
        res["oracle_units"] = [list(u) for u in units]
        ok &= err <= res["tol_oracle"]
        res["ok"] = bool(ok)
    if ws > 1:
        flag = torch.tensor([1.0 if (rank != 0 or ok) else 0.0], device=device)
        torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN)
        ok = bool(flag.item() > 0.5)
    return res, ok


def bench_decode(args, ws, rank, device):
    from prismkv_b200 import _lib, decode_attention
    from prismkv_b200.dist import split_sequence_decode
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
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]

    graphs = []
    exchange = None
    if mode == "sequence" and args.exchange == "xr":
        from prismkv_b200.dist import SequenceExchange
        exchange = SequenceExchange(quant, q, kc, wait_ms=args.wait_ms)
        out = exchange.out                     # the merged rows land in this rank's exchange buffer

    def seq_step():
        if exchange is not None:
            exchange.run(q, kc, vc)            # one launch: attention + cross-GPU merge
        else:
            split_sequence_decode(quant, q, kc, vc, out=out)

    def step(i=None):
        if i is not None:
            starts[i].record(stream)
        if mode == "sequence":
            if graphs:
                graphs[0].replay()
            else:
                seq_step()
        else:
            codec.attention(q, kc, vc, out=out)
        if i is not None:
            ends[i].record(stream)

    # parity first: one step, checked, before anything is timed
    step()
    torch.cuda.synchronize(device)
    parity, ok = parity_check(w, lw, mode, span, quant, q, kc, vc, out, ws, rank, device, plan["kernel"])
    if not ok:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "error": "parity check failed", "parity": parity}), flush=True)
        raise SystemExit(3)

    for _ in range(args.warmup):
        scrub()
        step()
    torch.cuda.synchronize(device)
    attn_only_ms = None
    if mode == "sequence":
        # the attention kernel alone over this rank's shard (roofline)
        ks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(20)]
        for a_, b_ in ks:
            scrub()
            a_.record(stream)
            codec.attention(q, kc, vc, partial=True)
            b_.record(stream)
        torch.cuda.synchronize(device)
        attn_only_ms = sum(a_.elapsed_time(b_) for a_, b_ in ks) / len(ks)
        _barrier(ws)
        # the step's launches captured in one CUDA graph (the all-gather path: attention, NCCL,
        # combine; the exchange path: its one kernel), so host-side Python between the timing
        # events and the launch stays out of the timed step
        g_ = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_):
            seq_step()
        graphs.append(g_)
        torch.cuda.synchronize(device)
        _barrier(ws)
        for j in range(4):
            scrub()
            graphs[0].replay()
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
    if exchange is not None:
        exchange.check()                        # raises if a bounded cross-GPU wait ran out
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
            o = exchange.run(d_q, d_kc, d_vc) if exchange is not None else split_sequence_decode(quant, d_q, d_kc, d_vc)
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

    parallelism = {"replicas": "single GPU" if ws == 1 else f"replicas x{ws}",
                   "batch": f"batch-sharded x{ws} (no collective)",
                   "sequence": f"sequence-sharded x{ws} (" + ("in-kernel exchange of partials over CUDA-IPC "
                                                                "peer memory, LSE merge by the last rank per unit"
                                                                if exchange is not None else
                                                                "NCCL all-gather of partials + LSE combine") + ")"}[mode]
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak" if mode == "replicas" else "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; shapes and distributions of the config)",
        "config": workload_config(w, total_bytes, parallelism),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": (_committed_traffic(plan["kernel"], w.name)
                                 if mode == "replicas" and not args.batch else None),
                     "kernel": plan["kernel"], "num_splits": plan["num_splits"],
                     "balanced": bool(plan["balanced"])},
        "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4)},
        "parity": parity,
        "gpu_launches": args.steps * (2 if (mode == "sequence" and exchange is None) else 1),
        "clocks": clk.summary(),
        "wall_s_timed": round(wall, 4),
    }
    if mode == "sequence":
        line["attn_ms_per_step"] = round(local_kern_ms, 5)
        line["config"]["step"] = ("one kernel per rank: attention over the shard, partials stored into every "
                                  "rank's buffer, merge + R by the rank completing each unit's count, bounded "
                                  "completion wait; replayed from a CUDA graph" if exchange is not None else
                                  "partial attention + NCCL all-gather + LSE combine, one CUDA graph per step")
    graphs.clear()                              # release the graphs holding collectives before teardown
    if exchange is not None:
        exchange.close()                        # collective: no rank frees a buffer a peer may write
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        # the reference's CPU path on the host cores, over the GPU arm's own codes and query for
        # the first unit; its output is also compared with this GPU step's output for that unit
        G = w.q_heads // w.kv_heads
        tokens = min(w.seq_len, args.cpu_tokens)
        unit = ReferenceUnit(w, kc[0, 0, :tokens].cpu(), vc[0, 0, :tokens].cpu(), q[0, :G].float().cpu())
        gbs, per, reps = time_reference(unit, budget_s=12.0, tokens=tokens)
        line["cpu_baseline"] = {"value": round(gbs, 5), "unit": "GB/s", "cores": os.cpu_count(), "kind": unit.kind,
                                "sample": unit.describe(tokens, reps, per)}
        if tokens == w.seq_len:
            line["cpu_baseline"]["max_abs_vs_gpu"] = float((unit.run(tokens) - out[0, :G].cpu()).abs().max())
    return line


def workload_config(w, total_bytes, parallelism):
    return {"workload": w.name, "batch": w.batch, "q_heads": w.q_heads, "kv_heads": w.kv_heads,
            "seq_len": w.seq_len, "head_dim": w.dim, "bits": "+".join(map(str, w.bits)),
            "codes": "uint8" if w.code_bytes == 1 else "uint16",
            "codebook": "learned+bias" if w.learned else "uniform-polar",
            "kv": "N(0,1), 1% of channels x8" if w.outliers else
                  ("N(0,1) x per-head U[0.5,2]" if w.head_scale else "N(0,1)"),
            "q_dtype": str(w.q_dtype).replace("torch.", ""),
            "bytes_per_step": total_bytes, "l2": L2Scrub.DESCRIPTION,
            "parallelism": parallelism}


def bench_encode(args, ws, rank, device, steps=None, warmup=None, cpu_baseline=True):
    """Encode of one layer's new tokens: 32768 tokens x kv heads, K and V, bf16 in -> packed codes
    (learned-gqa: learned codebooks + BiasTable, 8 KV heads; phi3-decode: uniform polar, 32 heads)."""
    from prismkv_b200 import _lib
    from prismkv_b200.synthetic import WORKLOADS, make_encode_input, make_quantizer

    steps = steps or args.steps
    warmup = warmup or args.warmup
    w = WORKLOADS[args.encode_workload]
    quant = make_quantizer(w)
    codec = quant.codec(device)
    tokens = 32768
    x = make_encode_input(w, device, tokens=tokens, seed=rank)
    codes = torch.empty(x.shape[0], w.m, dtype=torch.int16, device=device)
    scrub = L2Scrub(device)
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        scrub()
        codec.encode(x, out=codes)
    torch.cuda.synchronize(device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
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
    if _lib.device_error() != 0:
        raise RuntimeError("device error flag set during the encode benchmark")
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
    n_e2e = max(3, min(steps, 20))
    e0.record(stream)
    for _ in range(n_e2e):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1) / n_e2e, ws, device)
    line = {
        "metric": METRIC, "value": round(tokens * ws / (ms * 1e-3) / 1e6, 3), "unit": "Mtok/s", "n_gpus": ws,
        "steps": steps, "warmup": warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 in, f32 rotation", "data": "synthetic",
        "config": {"workload": f"{w.name}-encode", "tokens": tokens, "kv_heads": w.kv_heads, "head_dim": w.dim,
                   "input": "bf16", "codes": "uint16", "bytes_per_step": nbytes, "l2": L2Scrub.DESCRIPTION},
        "roofline": {"bound": "hbm", "achieved": round(nbytes / (local_ms * 1e-3) / 1e9, 2), "peak": peak,
                     "unit": "GB/s", "frac": round(nbytes / (local_ms * 1e-3) / 1e9 / peak, 4), "peak_kind": peak_kind,
                     "traffic": _committed_traffic(kernel, w.name), "kernel": kernel},
        "e2e": {"value": round(tokens * ws / (e2e_ms * 1e-3) / 1e6, 3), "unit": "Mtok/s",
                "h2d_bytes_per_step": h_x.numel() * h_x.element_size(),
                "d2h_bytes_per_step": h_codes.numel() * h_codes.element_size(), "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": steps, "clocks": clk.summary(),
    }
    if cpu_baseline and rank == 0 and ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = _encode_cpu_baseline(w, x, quant)
    return line


def _encode_cpu_baseline(w, x, quant, budget_s=8.0):
    """The reference's StackedPlaneQuantizer.encode (baseline/_ref; codebooks and BiasTable attached
    for learned workloads) on 256 tokens of the layer, or the oracle port without the install."""
    rows = 2 * w.kv_heads * 256                      # 256 tokens of the layer, K and V of every head
    xs = x[:rows].float().cpu()
    mods = _reference_modules()
    if mods is not None:
        RefQ, _, RefCB, RefBias = mods
        torch.set_num_threads(os.cpu_count())
        rq = RefQ(dim=w.dim, bits_z=w.bits[0], bits_r=w.bits[1], bits_theta=w.bits[2], seed=42)
        if w.learned:
            from prismkv_b200.synthetic import synthetic_bias, synthetic_codebook
            Cz, K = 1 << w.bits[0], 1 << (w.bits[1] + w.bits[2])
            rq._codebooks = RefCB(synthetic_codebook(Cz, K, rq.r_max, 11), Cz, K, rq.z_min, rq.z_max, rq.r_max)
            rq._bias = RefBias(synthetic_bias(Cz, 12), delta_z=(rq.z_max - rq.z_min) / Cz)
        fn, kind = (lambda a: rq.encode(a)), "reference"
        what = "PrismKV v1.4.1 (baseline/_ref) StackedPlaneQuantizer.encode"
    else:
        import oracle
        p = oracle.QuantParams.default(w.dim, *w.bits)
        host = quant.codec(x.device).host
        if host.xy_mode == 1:
            p.codebook = host.codebook
        R = quant.R.numpy()
        fn, kind = (lambda a: oracle.encode(a.numpy(), R, p)), "port"
        what = "NumPy restatement of StackedPlaneQuantizer.encode"
    fn(xs[:64])
    t0 = time.perf_counter()
    reps = 0
    while True:
        fn(xs)
        reps += 1
        if time.perf_counter() - t0 > budget_s or reps >= 20:
            break
    per = (time.perf_counter() - t0) / reps
    return {"value": round(256 / per / 1e6, 6), "unit": "Mtok/s", "cores": os.cpu_count(), "kind": kind,
            "sample": f"{rows} rows (256 tokens x {w.kv_heads} heads x K, V), {reps} reps, {per * 1e3:.1f} ms each; "
                      f"{what}; torch threads {torch.get_num_threads()}"}


def bench_reference(args, ws, rank):
    """The reference's own CPU path on the host cores, one bounded slice of the workload per step
    (rank 0 only; other ranks exit without work)."""
    if rank != 0:
        return None
    from prismkv_b200.synthetic import WORKLOADS, make_query, make_quantizer
    w = WORKLOADS[args.workload]
    G = w.q_heads // w.kv_heads
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    tokens = min(w.seq_len, args.cpu_tokens)
    # inputs: the GPU arm's first unit (its seeded K/V draws and query), encoded by the reference's
    # own quantizer on the host (set-up, not timed)
    kx, vx = _unit_vectors(w, tokens, dev)
    qv = make_query(w, dev, seed=100)[0, :G].float().cpu()
    mods = _reference_modules()
    if mods is not None:
        RefQ = mods[0]
        enc = RefQ(dim=w.dim, bits_z=w.bits[0], bits_r=w.bits[1], bits_theta=w.bits[2], seed=42)
        if w.learned:
            from prismkv_b200.synthetic import synthetic_bias, synthetic_codebook
            Cz, K = 1 << w.bits[0], 1 << (w.bits[1] + w.bits[2])
            enc._codebooks = mods[2](synthetic_codebook(Cz, K, enc.r_max, 11), Cz, K, enc.z_min, enc.z_max, enc.r_max)
            enc._bias = mods[3](synthetic_bias(Cz, 12), delta_z=(enc.z_max - enc.z_min) / Cz)
        kc, vc = enc.encode(kx), enc.encode(vx)
    else:
        import oracle
        p = oracle.QuantParams.default(w.dim, *w.bits)
        R = make_quantizer(w).R.numpy()
        kc = torch.from_numpy(oracle.encode(kx.numpy(), R, p))
        vc = torch.from_numpy(oracle.encode(vx.numpy(), R, p))
    unit = ReferenceUnit(w, kc, vc, qv)
    # size the slice so that warmup + steps stay within ~2 minutes
    t0 = time.perf_counter()
    unit.run(tokens)
    one = time.perf_counter() - t0
    budget = 120.0
    n_calls = args.steps + args.warmup
    if one * n_calls > budget:
        tokens = max(64, int(tokens * budget / (one * n_calls)))
    for _ in range(args.warmup):
        unit.run(tokens)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        unit.run(tokens)
    el = time.perf_counter() - t0
    gbs = unit.nbytes(tokens) * args.steps / el / 1e9
    per = el / args.steps
    return {"metric": METRIC, "value": round(gbs, 5), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(per * 1e3, 4), "higher_is_better": True,
            "scaling": "weak" if ws == 1 else "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; shapes and distributions of the config)", "impl": "reference",
            "config": workload_config(w, w.decode_bytes(), "single GPU" if ws == 1 else
                                      {"longctx-splitseq": f"sequence-sharded x{ws}", "aggressive-332":
                                       f"batch-sharded x{ws} (no collective)"}.get(w.name, f"replicas x{ws}")),
            "cpu_baseline": {"value": round(gbs, 5), "unit": "GB/s", "cores": os.cpu_count(), "kind": unit.kind,
                             "sample": unit.describe(tokens, args.steps, per)},
            "e2e": {"value": round(gbs, 5), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="prismkv", choices=["prismkv", "reference"])
    ap.add_argument("--workload", default="longctx-splitseq")
    ap.add_argument("--mode", default="decode", choices=["decode", "encode"])
    ap.add_argument("--encode-workload", default="learned-gqa", choices=["learned-gqa", "phi3-decode"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-encode", action="store_true", help="decode: leave the encode object out of the line")
    ap.add_argument("--cpu-tokens", type=int, default=16384,
                    help="tokens of the unit the reference's CPU path attends over per call")
    ap.add_argument("--batch", type=int, default=0,
                    help="decode: override the workload's batch (small cases for ncu captures)")
    ap.add_argument("--exchange", default="xr", choices=["xr", "nccl"],
                    help="split-sequence exchange: in-kernel over CUDA-IPC peer memory, or an NCCL all-gather")
    ap.add_argument("--wait-ms", type=float, default=2000.0,
                    help="bound on the in-kernel exchange's cross-GPU completion wait (device time)")
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
        if args.mode == "decode":
            line = bench_decode(args, ws, rank, device)
            if not args.no_encode and ws == 1:
                enc = bench_encode(args, ws, rank, device, steps=min(args.steps, 50), warmup=args.warmup)
                line["encode"] = {k: enc[k] for k in ("value", "unit", "ms_per_step", "config", "roofline", "e2e",
                                                      "cpu_baseline", "clocks") if k in enc}
                line["gpu_launches"] += enc["gpu_launches"]
        else:
            line = bench_encode(args, ws, rank, device)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if ws > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.path.insert(0, ROOT)
    sys.exit(main())
