"""bench.py's reference arm runs on the host's cores and prints one JSON line with the
benchmark contract's keys (impl, metric, value, unit, cpu_baseline, e2e with zero copy
bytes), on the workload the GPU arm measures; with the reference installed in baseline/_ref
it times the reference's own code."""

import json
import os
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 3
    assert d["unit"] == "GB/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["workload"] == "longctx-splitseq"
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    if os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "prismkv")):
        assert cb["kind"] == "reference" and "PolarAttentionApprox.forward" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_partition_shards_the_sharded_workloads_and_replicates_the_rest():
    """longctx splits its sequence and aggressive-332 its batch across ranks, covering every
    token / row exactly once; the other workloads run one replica per rank."""
    sys.path.insert(0, ROOT)
    import bench
    from prismkv_b200.synthetic import WORKLOADS
    for ws in (1, 2, 3, 8):
        for name, w in WORKLOADS.items():
            parts = [bench._partition(w, ws, r) for r in range(ws)]
            modes = {m for m, _, _ in parts}
            if ws > 1 and name == "longctx-splitseq":
                assert modes == {"sequence"}
                spans = [s for _, _, s in parts]
                assert spans[0][0] == 0 and spans[-1][1] == w.seq_len
                assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
                assert sum(lw.seq_len for _, lw, _ in parts) == w.seq_len
            elif ws > 1 and name == "aggressive-332":
                assert modes == {"batch"}
                assert sum(lw.batch for _, lw, _ in parts) == w.batch
            else:
                assert modes == {"replicas"} and all(lw == w for _, lw, _ in parts)
