"""CPU: bench.py's bookkeeping -- the algorithmic figures per chain-step, the
traffic record lookup that ties a committed ncu capture to the kernel sources
it was taken on, and the reference arm's JSON line (the oracle port on a
bounded sample; no GPU)."""
from __future__ import annotations

import json
import subprocess
import sys

from conftest import ROOT

sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def test_canonical_figures():
    wl = bench.WORKLOADS["3"]
    assert wl.N == 16384
    assert wl.step_flops == 4106 and wl.step_bytes_f32 == 472  # D8M8, FP32 at the reference ABI
    assert wl.fwd_flops == 793 and wl.bwd_flops == 3313
    assert wl.fwd_bytes == 120 and wl.bwd_bytes == 208  # BF16 k/q/v as read and written
    wl4 = bench.WORKLOADS["4"]
    assert wl4.N == 65536 and wl4.step_flops == 734 and wl4.step_bytes_f32 == 256
    assert wl4.shard(4) == 16384 and wl.shard(4) == 16384  # strong vs weak scaling


def test_traffic_records_match_the_current_sources():
    for key in ("3:backward_split<8,8,1,0,bf16>", "4:backward_chain<2,8,0,1,0,bf16>"):
        rec, src = bench._captured_traffic(key)
        assert rec is not None, src
        assert rec["sources"] == bench._kernel_sources_hash()
        assert rec["dram_bytes_per_full_launch"] > 0
    rec, src = bench._captured_traffic("3:no_such_kernel")
    assert rec is None and "no capture" in src


def test_reference_arm_prints_one_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, timeout=600, check=True).stdout
    lines = [ln for ln in out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["e2e"]["h2d_bytes_per_step"] == 0
