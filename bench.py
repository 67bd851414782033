"""Benchmark: Bayes-mixer recurrence forward + backward at B256 T512 H64 D8 M8.

One step = the chunked forward kernel + the single-launch replay backward
(full dynamics gradients, no final-state gradients: the trainer's
readout-only path) over N = B*H = 16384 chains of T = 512 tokens, chunk 64,
with BF16 keys/values/queries (the mixer's projection outputs) and FP32
decay / process / observation noise.  Inputs are seeded synthetic tensors with
the mixer's distributions.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 3|4]

``--config 4`` runs the low-state variant instead (D2 M8, B256 T2048, 256
heads -> 65,536 chains), sharded over the ranks (strong scaling).

N > 1 runs under torchrun: for config 3 every rank owns its own 16384 chains
(the layer shards over batch x heads with no exchange), so scaling is weak;
the time is the max over ranks.  ``--impl reference`` times the CPU
restatement of the reference algorithm (oracle/, FP32, all host threads) on a
bounded sample of the same workload; under torchrun only rank 0 runs it.

Besides the device-timed step (``value``) the line carries:
* ``e2e`` -- the public API (``bayesian_layer`` + autograd) with pinned host
  inputs copied in and the readouts and every gradient copied out each step;
* ``api`` -- the same public API on device-resident inputs;
* ``roofline`` -- the backward kernel against the FP32 rate measured live by
  the library's FMA probe (the binding roof) and the measured HBM bandwidth;
* ``parity`` -- a sample of chains of the last timed step checked against the
  FP64 CPU oracle outside the timed region (the oracle is the checker only).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "bayes-ssm_b200"))

FLOOR = 1e-6
METRIC = "Bayes mixer fwd+bwd tok/s/GPU (B256 T512 H64 D8 M8); % of FP32/HBM roofline"
UNIT = "tok/s"
CSRC = ROOT / "bayes-ssm_b200" / "csrc"


class Workload:
    """One benchmarked configuration and its algorithmic figures."""

    def __init__(self, name, b, t, h, d, m, chunk, scaling, dominant):
        self.name, self.B, self.T, self.H, self.D, self.M, self.CHUNK = name, b, t, h, d, m, chunk
        self.scaling, self.dominant = scaling, dominant
        self.N = b * h
        d_, m_ = d, m
        # Algorithmic bytes per chain-step at the dtypes read/written here (BF16
        # k/q/v and their gradients, FP32 everything else).  Forward: read k, q
        # (2D bf16), v (M bf16), decay (D f32), process + observation (2 f32);
        # write y (M f32).  Backward: re-read the same plus gy (M f32); write gk,
        # gq (2D bf16), gv (M bf16), gdecay (D f32), gprocess + gobservation.
        # Chunk-boundary checkpoints and the replay buffer are implementation
        # choices and are not counted.
        rd = 2 * d_ * 2 + m_ * 2 + d_ * 4 + 2 * 4
        self.fwd_bytes = rd + m_ * 4
        self.bwd_bytes = rd + m_ * 4 + rd
        # FLOPs per chain-step (FMA = 2): forward 4D^2+7DM+10D+M+1; backward =
        # recompute (forward - 2DM) + adjoint (18D^2+22DM+10D+M).
        self.fwd_flops = 4 * d_ * d_ + 7 * d_ * m_ + 10 * d_ + m_ + 1
        self.bwd_flops = (self.fwd_flops - 2 * d_ * m_) + (18 * d_ * d_ + 22 * d_ * m_ + 10 * d_ + m_)
        # canonical per chain-step figures (fwd + bwd, FP32 at the reference ABI)
        self.step_flops = 26 * d_ * d_ + 34 * d_ * m_ + 30 * d_ + 3 * m_ + 2
        self.step_bytes_f32 = 4 * (9 * d_ + 5 * m_ + 6)

    def config(self, n_gpus, chains):
        full = chains == self.shard(n_gpus)
        total = chains * n_gpus if self.scaling == "weak" else min(self.N, chains * n_gpus)
        return {"workload": self.name + ("" if full else f" [profiling size: {chains} chains per GPU]"),
                "B": self.B, "T": self.T, "H": self.H, "D": self.D, "M": self.M, "chunk": self.CHUNK,
                "chains_per_gpu": chains, "global_batch": total // self.H, "seq_len": self.T,
                "io_dtype": "bf16 k/q/v, fp32 decay/noise/state",
                "gradients": "k, v, q, decay, process, observation (readout-only loss)",
                "l2": "inputs and replay buffer larger than L2 (GBs moved per step)",
                "parallelism": f"dp{n_gpus} (chains sharded, no data-path collective)"}

    def shard(self, world):
        """Chains per rank: the whole set (weak) or a contiguous 1/world of it (strong)."""
        if self.scaling == "weak":
            return self.N
        return (self.N + world - 1) // world


WORKLOADS = {
    "3": Workload("Bayes mixer recurrence fwd + replay bwd (BASELINE config 3)", 256, 512, 64, 8, 8, 64,
                  "weak", "backward_split<8,8,1,0,bf16> (two-warp replay backward)"),
    "4": Workload("low-state variant D2 M8 fwd + replay bwd (BASELINE config 4), chains sharded over the GPUs",
                  256, 2048, 256, 2, 8, 64, "strong", "backward_chain<2,8,0,1,0,bf16> (one-warp replay backward)"),
}


def _peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _kernel_sources_hash() -> str:
    """Hash of the sources the recurrence kernels are built from."""
    h = hashlib.sha256()
    for name in ("bssm_chain.cu", "bssm_tmem.cuh", "bssm_internal.h", "bssm_common.cuh"):
        h.update((CSRC / name).read_bytes())
    return h.hexdigest()[:16]


def _captured_traffic(kernel_key: str):
    """DRAM bytes per full launch of the dominant kernel from the committed ncu
    capture (a ```json bench-traffic block in its profile), or None when that
    capture was taken on other kernel sources than the ones built here."""
    for prof in sorted((ROOT / "profiles").glob("*.md")):
        for blob in re.findall(r"```json bench-traffic\n(.*?)\n```", prof.read_text(), re.S):
            rec = json.loads(blob)
            if rec.get("kernel_key") != kernel_key:
                continue
            if rec.get("sources") != _kernel_sources_hash():
                return None, f"{prof.name}: capture of other kernel sources ({rec.get('sources')})"
            return rec, prof.name
    return None, "no capture on record"


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons from before the warm-up
    to after the timed loop; summary() keeps the samples stamped inside the
    timed region (mark_start / mark_end), or, when that region is shorter than
    the sampling interval, the nearest sample on each side of it (and says so).
    """

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.file, stderr=subprocess.DEVNULL)
            deadline = time.time() + 5.0  # wait for the first sample
            while time.time() < deadline and os.path.getsize(self.file.name) == 0:
                time.sleep(0.02)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()
        time.sleep(0.12)  # let the sample after the region land

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        from datetime import datetime

        if self.file is None or self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append(dict(t=ts, sm=float(parts[2]), smax=float(parts[3]), power=float(parts[4]),
                                 hw=parts[6], hwt=parts[7], swt=parts[8], pcap=parts[9]))
            except ValueError:
                continue
        os.unlink(self.file.name)
        window = "timed region"
        sel = [r for r in rows if self.t0 is not None and self.t0 <= r["t"] <= self.t1]
        if not sel and rows and self.t0 is not None:
            before = [r for r in rows if r["t"] < self.t0]
            after = [r for r in rows if r["t"] > self.t1]
            sel = ([before[-1]] if before else []) + ([after[0]] if after else [])
            window = "nearest samples (timed region shorter than the 50 ms sampling interval)"
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        reasons = []
        for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                          ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
            if any(r[key].lower() == "active" for r in sel):
                reasons.append(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in sel),
                "sm_max_mhz": max(r["smax"] for r in sel),
                "power_w_max": max(r["power"] for r in sel),
                "samples": len(sel), "window": window, "reasons": reasons}


def make_inputs(wl: Workload, n: int, seed: int, device):
    """Seeded synthetic inputs with the mixer's distributions; on the device
    they are generated there, in slices that bound the FP32 temporaries."""
    import torch
    import torch.nn.functional as F

    t, d, m = wl.T, wl.D, wl.M
    gen_dev = device if device is not None else "cpu"
    g = torch.Generator(device=gen_dev).manual_seed(seed)

    def make(tail, fn, dtype):
        out = torch.empty(n, *tail, device=gen_dev, dtype=dtype)
        step = max(1, (1 << 25) // (t * max(tail[-1] if len(tail) > 1 else 1, 1)))
        for i in range(0, n, step):
            j = min(n, i + step)
            out[i:j] = fn(torch.randn(j - i, *tail, generator=g, device=gen_dev)).to(dtype)
        return out

    bf = torch.bfloat16
    return dict(
        k=make((t, d), lambda x: F.normalize(x, dim=-1), bf),
        q=make((t, d), lambda x: F.normalize(x, dim=-1), bf),
        v=make((t, m), lambda x: x / math.sqrt(m), bf),
        a=make((t, d), lambda x: torch.sigmoid(2.0 + x), torch.float32),
        p=make((t,), lambda x: F.softplus(-4.0 + x), torch.float32),
        r=make((t,), lambda x: F.softplus(x) + 1e-4, torch.float32),
        gy=make((t, m), lambda x: x / math.sqrt(m), torch.float32),
    )


def run_reference(args, wl: Workload, rank: int) -> None:
    """CPU arm: the oracle port (FP32, all host threads), bounded sample."""
    if rank != 0:
        return
    from oracle import oracle

    # torchrun sets OMP_NUM_THREADS=1 per worker; this arm uses every host
    # thread it may run on (set before the oracle library starts OpenMP)
    oracle.set_threads(len(os.sched_getaffinity(0)))
    line = cpu_baseline_measure(wl, steps=args.steps, warmup=args.warmup)
    value = line["value"]
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * wl.B * wl.T / value, "higher_is_better": True, "scaling": wl.scaling,
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": wl.config(args.gpus, wl.shard(args.gpus)),
        "cpu_baseline": line,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def cpu_baseline_measure(wl: Workload, steps: int = 1, warmup: int = 0) -> dict:
    """Time oracle fwd+bwd (FP32) on a sample of chains; scale to tok/s.  The
    sample is sized for about 8 s of work per run, less when many runs are
    asked for, so that the whole measurement stays within a few minutes."""
    target_s = max(0.5, min(8.0, 150.0 / max(1, steps)))
    from oracle import oracle

    threads = oracle.num_threads()

    def arrays(n):
        return {k: v.float().numpy() for k, v in make_inputs(wl, n, 1234, None).items()}

    def one(arr):
        y, _, _ = oracle.forward(arr["k"], arr["v"], arr["q"], arr["a"], arr["p"], arr["r"],
                                 floor=FLOOR, precision="f32")
        oracle.backward(arr["k"], arr["v"], arr["q"], arr["a"], arr["p"], arr["r"], None, None,
                        arr["gy"], None, None, floor=FLOOR, precision="f32")
        return y

    # calibrate on a few chains, then size the sample for ~target_s of work
    # per run (capped at the full workload)
    small = max(8, 2 * threads)
    arr = arrays(small)
    t0 = time.perf_counter()
    one(arr)
    per_chain = (time.perf_counter() - t0) / small
    sample_chains = int(min(wl.N, max(small, target_s / max(per_chain, 1e-9))))
    arr = arrays(sample_chains)
    for _ in range(max(0, min(warmup, 1))):
        one(arr)
    times = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        one(arr)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    tokens = sample_chains * wl.T / wl.H  # a token of the workload carries H chains
    return {"value": tokens / sec, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{sample_chains} of {wl.N} chains x T={wl.T}, fwd+bwd, oracle FP32 "
                      f"(oracle/bayes_oracle.c, OpenMP over chains), median of {len(times)} run(s); "
                      f"tok/s = chains*T/H / seconds"}


def measure_fp32_peak(dev) -> dict:
    """FP32 FMA rate of this GPU at its current clocks (library probe kernel)."""
    import torch
    from bayes_ssm import _capi

    blocks, iters = 148 * 8, 4096
    out = torch.empty(blocks * 256, device=dev)
    sp = torch.cuda.current_stream(dev).cuda_stream
    flops = 0
    for _ in range(2):
        flops = _capi.fma_probe(out, blocks, iters, sp)
    best = float("inf")
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        _capi.fma_probe(out, blocks, iters, sp)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    return {"tflops": flops / (best / 1e3) / 1e12, "ms": best,
            "how": f"bssm_debug_fma_probe: {blocks} CTAs x 256 threads x 8 independent FMA chains x "
                   f"{8 * iters} steps, best of 5 CUDA-event timings, right before the warm-up"}


def parity_sample(wl: Workload, inp, y, grads, rank, count=16) -> dict:
    """Check sampled chains of the last timed step against the FP64 oracle
    (outside the timed region; the oracle is the checker only)."""
    import numpy as np
    import torch
    from oracle import oracle

    n = inp["k"].shape[0]
    rng = np.random.default_rng(77 + rank)
    fixed = [0, 33, n // 2, n - 1]
    idx = sorted(set(fixed) | set(int(x) for x in rng.choice(n, size=count - len(fixed), replace=False)))
    sel = torch.tensor(idx, dtype=torch.long, device=inp["k"].device)

    def np64(x):
        return x.index_select(0, sel).double().cpu().numpy()

    names = ("k", "v", "q", "a", "p", "r")
    arrs = [np64(inp[x]) for x in names]
    ry, _, _ = oracle.forward(*arrs, None, None, floor=FLOOR)
    rg = oracle.backward(*arrs, None, None, np64(inp["gy"]), None, None, floor=FLOOR)

    def rel(a, b):
        return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))

    errs = {"y": rel(np64(y), ry)}
    for x in names:
        errs["grad_" + x] = rel(np64(grads[x]), rg[x])
    tol = {x: (4e-3 if x in ("grad_k", "grad_v", "grad_q") else 1e-5) for x in errs}
    ok = all(math.isfinite(errs[x]) and errs[x] <= tol[x] for x in errs)
    return {"ok": ok, "chains": len(idx), "rel_l2": errs, "tolerance": tol}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", choices=tuple(WORKLOADS) + ("5",), default="3")
    ap.add_argument("--batch", type=int, default=256, help="config 5: sequences per GPU")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-api", action="store_true")
    ap.add_argument("--chains", type=int, default=None,
                    help="chains per GPU (default: the config's share of B*H; smaller for profiling)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.config == "5":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "config": "5", "unavailable":
                                  "the six-layer trainer's reference arm needs the reference's GPU stack "
                                  "(Inductor/Triton components); only the recurrence has a CPU port"}), flush=True)
            return
        run_trainer(args, world, rank, local_rank)
        return
    wl = WORKLOADS[args.config]
    if args.impl == "reference":
        run_reference(args, wl, rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    import bayes_ssm
    from bayes_ssm import _capi

    D, M, T, CHUNK = wl.D, wl.M, wl.T, wl.CHUNK
    n = args.chains if args.chains is not None else wl.shard(world)
    fp32_peak = measure_fp32_peak(dev)
    inp = make_inputs(wl, n, 100 + rank, dev)
    nb = (T + CHUNK - 1) // CHUNK
    f32 = dict(device=dev, dtype=torch.float32)
    out = torch.empty(n, T, M, **f32)
    mt = torch.empty(n, D, M, **f32)
    pt = torch.empty(n, D, D, **f32)
    bm = torch.empty(n, nb + 1, D, M, **f32)
    bc = torch.empty(n, nb + 1, D, D, **f32)
    grads = dict(k=torch.empty_like(inp["k"]), q=torch.empty_like(inp["q"]), v=torch.empty_like(inp["v"]),
                 a=torch.empty(n, T, D, **f32), p=torch.empty(n, T, **f32), r=torch.empty(n, T, **f32))
    # replay states: saved by the forward every 4 tokens inside each chunk, so
    # the backward needs no phase-A recomputation and no workspace
    rs_bytes = _capi.replay_states_bytes(D, M, n, T, CHUNK)
    rs = torch.empty(max(rs_bytes // 4, 1), device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    io = _capi.BSSM_BF16

    def fwd():
        _capi.forward_chunked(D, M, io, False, inp["k"], inp["v"], inp["q"], inp["a"], inp["p"],
                              inp["r"], None, None, out, mt, pt, bm, bc, n, T, CHUNK, FLOOR, sp,
                              replay_states=rs)

    def bwd():
        _capi.backward_chunked(D, M, io, False, True, False, inp["k"], inp["v"], inp["q"], inp["a"],
                               inp["p"], inp["r"], None, None, bm, bc, inp["gy"], None, None, grads["k"],
                               grads["v"], grads["q"], grads["a"], grads["p"], grads["r"], None, None, None, 0,
                               n, T, CHUNK, FLOOR, sp, replay_states=rs)

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        families = {}
        for _ in range(args.warmup):
            fwd()
            families["forward"] = _capi.last_family()
            bwd()
            families["backward"] = _capi.last_family()
        _capi.stream_status(sp)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clocks.mark_start()
        start.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            fwd()
            ev[i][1].record(stream)
            bwd()
            ev[i][2].record(stream)
        stop.record(stream)
        torch.cuda.synchronize()
        clocks.mark_end()
    # raises if a bounded in-kernel wait gave up during the timed steps
    _capi.stream_status(sp)
    if world > 1:
        dist.barrier()
    total_ms = start.elapsed_time(stop)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps
    step_ms = total_ms / args.steps
    t = torch.tensor([step_ms, fwd_ms, bwd_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms, fwd_ms, bwd_ms = (float(x) for x in t.tolist())
    chains_total = n * world
    tokens = chains_total // wl.H  # a token of the workload carries H chains
    value = tokens * T / (step_ms / 1e3)
    clk = clocks.summary()

    parity = None
    if not args.no_parity:
        parity = parity_sample(wl, inp, out, grads, rank)
        ok = torch.tensor([0.0 if parity["ok"] else 1.0], device=dev)
        if world > 1:
            dist.all_reduce(ok, op=dist.ReduceOp.MAX)
        parity["ok_all_ranks"] = bool(ok.item() == 0.0)

    api = None if args.no_api else measure_api(args, wl, dev, world, bayes_ssm, inp, n)
    e2e = None
    if not args.no_e2e:
        del rs, bm, bc
        torch.cuda.empty_cache()
        e2e = measure_e2e(args, wl, dev, rank, world, bayes_ssm, n)

    if rank == 0:
        hbm_peak, peak_kind = _peaks()
        chain_steps = n * T
        bwd_gbs = chain_steps * wl.bwd_bytes / (bwd_ms / 1e3) / 1e9
        bwd_tflops = chain_steps * wl.bwd_flops / (bwd_ms / 1e3) / 1e12
        fwd_gbs = chain_steps * wl.fwd_bytes / (fwd_ms / 1e3) / 1e9
        fwd_tflops = chain_steps * wl.fwd_flops / (fwd_ms / 1e3) / 1e12
        step_tflops = chain_steps * wl.step_flops / (step_ms / 1e3) / 1e12
        step_gbs = chain_steps * (wl.fwd_bytes + wl.bwd_bytes) / (step_ms / 1e3) / 1e9
        fp32 = fp32_peak["tflops"]
        key = f"{args.config}:{wl.dominant.split(' ')[0]}"
        rec, rec_src = _captured_traffic(key)
        traffic = None
        if rec is not None:  # captured for all B*H chains; traffic grows with the chains
            traffic = int(rec["dram_bytes_per_full_launch"] * n / wl.N)
        binding = "fp32" if bwd_tflops / fp32 >= bwd_gbs / hbm_peak else "hbm"
        roofline = {
            "kernel": wl.dominant,
            "bound": binding,
            "achieved": round(bwd_tflops if binding == "fp32" else bwd_gbs, 2),
            "peak": round(fp32 if binding == "fp32" else hbm_peak, 2),
            "unit": "TFLOP/s" if binding == "fp32" else "GB/s",
            "frac": round(bwd_tflops / fp32 if binding == "fp32" else bwd_gbs / hbm_peak, 4),
            "peak_source": ("measured live: " + fp32_peak["how"]) if binding == "fp32"
            else f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
            "traffic": traffic,
            "traffic_source": rec_src if traffic is not None else f"null: {rec_src}",
            "algorithmic_flops_per_launch": chain_steps * wl.bwd_flops,
            "algorithmic_bytes_per_launch": chain_steps * wl.bwd_bytes,
            "fp32": {"achieved": round(bwd_tflops, 2), "peak": round(fp32, 2), "unit": "TFLOP/s",
                     "frac": round(bwd_tflops / fp32, 4), "peak_source": "measured live (FMA probe)",
                     "nominal_peak": round(148 * 128 * 2 * 1.965e9 / 1e12, 1)},
            "hbm": {"achieved": round(bwd_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                    "frac": round(bwd_gbs / hbm_peak, 4), "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)"},
            "forward_kernel": {"ms": round(fwd_ms, 4), "GB/s": round(fwd_gbs, 1),
                               "TFLOP/s": round(fwd_tflops, 2), "fp32_frac": round(fwd_tflops / fp32, 4),
                               "hbm_frac": round(fwd_gbs / hbm_peak, 4)},
            "backward_kernel": {"ms": round(bwd_ms, 4), "GB/s": round(bwd_gbs, 1),
                                "TFLOP/s": round(bwd_tflops, 2)},
            # the whole step (forward + backward) against both bounds
            "step": {"TFLOP/s": round(step_tflops, 2), "fp32_frac": round(step_tflops / fp32, 4),
                     "GB/s": round(step_gbs, 1), "hbm_frac": round(step_gbs / hbm_peak, 4),
                     "flops_per_chain_step": wl.step_flops,
                     "bytes_per_chain_step_bf16_io": wl.fwd_bytes + wl.bwd_bytes},
        }
        if rec is not None and traffic is not None:
            roofline["traffic_capture"] = {x: rec[x] for x in ("case", "command") if x in rec}
        cpu = None
        if world == 1 and not args.no_cpu:
            cpu = cpu_baseline_measure(wl, steps=3, warmup=0)
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
            "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": wl.config(world, n),
            "value_is": "whole-job tok/s summed over all GPUs (the metric name's per-GPU figure is "
                        "value / n_gpus)",
            "per_gpu_value": round(value / world, 1),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "api": api,
            "parity_checked": bool(parity is not None and parity["ok_all_ranks"]), "parity": parity,
            "gpu_launches": 2 * args.steps * world, "kernel_families": families,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _api_step(bayes_ssm, d, chunk):
    leaves = {x: d[x].requires_grad_(True) for x in ("k", "v", "q", "a", "p", "r")}
    y, _, _ = bayes_ssm.bayesian_layer(leaves["k"], leaves["v"], leaves["q"], transition_diagonals=leaves["a"],
                                       process_variances=leaves["p"], observation_variances=leaves["r"],
                                       chunk_length=chunk, optimized=True)
    loss = y.square().sum()
    loss.backward()
    return y.detach(), loss.detach(), {x: leaves[x].grad for x in leaves}


def measure_api(args, wl, dev, world, bayes_ssm, inp, n):
    """Public API fwd + bwd on device-resident inputs: the kernels plus the
    API's validation passes, status checks and allocations."""
    import torch

    steps = max(3, min(args.steps, 20))
    base = {x: inp[x].detach() for x in ("k", "v", "q", "a", "p", "r")}

    def one():
        _api_step(bayes_ssm, {x: base[x].detach() for x in base}, wl.CHUNK)

    for _ in range(2):
        one()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        one()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    return {"value": round(n * world // wl.H * wl.T / (ms / 1e3), 1), "unit": UNIT, "ms_per_step": round(ms, 3),
            "steps": steps,
            "path": "bayes_ssm.bayesian_layer(optimized=True) + loss.backward() on device-resident inputs "
                    "(validation passes, stream-status checks and allocations included)"}


def measure_e2e(args, wl, dev, rank, world, bayes_ssm, n):
    """Public API (bayesian_layer + autograd) with host buffers: every step
    copies its inputs in from pinned host memory and copies the readouts, the
    loss and all six gradients out to pinned host memory.  Copies run on their
    own streams, one step ahead / behind the compute (PCIe is full duplex)."""
    import torch

    names = ("k", "v", "q", "a", "p", "r")
    made = make_inputs(wl, n, 100 + rank, dev)  # generated on the device, then moved to the host
    host = {x: made[x].cpu().pin_memory() for x in names}
    del made
    h2d = sum(host[x].numel() * host[x].element_size() for x in names)
    outs = {"y": torch.empty(n, wl.T, wl.M, dtype=torch.float32).pin_memory(),
            "loss": torch.empty((), dtype=torch.float32).pin_memory()}
    for x in names:
        outs["g" + x] = torch.empty_like(host[x]).pin_memory()
    d2h = sum(v.numel() * v.element_size() for v in outs.values())
    steps = max(3, min(args.steps, 10))
    compute = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def upload():
        with torch.cuda.stream(s_in):
            d = {x: host[x].to(dev, non_blocking=True) for x in names}
            ev = torch.cuda.Event()
            ev.record(s_in)
        return d, ev

    def run(count):
        nxt = upload()
        for i in range(count):
            d, ev = nxt
            compute.wait_event(ev)
            for x in names:
                d[x].record_stream(compute)
            if i + 1 < count:
                nxt = upload()  # the next step's inputs cross while this one computes
            y, loss, g = _api_step(bayes_ssm, d, wl.CHUNK)
            done = torch.cuda.Event()
            done.record(compute)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                for tns in (y, loss, *g.values()):
                    tns.record_stream(s_out)
                outs["y"].copy_(y, non_blocking=True)
                outs["loss"].copy_(loss, non_blocking=True)
                for x in names:
                    outs["g" + x].copy_(g[x], non_blocking=True)
        s_out.synchronize()

    run(2)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(compute)
    run(steps)
    done = torch.cuda.Event()
    done.record(s_out)
    compute.wait_event(done)
    e.record(compute)
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    return {"value": round(n * world // wl.H * wl.T / (ms / 1e3), 1), "unit": UNIT,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": round(ms, 3),
            "steps": steps,
            "path": "bayes_ssm.bayesian_layer(optimized=True) + loss.backward(); pinned host inputs copied "
                    "H2D every step; readouts, loss and all six gradients copied D2H every step; copies on "
                    "side streams overlapping the neighbouring steps' compute"}


TRAIN_METRIC = "six-layer LM training tok/s (B256/GPU x T512, BF16, NCCL DDP; BASELINE config 5)"


def run_trainer(args, world, rank, local_rank) -> None:
    """the six-layer ~101.94 M-parameter hybrid LM
    (bayes_ssm.six_layer, the reference's example/train_6layer.py model) --
    one training step = H2D of the step's token batch from pinned host
    memory, forward, cross-entropy, backward with the DDP gradient all-reduce
    over NCCL, clip, fused AdamW, and the loss read back; synthetic uniform
    tokens; time = max over ranks of CUDA-event time."""
    import torch
    import torch.distributed as dist
    from torch.nn.parallel import DistributedDataParallel as DDP

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    from bayes_ssm import _capi
    from bayes_ssm.six_layer import SixLayerLM, make_optimizer, parameter_count, train_step

    vocab, seq, batch = 32_000, 512, args.batch
    torch.manual_seed(123)
    model = SixLayerLM(vocab, 512, 64, 4, 8448, chunk_length=64, dtype=torch.bfloat16, device=dev)
    params = parameter_count(model)
    if world > 1:
        model = DDP(model, device_ids=[local_rank], output_device=local_rank, broadcast_buffers=False,
                    gradient_as_bucket_view=True, bucket_cap_mb=25.0, find_unused_parameters=False)
    opt = make_optimizer(model)
    g = torch.Generator().manual_seed(124 + rank)
    steps_total = args.warmup + args.steps
    host = torch.randint(vocab, (steps_total, batch, seq + 1), generator=g).pin_memory()
    loss_host = torch.empty(steps_total, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)

    def step(i):
        tok = host[i].to(dev, non_blocking=True)
        loss = train_step(model, opt, tok[:, :-1], tok[:, 1:], vocab_size=vocab, grad_clip=1.0)
        loss_host[i].copy_(loss, non_blocking=True)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    _capi.stream_status(stream.cuda_stream)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        clocks.mark_start()
        start.record(stream)
        for i in range(args.warmup, steps_total):
            step(i)
        stop.record(stream)
        torch.cuda.synchronize()
        clocks.mark_end()
    _capi.stream_status(stream.cuda_stream)
    ms = start.elapsed_time(stop) / args.steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = batch * seq * world / (ms / 1e3)
    # the gradient all-reduce DDP runs each step, timed alone (bucket-sized
    # pieces of the BF16 gradient), to name what the multi-GPU curve pays
    comm = None
    if world > 1:
        buf = torch.empty(params, device=dev, dtype=torch.bfloat16)
        bucket = 25 * 2 ** 20 // 2

        def allreduce():
            for off in range(0, params, bucket):
                dist.all_reduce(buf[off:off + bucket])

        for _ in range(3):
            allreduce()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(5):
            allreduce()
        e.record(stream)
        torch.cuda.synchronize()
        ar_ms = s.elapsed_time(e) / 5
        tt = torch.tensor([ar_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ar_ms = float(tt.item())
        nbytes = params * 2
        comm = {"gradient_bytes": nbytes, "allreduce_ms_alone": round(ar_ms, 3),
                "bus_GBps": round(2 * (world - 1) / world * nbytes / (ar_ms / 1e3) / 1e9, 1),
                "share_of_step_if_unoverlapped": round(ar_ms / ms, 4),
                "how": "NCCL all_reduce of the BF16 gradient in 25 MiB buckets (DDP's bucket size), timed alone"}
    losses = loss_host.tolist()
    if rank == 0:
        print(json.dumps({
            "metric": TRAIN_METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic uniform tokens",
            "config": {"workload": "six-layer hybrid LM training step (BASELINE config 5)", "model": "SixLayerLM",
                       "parameters": params, "global_batch": batch * world, "seq_len": seq, "vocab": vocab,
                       "blocks": "bayes,bayes,gqa,bayes,bayes,gqa", "chunk": 64, "optimizer": "AdamW(0.9,0.95) "
                       "fused, clip 1.0", "parallelism": f"dp{world} (NCCL DDP, 25 MiB buckets)" if world > 1
                       else "dp1"},
            "value_is": "whole-job tok/s summed over all GPUs", "per_gpu_value": round(value / world, 1),
            "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": batch * (seq + 1) * 8,
                    "d2h_bytes_per_step": 4, "note": "the timed step itself copies its tokens in and its loss out"},
            "communication": comm, "loss_first_last": [losses[0], losses[-1]],
            "peak_allocated_gib": round(torch.cuda.max_memory_allocated(dev) / 2 ** 30, 2),
            "gpu_launches": None, "clocks": clocks.summary(),
            "reference_gb300": {"value": 434215.0, "n_gpus": 2, "note": "example/results/"
                                "gb300_6layer_bayes_paper_d8_fused.json (CUDA graph + compiled GQA/SwiGLU)"},
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
