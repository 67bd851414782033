"""Secondary measurements for the other configurations named in the survey's
measurement plan (the headline, config 3, is ``bench.py``).

* ``--config 2``: the static associative scan (B4 T64 H8 -> 32 chains,
  D = M = 16), forward only.  It is latency-bound (2,048 chain-tokens), so
  it reports microseconds per call: through the API
  (``associative_static_bayesian_cuda``, which includes the reference's
  host-side input validation), through the C ABI alone, and for the eager
  PyTorch information-form path (``associative_static_bayesian``: cumulative
  sums and batched Cholesky on the same GPU).  No roofline fraction.
* ``--config 4``: D2 M8, B256 T2048, 256 heads -> 65,536 chains, chunk 64,
  BF16 k/q/v: forward + backward (all dynamics gradients, readout loss)
  through the C ABI, as ``bench.py`` does for config 3, in tok/s.

Each run prints one JSON line.  Inputs are seeded synthetic tensors with
the survey's distributions; timing is CUDA events after warm-up.
"""
from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "bayes-ssm_b200"))


def _time(fn, steps: int, warmup: int) -> float:
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps


def config2(steps: int, warmup: int) -> dict:
    import torch
    import torch.nn.functional as F
    import bayes_ssm
    from bayes_ssm import _capi
    g = torch.Generator().manual_seed(2)
    b, t, h, d, m = 4, 64, 8, 16, 16
    k = (torch.randn(b, h, t, d, generator=g) / math.sqrt(m)).cuda()
    q = (torch.randn(b, h, t, d, generator=g) / math.sqrt(m)).cuda()
    v = torch.randn(b, h, t, m, generator=g).cuda()
    r2 = (F.softplus(torch.randn(b, h, t, generator=g)) + 1e-2).cuda()
    kern = lambda: bayes_ssm.associative_static_bayesian_cuda(k, v, q, observation_variances=r2)
    eager = lambda: bayes_ssm.associative_static_bayesian(k, v, q, observation_variances=r2)
    yk, _, _ = kern()
    ye, _, _ = eager()
    rel = float((yk - ye).norm() / ye.norm())
    us_k = 1e3 * _time(kern, steps, warmup)
    us_e = 1e3 * _time(eager, steps, warmup)
    n = b * h
    kc, vc, qc = (x.reshape(n, t, -1).contiguous() for x in (k, v, q))
    rc = r2.reshape(n, t).contiguous()
    f32 = dict(device=k.device, dtype=torch.float32)
    out, mf, cf = torch.empty(n, t, m, **f32), torch.empty(n, d, m, **f32), torch.empty(n, d, d, **f32)
    status = torch.zeros(1, device=k.device, dtype=torch.int32)
    sp = torch.cuda.current_stream().cuda_stream
    raw = lambda: _capi.assoc_scan(d, m, kc, vc, qc, rc, None, None, out, mf, cf, status, n, t, 1e-6, sp)
    us_raw = 1e3 * _time(raw, steps, warmup)
    return {"config": "2", "workload": "static associative scan, B4 T64 H8 D16 M16 (32 chains), forward",
            "metric": "latency per call", "unit": "us", "kernel_only_us": round(us_raw, 2),
            "api_us": round(us_k, 2), "eager_torch_us": round(us_e, 2),
            "speedup_api_vs_eager": round(us_e / us_k, 2), "rel_l2_kernel_vs_eager": rel,
            "steps": steps, "warmup": warmup, "note": "latency-bound (2,048 chain-tokens); no roofline fraction"}


def config4(steps: int, warmup: int) -> dict:
    import torch
    import torch.nn.functional as F
    from bayes_ssm import _capi
    b, t, h, d, m, chunk, floor = 256, 2048, 256, 2, 8, 64, 1e-6
    n = b * h
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(4)
    f32 = dict(device=dev, dtype=torch.float32)

    def gen(*shape):
        return torch.randn(*shape, generator=g, device=dev)

    # generated on the device in slices to bound the FP32 temporaries
    def make(shape, fn, dtype):
        out = torch.empty(*shape, device=dev, dtype=dtype)
        step = 8192
        for i in range(0, shape[0], step):
            j = min(shape[0], i + step)
            out[i:j] = fn((j - i, *shape[1:])).to(dtype)
        return out

    kk = make((n, t, d), lambda s: F.normalize(gen(*s), dim=-1), torch.bfloat16)
    qq = make((n, t, d), lambda s: F.normalize(gen(*s), dim=-1), torch.bfloat16)
    vv = make((n, t, m), lambda s: gen(*s) / math.sqrt(m), torch.bfloat16)
    aa = make((n, t, d), lambda s: torch.sigmoid(2.0 + gen(*s)), torch.float32)
    pp = make((n, t), lambda s: F.softplus(-4.0 + gen(*s)), torch.float32)
    rr = make((n, t), lambda s: F.softplus(gen(*s)) + 1e-4, torch.float32)
    gy = make((n, t, m), lambda s: gen(*s) / math.sqrt(m), torch.float32)
    nb = (t + chunk - 1) // chunk
    out = torch.empty(n, t, m, **f32)
    mt, pt = torch.empty(n, d, m, **f32), torch.empty(n, d, d, **f32)
    bm, bc = torch.empty(n, nb + 1, d, m, **f32), torch.empty(n, nb + 1, d, d, **f32)
    gk, gq, gv = torch.empty_like(kk), torch.empty_like(qq), torch.empty_like(vv)
    gd, gp, gr = torch.empty(n, t, d, **f32), torch.empty(n, t, **f32), torch.empty(n, t, **f32)
    rs = torch.empty(max(_capi.replay_states_bytes(d, m, n, t, chunk) // 4, 1), **f32)
    sp = torch.cuda.current_stream().cuda_stream
    io = _capi.BSSM_BF16

    def fwd():
        _capi.forward_chunked(d, m, io, False, kk, vv, qq, aa, pp, rr, None, None, out, mt, pt, bm, bc,
                              n, t, chunk, floor, sp, replay_states=rs)

    def bwd():
        _capi.backward_chunked(d, m, io, False, True, False, kk, vv, qq, aa, pp, rr, None, None, bm, bc,
                               gy, None, None, gk, gv, gq, gd, gp, gr, None, None, None, 0, n, t, chunk,
                               floor, sp, replay_states=rs)

    ms_f = _time(fwd, steps, warmup)
    fam_f = _capi.last_family()
    ms_b = _time(bwd, steps, warmup)
    fam_b = _capi.last_family()
    ms = ms_f + ms_b
    return {"config": "4", "workload": "D2 M8, B256 T2048, 256 heads -> 65,536 chains, chunk 64, fwd + bwd",
            "metric": "tok/s/GPU", "unit": "tok/s", "value": round(b * t / (ms / 1e3), 1),
            "ms_per_step": round(ms, 4), "forward_ms": round(ms_f, 4), "backward_ms": round(ms_b, 4),
            "families": {"forward": fam_f, "backward": fam_b}, "steps": steps, "warmup": warmup,
            "io_dtype": "bf16 k/q/v, fp32 decay/noise/state", "data": "synthetic"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=("2", "4"), required=True)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    fn = config2 if args.config == "2" else config4
    print(json.dumps(fn(args.steps, max(3, args.warmup))), flush=True)


if __name__ == "__main__":
    main()
