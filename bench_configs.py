"""Secondary measurements for the other benchmark configurations (the
headline, config 3, is ``bench.py``).

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

* ``--config envelope``: the BayesianMixer prologue at config 3's mixer
  shape (B256 T512, 64 heads, key_dim 8, head_dim 8: a BF16 projection of
  2,176 channels per token) -> the recurrence's inputs, forward + backward,
  through the C ABI with FP32 outputs (the reference's state boundary) and
  with BF16 k/q/v (the headline recurrence's input dtype), beside the eager
  PyTorch op chain of the reference; and the readout epilogue (FP32 reads,
  BF16 gate and output) beside its PyTorch form; bytes-roofline fractions
  against the measured HBM copy bandwidth.

* ``--config mixer``: the whole BayesianMixer layer (``bayes_ssm.mixer``) at
  config 3's shape (B256 T512, width 512, 64 heads, key_dim 8, BF16
  parameters and activations): RMSNorm, projection GEMMs, the fused prologue,
  the recurrence, the fused readout, the output GEMM; forward + backward of a
  mean-square loss, with the FP32 state boundary (the reference's default) and
  with BF16 k/q/v, beside the same layer with the PyTorch op chains for the
  prologue and readout.

* ``--config envelope-profile``: the prologue and readout kernels alone at an
  eighth of that shape (B32), untimed: the case their ncu captures run on.

* ``--config rotation``: rotation dynamics (damped 2-D rotations per key pair,
  per-pair process noise) at config 3's shape (B256 T512 H64 D8 M8, chunk 64,
  FP32), forward + backward of a readout loss through the public
  ``bayesian_layer(rotation_radii=, rotation_angles=, optimized=True)``, beside
  the dense PyTorch path on the same GPU (the reference's only path for these
  dynamics), with 8 chains checked against that path in FP64 on the CPU.

* ``--config rotation-profile``: the rotation kernels alone at an eighth of
  that shape (B32, 2,048 chains), untimed: the case their ncu captures run on.

* ``--config d64-profile``: the (64, 64) kernels on 296 chains (B37 T512 H8,
  one wave at two CTAs per SM), untimed: the case their ncu captures run on.

* ``--config refcuda``: the reference's own CUDA kernels on the same GPU --
  catid/bayes-ssm installed unmodified into ``baseline/_ref`` (``pip install
  --target``), its D8 extension JIT-built by its own loader
  (``bayes_ssm/fused_cuda.py:23-55``, ``-O3``, here for sm_100 with
  ``TORCH_CUDA_ARCH_LIST=10.0`` and ``TORCH_EXTENSIONS_DIR`` inside
  ``baseline/_ref``) -- at config 3 (B256 T512 H64 D8 M8, chunk 64): the
  public ``bayesian_layer(optimized=True)`` fwd+bwd (BF16 inputs promoted to
  FP32, as the reference does) and its ``fused_diagonal_bayesian`` boundary
  on FP32 inputs, with a sample of chains checked against the CPU oracle.
  This process imports the reference's package in place of this one (both
  are named ``bayes_ssm``).

Each run prints one JSON line.  Inputs are seeded synthetic tensors with
the distributions of the reference's mixer; timing is CUDA events after
warm-up.
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


def envelope(steps: int, warmup: int) -> dict:
    import torch
    from bayes_ssm import _capi
    from bayes_ssm.envelope import paper_prologue_torch
    b, t, h, d, hd = 256, 512, 64, 8, 8
    sw, w = h * d, h * hd
    c, aux = 2 * sw + w, sw + 2 * h
    pch = c + aux
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(b, t, pch, generator=g, device=dev).to(torch.bfloat16)
    wt = torch.randn(c, 4, generator=g, device=dev) * 0.5
    bias = torch.randn(aux, generator=g, device=dev) * 0.1
    n = b * h
    f32 = dict(device=dev, dtype=torch.float32)
    sp = torch.cuda.current_stream().cuda_stream
    ws = torch.empty(_capi.envelope_partial_floats(b, t, h, d, hd), **f32)
    gx = torch.empty_like(x)
    gw, gb = torch.empty(c, 4, **f32), torch.empty(aux, **f32)
    gd, gp, go = (torch.randn(n, t, d, generator=g, device=dev), torch.randn(n, t, generator=g, device=dev),
                  torch.randn(n, t, generator=g, device=dev))
    dec, proc, obs = torch.empty(n, t, d, **f32), torch.empty(n, t, **f32), torch.empty(n, t, **f32)
    hbm = _peak_hbm()
    res = {}
    for name, odt in (("f32_out", torch.float32), ("bf16_out", torch.bfloat16)):
        code = _capi.BSSM_F32 if odt == torch.float32 else _capi.BSSM_BF16
        k, q = torch.empty(n, t, d, device=dev, dtype=odt), torch.empty(n, t, d, device=dev, dtype=odt)
        v = torch.empty(n, t, hd, device=dev, dtype=odt)
        gk, gq, gv = torch.randn_like(k), torch.randn_like(q), torch.randn_like(v)

        def fwd():
            _capi.envelope_prologue(x, _capi.BSSM_BF16, b, t, h, d, hd, pch, wt, bias, k, q, v, code, dec, proc,
                                    obs, sp)

        def bwd():
            _capi.envelope_prologue_backward(x, _capi.BSSM_BF16, b, t, h, d, hd, pch, wt, bias, gk, gq, gv, code,
                                             gd, gp, go, gx, pch, gw, gb, ws, sp)

        es = k.element_size()
        tok = b * t
        fwd_bytes = tok * (pch * 2 + (2 * sw + w) * es + sw * 4 + 2 * h * 4)
        bwd_bytes = tok * (pch * 2 + (2 * sw + w) * es + sw * 4 + 2 * h * 4 + pch * 2)
        ms_f, ms_b = _time(fwd, steps, warmup), _time(bwd, steps, warmup)
        res[name] = {"forward_ms": round(ms_f, 4), "backward_ms": round(ms_b, 4),
                     "forward_GBps": round(fwd_bytes / ms_f / 1e6, 1), "backward_GBps": round(bwd_bytes / ms_b / 1e6, 1),
                     "forward_frac": round(fwd_bytes / ms_f / 1e6 / hbm, 3),
                     "backward_frac": round(bwd_bytes / ms_b / 1e6 / hbm, 3),
                     "algorithmic_bytes": {"forward": fwd_bytes, "backward": bwd_bytes}}
    xe = x.detach().clone().requires_grad_()
    we = wt.reshape(c, 1, 4).detach().clone().requires_grad_()
    be = bias.detach().clone().requires_grad_()

    def eager():
        outs = paper_prologue_torch(xe, we, be, heads=h, key_dim=d, head_dim=hd)
        ups = [torch.ones_like(o) for o in outs]
        torch.autograd.grad(outs, (xe, we, be), ups)

    ms_e = _time(eager, max(3, steps // 4), warmup)
    # readout epilogue: FP32 reads [B*H, T, hd], BF16 gate -> BF16 [B, T, W]
    from bayes_ssm.envelope import read_epilogue_torch
    read = torch.randn(n, t, hd, generator=g, device=dev)
    gate = torch.randn(b, t, w, generator=g, device=dev).to(torch.bfloat16)
    nw = torch.rand(hd, generator=g, device=dev) + 0.5
    eps = float(torch.finfo(torch.bfloat16).eps)
    out = torch.empty(b, t, w, device=dev, dtype=torch.bfloat16)
    gout = torch.randn_like(out)
    g_read, g_gate = torch.empty_like(read), torch.empty_like(gate)
    g_nw = torch.empty(hd, **f32)
    ews = torch.empty(_capi.envelope_epilogue_partial_floats(b, t, h, hd), **f32)

    def efwd():
        _capi.envelope_epilogue(read, _capi.BSSM_F32, gate, _capi.BSSM_BF16, w, nw, eps, b, t, h, hd, out, sp)

    def ebwd():
        _capi.envelope_epilogue_backward(read, _capi.BSSM_F32, gate, _capi.BSSM_BF16, w, nw, eps, b, t, h, hd, gout,
                                         g_read, g_gate, w, g_nw, ews, sp)

    tok = b * t
    e_fwd_bytes = tok * w * (4 + 2 + 2)
    e_bwd_bytes = tok * w * (4 + 2 + 2 + 4 + 2)
    ms_ef, ms_eb = _time(efwd, steps, warmup), _time(ebwd, steps, warmup)
    re_, ge_, we_ = (z.detach().clone().requires_grad_() for z in (read, gate, nw))

    def eager_epi():
        o = read_epilogue_torch(re_, ge_, we_, heads=h, eps=eps)
        torch.autograd.grad(o, (re_, ge_, we_), gout)

    ms_ee = _time(eager_epi, max(3, steps // 4), warmup)
    # input RMSNorm over the width: BF16 [B*T, W]
    xr = torch.randn(b * t, w, generator=g, device=dev).to(torch.bfloat16)
    nrm = torch.rand(w, generator=g, device=dev) + 0.5
    xo, gxo = torch.empty_like(xr), torch.empty_like(xr)
    gyn = torch.randn_like(xr)
    gnw = torch.empty(w, **f32)
    nws = torch.empty(_capi.rms_norm_partial_floats(b * t, w), **f32)
    ms_nf = _time(lambda: _capi.rms_norm(xr, _capi.BSSM_BF16, b * t, w, nrm, eps, xo, sp), steps, warmup)
    ms_nb = _time(lambda: _capi.rms_norm_backward(xr, _capi.BSSM_BF16, b * t, w, nrm, eps, gyn, gxo, gnw, nws, sp),
                  steps, warmup)
    n_bytes_f, n_bytes_b = b * t * w * 2 * 2, b * t * w * 2 * 3
    norm = {"forward_ms": round(ms_nf, 4), "backward_ms": round(ms_nb, 4),
            "forward_frac": round(n_bytes_f / ms_nf / 1e6 / hbm, 3),
            "backward_frac": round(n_bytes_b / ms_nb / 1e6 / hbm, 3)}
    epilogue = {"forward_ms": round(ms_ef, 4), "backward_ms": round(ms_eb, 4),
                "forward_frac": round(e_fwd_bytes / ms_ef / 1e6 / hbm, 3),
                "backward_frac": round(e_bwd_bytes / ms_eb / 1e6 / hbm, 3),
                "algorithmic_bytes": {"forward": e_fwd_bytes, "backward": e_bwd_bytes},
                "eager_torch_fwd_bwd_ms": round(ms_ee, 4)}
    return {"config": "envelope", "workload": "BayesianMixer prologue, B256 T512 H64 D8 head_dim 8 "
            "(BF16 projection, 2,176 channels), fwd + bwd", "metric": "ms per fwd+bwd", "unit": "ms",
            "kernel": res, "eager_torch_fwd_bwd_ms": round(ms_e, 4), "readout_epilogue": epilogue, "input_rms_norm": norm,
            "speedup_f32_out": round(ms_e / (res["f32_out"]["forward_ms"] + res["f32_out"]["backward_ms"]), 2),
            "hbm_peak_GBps": hbm, "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)",
            "steps": steps, "warmup": warmup, "data": "synthetic"}


def mixer(steps: int, warmup: int) -> dict:
    import torch
    from bayes_ssm.mixer import BayesianMixer
    b, t, width, heads, d = 256, 512, 512, 64, 8
    torch.manual_seed(5)
    x = torch.randn(b, t, width, device="cuda", dtype=torch.bfloat16)
    res = {}
    for name, bf16_io, fused in (("fused_fp32_state_io", False, True), ("fused_bf16_state_io", True, True),
                                 ("torch_envelope_fp32_state_io", False, False)):
        m = BayesianMixer(width, heads, key_dim=d, chunk_length=64, bf16_state_io=bf16_io, fused_envelope=fused,
                          dtype=torch.bfloat16, device="cuda")

        def step():
            m.zero_grad(set_to_none=True)
            y = m(x)
            y.float().square().mean().backward()

        ms = _time(step, max(3, steps // 2), warmup)
        res[name] = {"ms_per_step": round(ms, 4), "tok_per_s": round(b * t / (ms / 1e3), 1)}
        del m
        torch.cuda.empty_cache()
    return {"config": "mixer", "workload": "BayesianMixer layer fwd + bwd, B256 T512 width 512, 64 heads, key_dim 8, "
            "BF16 (config 3's mixer; GEMMs and input RMSNorm by PyTorch)", "metric": "tok/s/GPU", "unit": "tok/s",
            "results": res, "steps": max(3, steps // 2), "warmup": warmup, "data": "synthetic"}


def d64(steps: int, warmup: int) -> dict:
    """Key dim 64 x value dim 64 (the reference trainer's layer at 8 heads of
    width 64): B256 T512 H8 -> 2,048 chains, chunk 64, FP32 inputs, forward +
    backward with all dynamics gradients of a readout loss, through the C ABI;
    8 chains checked against the FP64 oracle."""
    import numpy as np
    import torch
    import torch.nn.functional as F
    from bayes_ssm import _capi
    from oracle import oracle
    b, t, h, d, m, chunk, floor = 256, 512, 8, 64, 64, 64, 1e-6
    n = b * h
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(64)

    def rn(*shape):
        return torch.randn(*shape, generator=g, device=dev)

    kk = F.normalize(rn(n, t, d), dim=-1)
    qq = F.normalize(rn(n, t, d), dim=-1)
    vv = rn(n, t, m) / math.sqrt(m)
    aa = torch.sigmoid(2.0 + rn(n, t, d))
    pp = F.softplus(-4.0 + rn(n, t))
    rr = F.softplus(rn(n, t)) + 1e-4
    gy = rn(n, t, m) / math.sqrt(m)
    nb = (t + chunk - 1) // chunk
    f32 = dict(device=dev, dtype=torch.float32)
    out = torch.empty(n, t, m, **f32)
    mt, pt = torch.empty(n, d, m, **f32), torch.empty(n, d, d, **f32)
    bm, bc = torch.empty(n, nb + 1, d, m, **f32), torch.empty(n, nb + 1, d, d, **f32)
    gk, gq, gv = torch.empty_like(kk), torch.empty_like(qq), torch.empty_like(vv)
    gd, gp, gr = torch.empty(n, t, d, **f32), torch.empty(n, t, **f32), torch.empty(n, t, **f32)
    wsb = _capi.workspace_bytes(d, m, n, t, chunk)
    ws = torch.empty(max(wsb, 1), device=dev, dtype=torch.uint8)
    sp = torch.cuda.current_stream().cuda_stream
    io = _capi.BSSM_F32

    def fwd():
        _capi.forward_chunked(d, m, io, False, kk, vv, qq, aa, pp, rr, None, None, out, mt, pt, bm, bc, n, t, chunk,
                              floor, sp)

    def bwd():
        _capi.backward_chunked(d, m, io, False, True, False, kk, vv, qq, aa, pp, rr, None, None, bm, bc, gy, None,
                               None, gk, gv, gq, gd, gp, gr, None, None, ws, wsb, n, t, chunk, floor, sp)

    ms_f = _time(fwd, steps, warmup)
    ms_b = _time(bwd, steps, warmup)
    _capi.stream_status(sp)
    idx = torch.tensor([0, 1, n // 2, n - 1, 100, 777, 1500, 2000], device=dev)

    def np64(x):
        return x.index_select(0, idx).double().cpu().numpy()

    arrs = [np64(x) for x in (kk, vv, qq, aa, pp, rr)]
    ry, _, _ = oracle.forward(*arrs, None, None, floor=floor)
    rg = oracle.backward(*arrs, None, None, np64(gy), None, None, floor=floor)

    def rel(x, want):
        return float(np.linalg.norm(np64(x) - want) / np.linalg.norm(want))

    parity = {"y": rel(out, ry)}
    for name, gr_ in zip("kvqapr", (gk, gv, gq, gd, gp, gr)):
        parity["grad_" + name] = rel(gr_, rg[name])
    chain_steps = n * t
    flops = chain_steps * (26 * d * d + 34 * d * m + 30 * d + 3 * m + 2)
    ms = ms_f + ms_b
    return {"config": "d64", "workload": "D64 M64, B256 T512 H8 -> 2,048 chains, chunk 64, FP32, fwd + bwd "
            "(all dynamics gradients, readout loss)", "metric": "tok/s/GPU", "unit": "tok/s",
            "value": round(b * t / (ms / 1e3), 1), "ms_per_step": round(ms, 4), "forward_ms": round(ms_f, 4),
            "backward_ms": round(ms_b, 4), "step_tflops": round(flops / (ms / 1e3) / 1e12, 2),
            "workspace_bytes": wsb, "parity_vs_oracle_rel_l2": parity, "parity_chains": int(idx.numel()),
            "family": _capi.last_family(), "steps": steps, "warmup": warmup, "data": "synthetic"}


def rotation(steps: int, warmup: int) -> dict:
    """Rotation dynamics at config 3's shape through the public API (see the
    module doc): the kernels, the dense path on the GPU, and parity."""
    import numpy as np
    import torch
    import torch.nn.functional as F
    import bayes_ssm
    b, t, h, d, m, chunk = 256, 512, 64, 8, 8, 64
    n, j = b * h, d // 2
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(8)

    def rn(*shape):
        return torch.randn(*shape, generator=g, device=dev)

    base = dict(k=F.normalize(rn(n, t, d), dim=-1), v=rn(n, t, m) / math.sqrt(m), q=F.normalize(rn(n, t, d), dim=-1),
                radii=0.85 + 0.2 * torch.rand(n, t, j, generator=g, device=dev), angles=0.4 * rn(n, t, j),
                p=F.softplus(-3.0 + rn(n, t, j)), r=F.softplus(rn(n, t)) + 1e-3)
    gy = rn(n, t, m) / math.sqrt(m)

    def step(inp, optimized, out=None):
        leaves = {x: v.detach().requires_grad_() for x, v in inp.items()}
        y, _, _ = bayes_ssm.bayesian_layer(leaves["k"], leaves["v"], leaves["q"], rotation_radii=leaves["radii"],
                                           rotation_angles=leaves["angles"], process_variances=leaves["p"],
                                           observation_variances=leaves["r"], chunk_length=chunk,
                                           optimized=optimized)
        grads = torch.autograd.grad(y, list(leaves.values()), gy)
        if out is not None:
            out["y"] = y.detach()
            out.update({x: gr_ for x, gr_ in zip(leaves, grads)})

    ms_k = _time(lambda: step(base, True), steps, warmup)
    ms_dense = _time(lambda: step(base, False), 1, 1)
    got = {}
    step(base, True, got)
    idx = torch.tensor([0, 1, n // 2, n - 1, 77, 4321, 9000, 16000], device=dev)
    sub = {x: v.index_select(0, idx).double().cpu() for x, v in base.items()}
    gy_sub = gy.index_select(0, idx).double().cpu()
    leaves = {x: v.clone().requires_grad_() for x, v in sub.items()}
    y0, _, _ = bayes_ssm.bayesian_layer(leaves["k"], leaves["v"], leaves["q"], rotation_radii=leaves["radii"],
                                        rotation_angles=leaves["angles"], process_variances=leaves["p"],
                                        observation_variances=leaves["r"], chunk_length=chunk, optimized=False)
    want = dict(zip(leaves, torch.autograd.grad(y0, list(leaves.values()), gy_sub)))
    want["y"] = y0.detach()

    def rel(x):
        a = got[x].index_select(0, idx).double().cpu().numpy()
        e = want[x].numpy()
        return float(np.linalg.norm(a - e) / np.linalg.norm(e))

    parity = {x: rel(x) for x in ("y", "k", "v", "q", "radii", "angles", "p", "r")}
    return {"config": "rotation", "workload": "rotation dynamics, B256 T512 H64 D8 M8, chunk 64, FP32, fwd + bwd "
            "through bayesian_layer(optimized=True), readout gradient given", "metric": "tok/s/GPU", "unit": "tok/s",
            "value": round(b * t / (ms_k / 1e3), 1), "ms_per_step": round(ms_k, 4),
            "dense_torch_gpu_ms_per_step": round(ms_dense, 2), "speedup_vs_dense": round(ms_dense / ms_k, 1),
            "parity_vs_dense_fp64_rel_l2": parity, "parity_chains": int(idx.numel()), "steps": steps,
            "warmup": warmup, "data": "synthetic"}


def rotation_profile(steps: int, warmup: int) -> dict:
    """The rotation kernels through the C ABI on 2,048 chains (B32 T512 H64 D8
    M8, chunk 64, FP32): ``steps`` forward + backward pairs, untimed -- the
    small case an ncu capture of ``rot_forward`` / ``rot_backward`` runs on."""
    import torch
    import torch.nn.functional as F
    from bayes_ssm import _capi
    b, t, h, d, m, chunk, floor = 32, 512, 64, 8, 8, 64, 1e-6
    n, j = b * h, d // 2
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(8)

    def rn(*shape):
        return torch.randn(*shape, generator=g, device=dev)

    k, q, v = F.normalize(rn(n, t, d), dim=-1), F.normalize(rn(n, t, d), dim=-1), rn(n, t, m) / math.sqrt(m)
    rho = 0.85 + 0.1 * torch.rand(n, t, j, generator=g, device=dev)
    ang = 0.4 * rn(n, t, j)
    cs, sn = rho * ang.cos(), rho * ang.sin()
    pp, rr = F.softplus(-3.0 + rn(n, t, j)), F.softplus(rn(n, t)) + 1e-3
    gy = rn(n, t, m) / math.sqrt(m)
    nb = (t + chunk - 1) // chunk
    f32 = dict(device=dev, dtype=torch.float32)
    out, mt, pt = torch.empty(n, t, m, **f32), torch.empty(n, d, m, **f32), torch.empty(n, d, d, **f32)
    bm, bc = torch.empty(n, nb + 1, d, m, **f32), torch.empty(n, nb + 1, d, d, **f32)
    gk, gv, gq = torch.empty_like(k), torch.empty_like(v), torch.empty_like(q)
    gc, gs, gp = (torch.empty(n, t, j, **f32) for _ in range(3))
    gr = torch.empty(n, t, **f32)
    wsb = _capi.rotation_workspace_bytes(d, m, n, t, chunk)
    ws = torch.empty(max(wsb, 1), device=dev, dtype=torch.uint8)
    sp = torch.cuda.current_stream().cuda_stream
    for _ in range(steps):
        _capi.rotation_forward(d, m, k, v, q, cs, sn, pp, rr, None, None, out, mt, pt, bm, bc, n, t, chunk, floor, sp)
        _capi.rotation_backward(d, m, False, k, v, q, cs, sn, pp, rr, bm, bc, gy, None, None, gk, gv, gq, gc, gs,
                                gp, gr, None, None, ws, wsb, n, t, chunk, floor, sp)
    torch.cuda.synchronize()
    _capi.stream_status(sp)
    return {"config": "rotation-profile", "workload": "rotation fwd + bwd, B32 T512 H64 D8 M8 = 2,048 chains "
            "(profiling case)", "launches": 2 * steps, "timed": False}


def d64_profile(steps: int, warmup: int) -> dict:
    """The (64, 64) forward and backward on 296 chains (B37 T512 H8, chunk 64,
    FP32): ``steps`` forward + backward pairs, untimed -- the small case an ncu
    capture of ``d64_forward`` / ``d64_backward`` runs on (one wave at two CTAs
    per SM, as every wave of the full launch)."""
    import torch
    import torch.nn.functional as F
    from bayes_ssm import _capi
    b, t, h, d, m, chunk, floor = 37, 512, 8, 64, 64, 64, 1e-6
    n = b * h
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(64)

    def rn(*shape):
        return torch.randn(*shape, generator=g, device=dev)

    kk, qq = F.normalize(rn(n, t, d), dim=-1), F.normalize(rn(n, t, d), dim=-1)
    vv, aa = rn(n, t, m) / math.sqrt(m), torch.sigmoid(2.0 + rn(n, t, d))
    pp, rr = F.softplus(-4.0 + rn(n, t)), F.softplus(rn(n, t)) + 1e-4
    gy = rn(n, t, m) / math.sqrt(m)
    nb = (t + chunk - 1) // chunk
    f32 = dict(device=dev, dtype=torch.float32)
    out = torch.empty(n, t, m, **f32)
    mt, pt = torch.empty(n, d, m, **f32), torch.empty(n, d, d, **f32)
    bm, bc = torch.empty(n, nb + 1, d, m, **f32), torch.empty(n, nb + 1, d, d, **f32)
    gk, gq, gv = torch.empty_like(kk), torch.empty_like(qq), torch.empty_like(vv)
    gd, gp, gr = torch.empty(n, t, d, **f32), torch.empty(n, t, **f32), torch.empty(n, t, **f32)
    wsb = _capi.workspace_bytes(d, m, n, t, chunk)
    ws = torch.empty(max(wsb, 1), device=dev, dtype=torch.uint8)
    sp = torch.cuda.current_stream().cuda_stream
    for _ in range(steps):
        _capi.forward_chunked(d, m, _capi.BSSM_F32, False, kk, vv, qq, aa, pp, rr, None, None, out, mt, pt, bm, bc,
                              n, t, chunk, floor, sp)
        _capi.backward_chunked(d, m, _capi.BSSM_F32, False, True, False, kk, vv, qq, aa, pp, rr, None, None, bm, bc,
                               gy, None, None, gk, gv, gq, gd, gp, gr, None, None, ws, wsb, n, t, chunk, floor, sp)
    torch.cuda.synchronize()
    _capi.stream_status(sp)
    return {"config": "d64-profile", "workload": "D64 M64 fwd + bwd, B37 T512 H8 = 296 chains (profiling case)",
            "launches": 2 * steps, "timed": False}


def envelope_profile(steps: int, warmup: int) -> dict:
    """The prologue kernels alone at an eighth of config 3's mixer shape
    (B32 T512, 64 heads, key_dim 8, head_dim 8, BF16 projection, FP32
    outputs): ``steps`` forward + backward pairs, untimed -- the small case an
    ncu capture of ``prologue_kernel`` / ``prologue_backward_kernel`` runs on."""
    import torch
    from bayes_ssm import _capi
    b, t, h, d, hd = 32, 512, 64, 8, 8
    sw, w = h * d, h * hd
    c, aux = 2 * sw + w, sw + 2 * h
    pch = c + aux
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(b, t, pch, generator=g, device=dev).to(torch.bfloat16)
    wt = torch.randn(c, 4, generator=g, device=dev) * 0.5
    bias = torch.randn(aux, generator=g, device=dev) * 0.1
    n = b * h
    f32 = dict(device=dev, dtype=torch.float32)
    k, q, v = torch.empty(n, t, d, **f32), torch.empty(n, t, d, **f32), torch.empty(n, t, hd, **f32)
    dec, proc, obs = torch.empty(n, t, d, **f32), torch.empty(n, t, **f32), torch.empty(n, t, **f32)
    gk, gq, gv = torch.randn_like(k), torch.randn_like(q), torch.randn_like(v)
    gd, gp, go = torch.randn_like(dec), torch.randn_like(proc), torch.randn_like(obs)
    gx = torch.empty_like(x)
    gw, gb = torch.empty(c, 4, **f32), torch.empty(aux, **f32)
    ws = torch.empty(_capi.envelope_partial_floats(b, t, h, d, hd), **f32)
    sp = torch.cuda.current_stream().cuda_stream
    for _ in range(steps):
        _capi.envelope_prologue(x, _capi.BSSM_BF16, b, t, h, d, hd, pch, wt, bias, k, q, v, _capi.BSSM_F32, dec,
                                proc, obs, sp)
        _capi.envelope_prologue_backward(x, _capi.BSSM_BF16, b, t, h, d, hd, pch, wt, bias, gk, gq, gv,
                                         _capi.BSSM_F32, gd, gp, go, gx, pch, gw, gb, ws, sp)
    # the readout at the same shape (FP32 reads, BF16 gate), through the public wrapper
    from bayes_ssm.envelope import read_epilogue
    read = torch.randn(n, t, hd, generator=g, device=dev).requires_grad_()
    gate = torch.randn(b, t, w, generator=g, device=dev).to(torch.bfloat16).requires_grad_()
    nw = (torch.rand(hd, generator=g, device=dev) + 0.5).requires_grad_()
    up = torch.randn(b, t, w, generator=g, device=dev).to(torch.bfloat16)
    for _ in range(steps):
        torch.autograd.grad(read_epilogue(read, gate, nw, heads=h), (read, gate, nw), up)
    torch.cuda.synchronize()
    return {"config": "envelope-profile", "workload": "prologue and readout fwd + bwd, B32 T512 H64 D8 head_dim 8 "
            "(profiling case)", "launches": 4 * steps, "timed": False}


def refcuda64(steps: int, warmup: int) -> dict:
    """The reference's D64 kernels at the ``--config d64`` workload."""
    return refcuda(steps, warmup, key_dim=64)


def refcuda(steps: int, warmup: int, key_dim: int = 8) -> dict:
    """The reference's CUDA path at config 3 on this GPU (see the module doc);
    ``key_dim=64`` runs the D64 M64 workload of ``--config d64`` instead."""
    import os
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "bayes_ssm" / "fused_cuda.py").exists():
        return {"config": "refcuda", "unavailable": "baseline/_ref holds no reference install"}
    os.environ.setdefault("TORCH_EXTENSIONS_DIR", str(ref / "_ext"))
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"  # B200 (sm_100a); the prebuilt extension matches it
    sys.path[:] = [p for p in sys.path if not p.endswith("bayes-ssm_b200")]
    sys.path.insert(0, str(ref))
    import time

    import numpy as np
    import torch
    import torch.nn.functional as F

    import bayes_ssm as ref_pkg
    from bayes_ssm import fused_cuda as ref_fc
    assert str(ref) in ref_pkg.__file__, ref_pkg.__file__
    from oracle import oracle

    if key_dim == 64:
        b, t, h, d, m, chunk, floor = 256, 512, 8, 64, 64, 64, 1e-6
    else:
        b, t, h, d, m, chunk, floor = 256, 512, 64, 8, 8, 64, 1e-6
    n = b * h
    dev = torch.device("cuda")
    t0 = time.perf_counter()
    ext = ref_fc._load_extension(d)
    build_s = time.perf_counter() - t0
    if ext is None:
        return {"config": "refcuda", "unavailable": f"reference extension did not load: {ref_fc._LOAD_ERRORS.get(d)}"}
    g = torch.Generator(device=dev).manual_seed(3)

    def rn(*shape):
        return torch.randn(*shape, generator=g, device=dev)

    k = F.normalize(rn(n, t, d), dim=-1).to(torch.bfloat16)
    q = F.normalize(rn(n, t, d), dim=-1).to(torch.bfloat16)
    v = (rn(n, t, m) / math.sqrt(m)).to(torch.bfloat16)
    a = torch.sigmoid(2.0 + rn(n, t, d))
    p = F.softplus(-4.0 + rn(n, t))
    r = F.softplus(rn(n, t)) + 1e-4
    gy = rn(n, t, m) / math.sqrt(m)

    def api_step():
        leaves = [x.detach().requires_grad_() for x in (k, v, q, a, p, r)]
        y, _, _ = ref_pkg.bayesian_layer(leaves[0], leaves[1], leaves[2], transition_diagonals=leaves[3],
                                         process_variances=leaves[4], observation_variances=leaves[5],
                                         chunk_length=chunk, optimized=True)
        y.backward(gy)
        return y, [x.grad for x in leaves]

    kf, vf, qf = k.float(), v.float(), q.float()
    m0 = torch.zeros(n, d, m, device=dev)
    c0 = torch.eye(d, device=dev).expand(n, d, d).contiguous()

    def boundary_step():
        leaves = [x.detach().requires_grad_() for x in (kf, vf, qf, a, p, r)]
        out = ref_fc.fused_diagonal_bayesian(*leaves, m0, c0, chunk_length=chunk, denominator_floor=floor)
        out[0].backward(gy)
        return out[0]

    y, grads = api_step()
    torch.cuda.synchronize()
    if boundary_step() is None:
        return {"config": "refcuda", "unavailable": "reference fused boundary declined the inputs"}
    # the reference's own GPU outputs on a sample of chains vs the FP64 oracle
    rng = np.random.default_rng(0)
    idx = torch.tensor(sorted(set([0, n // 2, n - 1]) | set(int(i) for i in rng.choice(n, 13, replace=False))),
                       device=dev)

    def np64(x):
        return x.index_select(0, idx).double().cpu().numpy()

    arrs = [np64(x) for x in (k, v, q, a, p, r)]
    ry, _, _ = oracle.forward(*arrs, None, None, floor=floor)
    rg = oracle.backward(*arrs, None, None, np64(gy), None, None, floor=floor)

    def rel(x, want):
        return float(np.linalg.norm(np64(x) - want) / np.linalg.norm(want))

    parity = {"y": rel(y.detach(), ry)}
    for name, gr in zip("kvqapr", grads):
        parity["grad_" + name] = rel(gr, rg[name])
    ms_api = _time(api_step, steps, warmup)
    ms_bnd = _time(boundary_step, steps, warmup)
    tok = b * t
    return {"config": "refcuda" if key_dim == 8 else "refcuda64",
            "workload": "reference CUDA kernels (catid/bayes-ssm, unmodified, JIT-built for sm_100) at "
            + ("config 3: B256 T512 H64 D8 M8" if key_dim == 8 else "B256 T512 H8 D64 M64")
            + ", chunk 64, fwd + bwd, readout loss gradient",
            "metric": "tok/s/GPU", "unit": "tok/s",
            "api": {"ms_per_step": round(ms_api, 3), "tok_per_s": round(tok / (ms_api / 1e3), 1),
                    "path": "reference bayesian_layer(optimized=True) + backward, BF16 k/q/v promoted to FP32"},
            "boundary": {"ms_per_step": round(ms_bnd, 3), "tok_per_s": round(tok / (ms_bnd / 1e3), 1),
                         "path": "reference fused_cuda.fused_diagonal_bayesian on FP32 inputs + backward"},
            "parity_vs_oracle_rel_l2": parity, "parity_chains": int(idx.numel()),
            "extension_load_s": round(build_s, 1), "arch_list": os.environ.get("TORCH_CUDA_ARCH_LIST"),
            "steps": steps, "warmup": warmup, "data": "synthetic"}


def _peak_hbm() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, ValueError, KeyError):
        return 6650.0


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=("2", "4", "d64", "d64-profile", "envelope", "envelope-profile", "mixer",
                                         "refcuda", "refcuda64", "rotation", "rotation-profile"), required=True)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    fn = {"2": config2, "4": config4, "d64": d64, "d64-profile": d64_profile, "envelope": envelope,
          "envelope-profile": envelope_profile,
          "mixer": mixer, "refcuda": refcuda, "refcuda64": refcuda64, "rotation": rotation,
          "rotation-profile": rotation_profile}[args.config]
    print(json.dumps(fn(args.steps, max(3, args.warmup))), flush=True)


if __name__ == "__main__":
    main()
