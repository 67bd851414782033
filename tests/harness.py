"""Shared helpers for the kernel tests: seeded inputs and raw C-ABI calls.

Inputs follow the reference's distributions: ``paper`` is the dynamic
paper-feature mixer shape (unit-norm k, q; decay sigmoid(N(2,1)); process
softplus(N(-4,1)); observation softplus(N(0,1)) + 1e-4), ``unit`` is the
reference unit test's (tests/test_bayesian_layer_diagonal.py:54-74).
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from bayes_ssm import _capi


def make_inputs(n, t, d, m, *, seed=0, dist="paper", init="identity", io_dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    if dist == "paper":
        k = F.normalize(torch.randn(n, t, d, generator=g), dim=-1)
        q = F.normalize(torch.randn(n, t, d, generator=g), dim=-1)
        v = torch.randn(n, t, m, generator=g) / math.sqrt(m)
        a = torch.sigmoid(2.0 + torch.randn(n, t, d, generator=g))
        p = F.softplus(-4.0 + torch.randn(n, t, generator=g))
        r = F.softplus(torch.randn(n, t, generator=g)) + 1e-4
    else:
        k = torch.randn(n, t, d, generator=g)
        v = torch.randn(n, t, m, generator=g)
        q = torch.randn(n, t, d, generator=g)
        a = 0.8 + 0.15 * torch.rand(n, t, d, generator=g)
        p = 0.1 + 0.2 * torch.rand(n, t, generator=g)
        r = 0.2 + torch.rand(n, t, generator=g)
    if init == "random":
        m0 = torch.randn(n, d, m, generator=g) * 0.3
        b = torch.randn(n, d, d, generator=g) / math.sqrt(d)
        p0 = torch.eye(d) + 0.5 * b @ b.transpose(-1, -2)
        p0 = 0.5 * (p0 + p0.transpose(-1, -2))
    else:
        m0 = None
        p0 = None
    k, q, v = (x.to(io_dtype) for x in (k, q, v))
    return dict(k=k, v=v, q=q, a=a.float(), p=p.float(), r=r.float(),
                M0=None if m0 is None else m0.float(), P0=None if p0 is None else p0.float())


def to_np64(x):
    return None if x is None else x.detach().float().cpu().numpy().astype(np.float64)


def io_code(dtype):
    return _capi.BSSM_BF16 if dtype == torch.bfloat16 else _capi.BSSM_F32


def cuda(x):
    return None if x is None else x.cuda().contiguous()


def capi_forward(inp, *, chunks, floor=1e-6, fixed=False, replay_states=True):
    """Forward through bssm_forward_chunked_ex (optionally saving the replay
    states the backward then reuses); returns device tensors."""
    k, v, q = cuda(inp["k"]), cuda(inp["v"]), cuda(inp["q"])
    a, p, r = cuda(inp["a"]), cuda(inp["p"]), cuda(inp["r"])
    m0, p0 = cuda(inp["M0"]), cuda(inp["P0"])
    n, t, d = k.shape
    m = v.shape[-1]
    nb = (t + chunks - 1) // chunks
    dev = k.device
    out = torch.empty(n, t, m, device=dev)
    mt = torch.empty(n, d, m, device=dev)
    pt = torch.empty(n, d, d, device=dev)
    bm = torch.empty(n, nb + 1, d, m, device=dev)
    bc = torch.empty(n, nb + 1, d, d, device=dev)
    rs = None
    if replay_states:
        nbytes = _capi.replay_states_bytes(d, m, n, t, chunks)
        rs = torch.full((nbytes // 4,), float("nan"), device=dev) if nbytes else None
    _capi.forward_chunked(d, m, io_code(k.dtype), fixed, k, v, q, None if fixed else a,
                          None if fixed else p, None if fixed else r, m0, p0, out, mt, pt, bm, bc,
                          n, t, chunks, floor, torch.cuda.current_stream().cuda_stream,
                          replay_states=rs)
    # synchronises; raises if a bounded in-kernel wait gave up
    _capi.stream_status(torch.cuda.current_stream().cuda_stream)
    return dict(y=out, MT=mt, PT=pt, bm=bm, bc=bc, rs=rs)


def capi_backward(inp, fwd, gy, gmt, gpt, *, chunks, floor=1e-6, fixed=False, need_dyn=True,
                  need_init=True):
    k, v, q = cuda(inp["k"]), cuda(inp["v"]), cuda(inp["q"])
    a, p, r = cuda(inp["a"]), cuda(inp["p"]), cuda(inp["r"])
    n, t, d = k.shape
    m = v.shape[-1]
    dev = k.device
    gk, gv, gq = torch.empty_like(k), torch.empty_like(v), torch.empty_like(q)
    gd = torch.full((n, t, d), float("nan"), device=dev) if need_dyn else None
    gp = torch.full((n, t), float("nan"), device=dev) if need_dyn else None
    gr = torch.full((n, t), float("nan"), device=dev) if need_dyn else None
    gm0 = torch.full((n, d, m), float("nan"), device=dev) if need_init else None
    gc0 = torch.full((n, d, d), float("nan"), device=dev) if need_init else None
    rs = fwd.get("rs")
    nbytes = 0 if rs is not None else _capi.workspace_bytes(d, m, n, t, chunks)
    ws = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
    _capi.backward_chunked(d, m, io_code(k.dtype), fixed, need_dyn, need_init, k, v, q,
                           None if fixed else a, None if fixed else p, None if fixed else r, None,
                           None, fwd["bm"], fwd["bc"], cuda(gy), cuda(gmt), cuda(gpt), gk, gv, gq,
                           gd, gp, gr, gm0, gc0, ws, nbytes, n, t, chunks, floor,
                           torch.cuda.current_stream().cuda_stream, replay_states=rs)
    _capi.stream_status(torch.cuda.current_stream().cuda_stream)
    return dict(k=gk, v=gv, q=gq, a=gd, p=gp, r=gr, M0=gm0, P0=gc0)


def rel_l2(actual, expected) -> float:
    a = np.asarray(actual, dtype=np.float64).ravel()
    e = np.asarray(expected, dtype=np.float64).ravel()
    den = np.linalg.norm(e)
    num = np.linalg.norm(a - e)
    if den == 0.0:
        return float(num)
    return float(num / den)


def cosine(actual, expected) -> float:
    a = np.asarray(actual, dtype=np.float64).ravel()
    e = np.asarray(expected, dtype=np.float64).ravel()
    na, ne = np.linalg.norm(a), np.linalg.norm(e)
    if na == 0.0 and ne == 0.0:
        return 1.0
    return float(a @ e / (na * ne))


def assert_parity(actual, expected, *, rel=1e-5, cos=0.99999, what=""):
    """North-star FP32 bar: relative L2 error <= rel and cosine >= cos."""
    actual = actual.detach().float().cpu().numpy() if isinstance(actual, torch.Tensor) else actual
    assert np.all(np.isfinite(actual)), f"{what}: non-finite output"
    r = rel_l2(actual, expected)
    c = cosine(actual, expected)
    assert r <= rel and c >= cos, f"{what}: rel_l2={r:.3e} (<= {rel:g}) cosine={c:.8f} (>= {cos})"
