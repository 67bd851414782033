"""Host side of the sm_100a static associative scan (``csrc/bssm_assoc_scan.cu``)."""
from __future__ import annotations

import contextlib

import torch
from torch import Tensor

from . import _capi
from .bayesian_layer import _is_cuda_graph_capturing

MAX_KEY_DIM = 32
MAX_VALUE_DIM = 256
MAX_CHAINS_PER_LAUNCH = 65535
_NO_SWITCH = contextlib.nullcontext()  # the inputs' device is already current


def assoc_scan_cuda(keys: Tensor, values: Tensor, queries: Tensor, r2: Tensor, mean0, cov0, *,
                    batch, denominator_floor: float):
    """Run the kernel on validated, promoted inputs; returns (reads, M_T, P_T).

    The scan is forward only (as the reference's); inputs that require
    gradients are rejected rather than silently detached.
    """
    t, d = keys.shape[-2:]
    m = values.shape[-1]
    if d > MAX_KEY_DIM or m > MAX_VALUE_DIM:
        raise NotImplementedError(
            f"associative_static_bayesian_cuda supports key_dim <= {MAX_KEY_DIM} and value_dim <= "
            f"{MAX_VALUE_DIM} (got {d}, {m}); use associative_static_bayesian for larger states")
    if keys.dtype != torch.float32:
        raise TypeError("associative_static_bayesian_cuda computes in float32; pass float32/bf16/fp16/fp8 inputs")
    if torch.is_grad_enabled() and any(x is not None and x.requires_grad
                                       for x in (keys, values, queries, r2, mean0, cov0)):
        raise RuntimeError("associative_static_bayesian_cuda is forward-only; call it under torch.no_grad() "
                           "or use bayesian_layer(..., optimized=True) for gradients")
    n = 1
    for s in batch:
        n *= int(s)
    dev = keys.device
    f32 = torch.float32

    def chains(x, tail):
        if x is None:
            return None
        if x.dtype == f32 and x.is_contiguous() and tuple(x.shape) == (*batch, *tail):
            return x.view(n, *tail)  # already one row per chain: no expand / copy
        return x.to(f32).expand(*batch, *tail).reshape(n, *tail).contiguous()

    k, v, q = chains(keys, (t, d)), chains(values, (t, m)), chains(queries, (t, d))
    r = chains(r2, (t,))
    m0, c0 = chains(mean0, (d, m)), chains(cov0, (d, d))
    out = torch.empty(n, t, m, device=dev, dtype=f32)
    mt = torch.empty(n, d, m, device=dev, dtype=f32)
    pt = torch.empty(n, d, d, device=dev, dtype=f32)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev) if dev.index != torch.cuda.current_device() else _NO_SWITCH:
        for lo in range(0, n, MAX_CHAINS_PER_LAUNCH):
            hi = min(n, lo + MAX_CHAINS_PER_LAUNCH)
            sl = slice(lo, hi)
            _capi.assoc_scan(d, m, k[sl], v[sl], q[sl], r[sl], None if m0 is None else m0[sl],
                             None if c0 is None else c0[sl], out[sl], mt[sl], pt[sl], status, hi - lo,
                             t, denominator_floor, stream)
    if not _is_cuda_graph_capturing(keys):
        code = int(status.item())
        if code & 2:
            raise ValueError("associative_static_bayesian requires finite observation_variances "
                             "greater than or equal to denominator_floor")
        if code & 1:
            raise torch.linalg.LinAlgError(
                "associative_static_bayesian_cuda: a precision matrix is not positive definite")
    return (out.reshape(*batch, t, m), mt.reshape(*batch, d, m), pt.reshape(*batch, d, d))
