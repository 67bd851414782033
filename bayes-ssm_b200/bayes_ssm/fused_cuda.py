"""Autograd boundary over the sm_100a chunked recurrence kernels.

Mirrors catid/bayes-ssm ``bayes_ssm/fused_cuda.py`` (``fused_diagonal_bayesian``
:325-388, ``_ChunkedBayesianFunction`` :58-322): the forward saves the inputs
and the chunk-boundary states; the backward replays each chunk from its
boundary and runs the reverse adjoint -- here in a single kernel launch.

Differences from the reference boundary, all deliberate:

* the kernels are reached through a C ABI (``_capi``), not a JIT pybind
  module, and a missing library raises instead of returning ``None``;
* BF16 keys/values/queries are consumed directly (widened in registers) and
  their gradients are produced in BF16, which is exactly what the reference's
  ``.to(float32)`` promotion followed by its autograd cast-back computes;
* gradients of the initial mean and covariance are supported (the reference
  routes those callers to its dense path).
"""
from __future__ import annotations

import os
from typing import Optional

import torch
from torch import Tensor

from . import _capi

SUPPORTED_DIMS = _capi.SUPPORTED


def _io_dtype(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return _capi.BSSM_F32
    if dtype == torch.bfloat16:
        return _capi.BSSM_BF16
    raise TypeError(f"fused Bayesian kernels take float32 or bfloat16 keys/values/queries, got {dtype}")


def _save_replay_states() -> bool:
    return os.environ.get("BAYES_SSM_SAVE_REPLAY_STATES", "1") != "0"


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _status(device: torch.device) -> None:
    """Raise if a bounded wait inside a kernel gave up (``_capi.WaitTimeout``).

    The thread-per-chain kernels never hang on their own copies: a wait that
    runs out is counted on the device and the kernel finishes with wrong
    outputs.  This synchronises the stream and turns such a count into an
    exception, so no call returns outputs or gradients after a give-up.  It is
    skipped while a CUDA graph is being captured (no host synchronisation is
    legal there); call ``_capi.stream_status`` after replaying a graph.
    """
    if torch.cuda.is_current_stream_capturing():
        return
    _capi.stream_status(_stream(device))


class _ChunkedBayesianFunction(torch.autograd.Function):
    """Exact chunked recurrence: forward kernel + single-launch replay backward."""

    @staticmethod
    def forward(ctx, keys, values, queries, decay, process, observation, initial_mean,
                initial_covariance, chunk_length: int, denominator_floor: float,
                fixed_dynamics: bool, pending_checks=None):
        n, t, d = keys.shape
        m = values.shape[-1]
        dev = keys.device
        nb = (t + chunk_length - 1) // chunk_length
        f32 = dict(device=dev, dtype=torch.float32)
        out = torch.empty(n, t, m, **f32)
        mean_final = torch.empty(n, d, m, **f32)
        cov_final = torch.empty(n, d, d, **f32)
        bmean = torch.empty(n, nb + 1, d, m, **f32)
        bcov = torch.empty(n, nb + 1, d, d, **f32)
        # Replay states: the forward also saves the state every 4 tokens inside
        # each chunk so the backward replays 4-token spans without first
        # recomputing the chunk (memory N*T/4*(D*M+D*D)*4 bytes; set
        # BAYES_SSM_SAVE_REPLAY_STATES=0 to trade it for that recomputation).
        rs = None
        if _save_replay_states() and any(ctx.needs_input_grad[:8]):
            rs_bytes = _capi.replay_states_bytes(d, m, n, t, int(chunk_length))
            if rs_bytes:
                rs = torch.empty(rs_bytes // 4, **f32)
        with torch.cuda.device(dev):
            _capi.forward_chunked(d, m, _io_dtype(keys.dtype), fixed_dynamics, keys, values, queries,
                                  None if fixed_dynamics else decay,
                                  None if fixed_dynamics else process,
                                  None if fixed_dynamics else observation,
                                  initial_mean, initial_covariance, out, mean_final, cov_final,
                                  bmean, bcov, n, t, int(chunk_length), denominator_floor,
                                  _stream(dev), replay_states=rs)
            if pending_checks is not None:
                # the caller's input checks, read back after the kernel was
                # enqueued: one synchronisation covers both; a failing check
                # raises and the outputs are dropped
                pending_checks.flush()
            _status(dev)
        ctx.save_for_backward(keys, values, queries, decay, process, observation, bmean, bcov, rs)
        ctx.chunk_length = int(chunk_length)
        ctx.denominator_floor = float(denominator_floor)
        ctx.fixed_dynamics = bool(fixed_dynamics)
        ctx.set_materialize_grads(False)
        return out, mean_final, cov_final

    @staticmethod
    def backward(ctx, grad_out, grad_mean, grad_cov):
        keys, values, queries, decay, process, observation, bmean, bcov, rs = ctx.saved_tensors
        n, t, d = keys.shape
        m = values.shape[-1]
        dev = keys.device
        needs = ctx.needs_input_grad
        need_dyn = bool(needs[3] or needs[4] or needs[5])
        need_init = bool(needs[6] or needs[7])
        gy = None if grad_out is None else _aligned(grad_out.contiguous().float())
        gmf = None if grad_mean is None else _aligned(grad_mean.contiguous().float())
        gcf = None if grad_cov is None else _aligned(grad_cov.contiguous().float())
        gk = torch.empty_like(keys)
        gv = torch.empty_like(values)
        gq = torch.empty_like(queries)
        f32 = dict(device=dev, dtype=torch.float32)
        gd = torch.empty(n, t, d, **f32) if need_dyn else None
        gp = torch.empty(n, t, **f32) if need_dyn else None
        gr = torch.empty(n, t, **f32) if need_dyn else None
        gm0 = torch.empty(n, d, m, **f32) if need_init else None
        gc0 = torch.empty(n, d, d, **f32) if need_init else None
        ws_bytes = 0 if rs is not None else _capi.workspace_bytes(d, m, n, t, ctx.chunk_length)
        ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
        fixed = ctx.fixed_dynamics
        with torch.cuda.device(dev):
            _capi.backward_chunked(d, m, _io_dtype(keys.dtype), fixed, need_dyn, need_init, keys,
                                   values, queries, None if fixed else decay,
                                   None if fixed else process, None if fixed else observation,
                                   None, None, bmean, bcov, gy, gmf, gcf, gk, gv, gq, gd, gp, gr,
                                   gm0, gc0, ws, ws_bytes, n, t, ctx.chunk_length,
                                   ctx.denominator_floor, _stream(dev), replay_states=rs)
            _status(dev)
        return (gk if needs[0] else None, gv if needs[1] else None, gq if needs[2] else None,
                gd if needs[3] else None, gp if needs[4] else None, gr if needs[5] else None,
                gm0 if needs[6] else None, gc0 if needs[7] else None, None, None, None, None)


def _aligned(x: Tensor) -> Tensor:
    """The kernels need 16-byte aligned tensors; re-home an offset view."""
    return x if x.data_ptr() % 16 == 0 else x.clone(memory_format=torch.contiguous_format)


def kernel_supports(key_dim: int, value_dim: int) -> bool:
    return (key_dim, value_dim) in SUPPORTED_DIMS


def fused_diagonal_bayesian(
    keys: Tensor,
    values: Tensor,
    queries: Tensor,
    decay: Tensor,
    process: Tensor,
    observation: Tensor,
    initial_mean: Optional[Tensor],
    initial_covariance: Optional[Tensor],
    *,
    chunk_length: int,
    denominator_floor: float,
    fixed_dynamics: bool = False,
    _pending_checks=None,
) -> tuple[Tensor, Tensor, Tensor]:
    """Run the chunked CUDA recurrence on ``[N,T,*]`` inputs.

    keys/queries ``[N,T,D]``, values ``[N,T,M]`` (float32, or all bfloat16);
    decay ``[N,T,D]``, process/observation ``[N,T]``, initial mean ``[N,D,M]``
    and covariance ``[N,D,D]`` (float32, broadcast views allowed).  Returns
    ``(readouts [N,T,M], final_mean, final_covariance)`` in float32.

    Unlike the reference (which returns ``None`` so the caller can fall back),
    an unsupported shape or dtype raises ``ValueError``/``TypeError`` and a
    missing library raises ``_capi.ExtensionUnavailable``.
    """
    if keys.device.type != "cuda":
        raise ValueError("fused_diagonal_bayesian requires CUDA tensors")
    if keys.ndim != 3 or values.ndim != 3 or queries.ndim != 3:
        raise ValueError("fused_diagonal_bayesian expects [N,T,D] keys/queries and [N,T,M] values")
    n, t, d = keys.shape
    m = values.shape[-1]
    if not kernel_supports(d, m):
        raise ValueError(f"no kernel for key_dim={d}, value_dim={m}; supported: {SUPPORTED_DIMS}")
    if queries.shape != keys.shape or values.shape[:2] != keys.shape[:2]:
        raise ValueError("keys/queries/values batch and time dimensions must match")
    if not (keys.dtype == values.dtype == queries.dtype) or keys.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("keys, values and queries must all be float32 or all bfloat16")
    if not isinstance(chunk_length, int) or chunk_length <= 0:
        raise ValueError("chunk_length must be a positive integer")
    f32 = torch.float32
    dev = keys.device

    def prep(x, shape):
        if x is None:
            return None
        return _aligned(x.to(device=dev, dtype=f32).expand(shape).contiguous())

    decay = prep(decay, (n, t, d))
    process = prep(process, (n, t))
    observation = prep(observation, (n, t))
    initial_mean = prep(initial_mean, (n, d, m))
    initial_covariance = prep(initial_covariance, (n, d, d))
    if decay is None or process is None or observation is None:
        if not fixed_dynamics:
            raise ValueError("decay, process and observation are required unless fixed_dynamics=True")
        ones = torch.ones((), device=dev, dtype=f32)
        decay = ones.expand(n, t, d) if decay is None else decay
        process = ones.expand(n, t) if process is None else process
        observation = ones.expand(n, t) if observation is None else observation
    if d == 64 and keys.dtype != f32:  # the (64, 64) kernels read float32 projections only
        keys, values, queries = keys.to(f32), values.to(f32), queries.to(f32)
    keys = _aligned(keys.contiguous())
    values = _aligned(values.contiguous())
    queries = _aligned(queries.contiguous())
    return _ChunkedBayesianFunction.apply(
        keys, values, queries, decay, process, observation, initial_mean, initial_covariance,
        int(chunk_length), float(denominator_floor), bool(fixed_dynamics), _pending_checks)


__all__ = ["fused_diagonal_bayesian", "kernel_supports", "SUPPORTED_DIMS"]
