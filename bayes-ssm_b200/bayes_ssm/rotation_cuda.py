"""Autograd boundary over the rotation-dynamics kernels (``bssm_rotation.cu``).

The reference runs rotation dynamics only through its dense PyTorch path
(``bayes_ssm/bayesian_layer.py:254-340``: ``make_rotation_dynamics`` builds
block-diagonal damped rotations, ``make_rotation_process_covariances`` the
per-pair noise ``diag(l^2, 0)``).  Here the same model runs on the GPU with
the 2 x 2 block structure used directly.  The kernels take the rotation as
``cos = rho cos(theta)`` and ``sin = rho sin(theta)`` per key pair and return
their gradients; ``bayesian_layer`` forms them from the radii and angles with
the reference's own operations, so autograd carries the gradients on to the
radii (through the same clamps) and the angles.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _capi

SUPPORTED = ((2, 8), (4, 8), (8, 8))


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _RotationFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, keys, values, queries, cosines, sines, process, observation, initial_mean,
                initial_covariance, chunk_length: int, denominator_floor: float, pending_checks=None):
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
        with torch.cuda.device(dev):
            _capi.rotation_forward(d, m, keys, values, queries, cosines, sines, process, observation, initial_mean,
                                   initial_covariance, out, mean_final, cov_final, bmean, bcov, n, t,
                                   int(chunk_length), denominator_floor, _stream(dev))
            if pending_checks is not None:  # one read-back covers the input checks and the kernel
                pending_checks.flush()
        ctx.save_for_backward(keys, values, queries, cosines, sines, process, observation, bmean, bcov)
        ctx.chunk_length = int(chunk_length)
        ctx.denominator_floor = float(denominator_floor)
        ctx.set_materialize_grads(False)
        return out, mean_final, cov_final

    @staticmethod
    def backward(ctx, grad_out, grad_mean, grad_cov):
        keys, values, queries, cosines, sines, process, observation, bmean, bcov = ctx.saved_tensors
        n, t, d = keys.shape
        m = values.shape[-1]
        j = d // 2
        dev = keys.device
        needs = ctx.needs_input_grad
        need_init = bool(needs[7] or needs[8])
        gy = None if grad_out is None else grad_out.contiguous().float()
        gmf = None if grad_mean is None else grad_mean.contiguous().float()
        gcf = None if grad_cov is None else grad_cov.contiguous().float()
        f32 = dict(device=dev, dtype=torch.float32)
        gk, gv, gq = torch.empty_like(keys), torch.empty_like(values), torch.empty_like(queries)
        gc, gs, gp = (torch.empty(n, t, j, **f32) for _ in range(3))
        gr = torch.empty(n, t, **f32)
        gm0 = torch.empty(n, d, m, **f32) if need_init else None
        gc0 = torch.empty(n, d, d, **f32) if need_init else None
        wsb = _capi.rotation_workspace_bytes(d, m, n, t, ctx.chunk_length)
        ws = torch.empty(wsb, device=dev, dtype=torch.uint8) if wsb else None
        with torch.cuda.device(dev):
            _capi.rotation_backward(d, m, need_init, keys, values, queries, cosines, sines, process, observation,
                                    bmean, bcov, gy, gmf, gcf, gk, gv, gq, gc, gs, gp, gr, gm0, gc0, ws, wsb, n, t,
                                    ctx.chunk_length, ctx.denominator_floor, _stream(dev))
        return (gk, gv, gq, gc, gs, gp, gr, gm0 if needs[7] else None, gc0 if needs[8] else None, None, None,
                None)


class _CoefficientsFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, radii, angles):
        cosines, sines = torch.empty_like(radii), torch.empty_like(radii)
        with torch.cuda.device(radii.device):
            _capi.rotation_coefficients(radii, angles, cosines, sines, _stream(radii.device))
        ctx.save_for_backward(radii, angles)
        ctx.set_materialize_grads(False)
        return cosines, sines

    @staticmethod
    def backward(ctx, grad_cosines, grad_sines):
        radii, angles = ctx.saved_tensors
        if grad_cosines is None and grad_sines is None:
            return None, None
        gc = None if grad_cosines is None else grad_cosines.contiguous()
        gs = None if grad_sines is None else grad_sines.contiguous()
        g_radii, g_angles = torch.empty_like(radii), torch.empty_like(angles)
        with torch.cuda.device(radii.device):
            _capi.rotation_coefficients_backward(radii, angles, gc, gs, g_radii, g_angles, _stream(radii.device))
        return g_radii, g_angles


def rotation_coefficients(radii: Tensor, angles: Tensor):
    """``(rho cos(angles), rho sin(angles))`` with the reference's radius
    handling (``bayesian_layer.py``: radii clamped to [tiny, 1], then
    ``make_rotation_dynamics``' ``exp(log(radius))`` clipped at 1), in one
    kernel each way; same-shape contiguous float32 CUDA tensors."""
    return _CoefficientsFunction.apply(radii, angles)


def coefficients_apply(radii, angles) -> bool:
    """Whether :func:`rotation_coefficients` takes these tensors (else the
    caller runs the same chain as PyTorch operations)."""
    return (isinstance(radii, Tensor) and isinstance(angles, Tensor) and radii.is_cuda and angles.is_cuda
            and radii.device == angles.device and radii.dtype == angles.dtype == torch.float32
            and radii.shape == angles.shape and radii.is_contiguous() and angles.is_contiguous()
            and radii.data_ptr() % 4 == 0 and angles.data_ptr() % 4 == 0)


def rotation_bayesian(keys: Tensor, values: Tensor, queries: Tensor, cosines: Tensor, sines: Tensor,
                      process: Tensor, observation: Tensor, initial_mean, initial_covariance, *,
                      chunk_length: int, denominator_floor: float, _pending_checks=None):
    """``[N,T,*]`` float32 inputs (cosines, sines, process ``[N,T,D/2]``,
    observation ``[N,T]``) -> ``(readouts [N,T,M], final_mean, final_covariance)``."""
    n, t, d = keys.shape
    m = values.shape[-1]
    if (d, m) not in SUPPORTED:
        raise ValueError(f"no rotation kernel for key_dim={d}, value_dim={m}; supported: {SUPPORTED}")
    f32 = torch.float32

    def prep(x, shape):
        return None if x is None else x.to(dtype=f32).expand(shape).contiguous()

    j = d // 2
    return _RotationFunction.apply(
        prep(keys, (n, t, d)), prep(values, (n, t, m)), prep(queries, (n, t, d)), prep(cosines, (n, t, j)),
        prep(sines, (n, t, j)), prep(process, (n, t, j)), prep(observation, (n, t)), prep(initial_mean, (n, d, m)),
        prep(initial_covariance, (n, d, d)), int(chunk_length), float(denominator_floor), _pending_checks)


__all__ = ["rotation_bayesian", "rotation_coefficients", "SUPPORTED"]
