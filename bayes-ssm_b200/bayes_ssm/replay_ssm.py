"""ReplaySSM module and the static associative scan (A = I, Q = 0).

Same API as catid/bayes-ssm ``bayes_ssm/replay_ssm.py``: ``ReplaySSM`` (:34-145),
``associative_static_bayesian`` (:155-270) and
``associative_static_bayesian_cuda`` (:276-339).

* ``ReplaySSM.forward`` calls :func:`bayesian_layer` with ``optimized=True,
  replay_ssm=True``; on CUDA with a supported shape that is the sm_100a
  chunked kernel pair, whose backward replays each chunk from its boundary
  state (the reference's CUDA replay; its own module used an Inductor replay).
* ``associative_static_bayesian`` is the information-form scan in PyTorch
  (CPU or any device): prefix sums of ``k k^T / r`` and ``k v^T / r``, a
  symmetrised Cholesky per prefix, ``M_t = Lambda_t^{-1} N_t``.
* ``associative_static_bayesian_cuda`` runs the hand-written sm_100a scan
  kernel (``csrc/bssm_assoc_scan.cu``): a blocked prefix sum of the
  information increments and a warp-per-matrix FP32 Cholesky.
"""
from __future__ import annotations

import math
from numbers import Real
from typing import Optional

import torch
from torch import Tensor, nn

from .bayesian_layer import _broadcastable, _check_finite, _validate_covariance, bayesian_layer


class ReplaySSM(nn.Module):
    """Exact dense Bayesian recurrence with chunk-replay backward."""

    def __init__(self, key_dim: int, value_dim: int, *, process_variance: float = 0.05,
                 observation_variance: float = 0.2, initial_covariance: float = 1.0,
                 chunk_length: int = 64, denominator_floor: float = 1e-6) -> None:
        super().__init__()
        if not isinstance(key_dim, int) or isinstance(key_dim, bool) or key_dim <= 0:
            raise ValueError("key_dim must be a positive integer")
        if not isinstance(value_dim, int) or isinstance(value_dim, bool) or value_dim <= 0:
            raise ValueError("value_dim must be a positive integer")
        if not isinstance(chunk_length, int) or isinstance(chunk_length, bool) or chunk_length <= 0:
            raise ValueError("chunk_length must be a positive integer")
        for name, value in (
            ("process_variance", process_variance),
            ("observation_variance", observation_variance),
            ("initial_covariance", initial_covariance),
            ("denominator_floor", denominator_floor),
        ):
            if not isinstance(value, Real) or not torch.isfinite(torch.tensor(float(value))):
                raise ValueError(f"{name} must be finite")
        if process_variance < 0 or observation_variance <= 0 or initial_covariance <= 0:
            raise ValueError("process variance must be nonnegative; observation and initial covariance positive")
        if denominator_floor <= 0:
            raise ValueError("denominator_floor must be positive")
        self.key_dim = key_dim
        self.value_dim = value_dim
        self.chunk_length = chunk_length
        self.denominator_floor = float(denominator_floor)
        self.register_buffer("process_variance", torch.tensor(float(process_variance)), persistent=False)
        self.register_buffer("observation_variance", torch.tensor(float(observation_variance)), persistent=False)
        self.register_buffer("initial_covariance", torch.eye(key_dim) * float(initial_covariance), persistent=False)

    def forward(self, keys: Tensor, values: Tensor, queries: Tensor, *,
                transitions: Optional[Tensor] = None, transition_diagonals: Optional[Tensor] = None,
                process_variances: Optional[Tensor | Real] = None,
                observation_variances: Optional[Tensor | Real] = None) -> tuple[Tensor, Tensor, Tensor]:
        if keys.shape[-1] != self.key_dim or queries.shape[-1] != self.key_dim:
            raise ValueError("keys and queries must end in key_dim")
        if values.shape[-1] != self.value_dim:
            raise ValueError("values must end in value_dim")
        process = self.process_variance if process_variances is None else process_variances
        observation = self.observation_variance if observation_variances is None else observation_variances
        return bayesian_layer(
            keys, values, queries, transitions=transitions,
            transition_diagonals=transition_diagonals, process_variances=process,
            observation_variances=observation,
            initial_covariance=self.initial_covariance.to(device=keys.device),
            denominator_floor=self.denominator_floor, chunk_length=self.chunk_length,
            optimized=True, replay_ssm=True,
        )

    def associative_scan(self, keys: Tensor, values: Tensor, queries: Tensor, *,
                         observation_variances: Optional[Tensor | Real] = None
                         ) -> tuple[Tensor, Tensor, Tensor]:
        """Static scan; valid only for ``A=I`` and ``Q=0`` (rejects process noise)."""
        if bool(self.process_variance.detach().item() != 0.0):
            raise ValueError("associative_scan requires process_variance=0")
        if observation_variances is None:
            observation_variances = self.observation_variance
        scan = associative_static_bayesian_cuda if keys.is_cuda else associative_static_bayesian
        return scan(keys, values, queries, observation_variances=observation_variances,
                    initial_covariance=self.initial_covariance.to(device=keys.device),
                    denominator_floor=self.denominator_floor)


def _scan_inputs(keys, values, queries, observation_variances, initial_mean, initial_covariance,
                 denominator_floor, *, kernel_checks: bool = False):
    """Validation and promotion shared by the PyTorch and CUDA scans
    (reference ``replay_ssm.py:183-242``).

    With ``kernel_checks`` (the CUDA scan) the defaults are not built — the
    identity covariance and zero mean are valid by construction and are
    returned as ``None`` — and float32 observation variances are left to the
    kernel, which flags a non-finite value or one below the floor while it
    stages each token (the same comparison in the same dtype; the caller
    raises the same ``ValueError`` after the launch).
    """
    if keys.ndim < 2 or values.ndim < 2 or queries.ndim < 2:
        raise ValueError("keys, values and queries must have time and feature dimensions")
    if not all(value.is_floating_point() for value in (keys, values, queries)):
        raise TypeError("keys, values and queries must have floating-point dtype")
    if not (keys.device == values.device == queries.device):
        raise ValueError("keys, values and queries must be on the same device")
    if keys.shape[:-1] != queries.shape[:-1] or keys.shape[:-2] != values.shape[:-2]:
        raise ValueError("keys/queries batch-time dimensions must match values")
    t, d = keys.shape[-2:]
    if values.shape[-2] != t:
        raise ValueError("values and keys must have the same sequence length")
    m = values.shape[-1]
    try:
        dtype = torch.promote_types(torch.promote_types(keys.dtype, values.dtype),
                                    torch.promote_types(queries.dtype, torch.float32))
    except (RuntimeError, TypeError):
        dtype = torch.float32
    keys, values, queries = keys.to(dtype), values.to(dtype), queries.to(dtype)
    batch = keys.shape[:-2]
    device = keys.device
    if initial_covariance is None:
        covariance0 = None if kernel_checks else torch.eye(d, device=device, dtype=dtype).expand(*batch, d, d)
    else:
        covariance0 = initial_covariance.to(device=device, dtype=dtype)
    if covariance0 is not None:
        if covariance0.shape[-2:] != (d, d):
            raise ValueError("initial_covariance must end in [key_dim, key_dim]")
        if not _broadcastable(covariance0.shape[:-2], batch):
            raise ValueError("initial_covariance batch dimensions are not broadcastable to keys")
        covariance0 = covariance0.expand(*batch, d, d)
        _validate_covariance(covariance0, "initial_covariance", d)
    if initial_mean is None:
        mean0 = None if kernel_checks else torch.zeros(*batch, d, m, device=device, dtype=dtype)
    else:
        mean0 = initial_mean.to(device=device, dtype=dtype)
    if mean0 is not None:
        if mean0.shape[-2:] != (d, m):
            raise ValueError("initial_mean must end in [key_dim, value_dim]")
        if not _broadcastable(mean0.shape[:-2], batch):
            raise ValueError("initial_mean batch dimensions are not broadcastable to keys")
        mean0 = mean0.expand(*batch, d, m)
        _check_finite(mean0, "initial_mean")
    if not isinstance(denominator_floor, Real) or not math.isfinite(float(denominator_floor)) \
            or denominator_floor <= 0:
        raise ValueError("denominator_floor must be finite and positive")
    r2 = torch.as_tensor(observation_variances, device=device, dtype=dtype)
    r2 = torch.broadcast_to(r2, (*batch, t))
    # The information form divides by r itself; a variance below the floor
    # would make it disagree with the floored dense recurrence, so reject it.
    on_kernel = kernel_checks and dtype == torch.float32
    if r2.numel() and not on_kernel and (not bool(torch.isfinite(r2).all())
                                         or bool((r2 < float(denominator_floor)).any())):
        raise ValueError(
            "associative_static_bayesian requires finite observation_variances "
            "greater than or equal to denominator_floor"
        )
    return keys, values, queries, r2, mean0, covariance0, batch, t, d, m, dtype, device


def associative_static_bayesian(keys: Tensor, values: Tensor, queries: Tensor, *,
                                observation_variances: Tensor | Real = 1.0,
                                initial_mean: Optional[Tensor] = None,
                                initial_covariance: Optional[Tensor] = None,
                                denominator_floor: float = 1e-6) -> tuple[Tensor, Tensor, Tensor]:
    """Exact information-form prefix scan for the static, no-process-noise case.

    Equivalent to ``bayesian_layer(..., process_variances=0, transitions=None)``
    up to solve roundoff.  Raises ``ValueError`` when an observation variance
    is non-finite or below ``denominator_floor``.
    """
    (keys, values, queries, r2, mean0, covariance0, batch, t, d, m, dtype,
     device) = _scan_inputs(keys, values, queries, observation_variances, initial_mean,
                            initial_covariance, denominator_floor)
    if t == 0:
        return torch.empty(*batch, 0, m, device=device, dtype=dtype), mean0, covariance0
    precision0 = torch.linalg.inv(covariance0)
    natural0 = precision0 @ mean0
    weighted = keys / r2[..., :, None]
    precision = precision0.unsqueeze(-3) + (keys[..., :, :, None] * weighted[..., :, None, :]).cumsum(dim=-3)
    natural = natural0.unsqueeze(-3) + (weighted[..., :, :, None] * values[..., :, None, :]).cumsum(dim=-3)
    precision = (precision + precision.transpose(-1, -2)) * 0.5
    chol = torch.linalg.cholesky(precision)
    mean = torch.cholesky_solve(natural, chol)
    reads = (mean.transpose(-1, -2) @ queries.unsqueeze(-1)).squeeze(-1)
    covariance = torch.cholesky_inverse(chol[..., -1, :, :])
    return reads, mean[..., -1, :, :], covariance


def associative_static_bayesian_cuda(keys: Tensor, values: Tensor, queries: Tensor, *,
                                     observation_variances: Tensor | Real = 1.0,
                                     initial_mean: Optional[Tensor] = None,
                                     initial_covariance: Optional[Tensor] = None,
                                     denominator_floor: float = 1e-6) -> tuple[Tensor, Tensor, Tensor]:
    """Static scan on the sm_100a kernel (CUDA tensors only; forward only)."""
    if not isinstance(keys, Tensor) or not keys.is_cuda:
        raise ValueError("associative_static_bayesian_cuda requires CUDA tensors")
    if not values.is_cuda or not queries.is_cuda:
        raise ValueError("keys, values, and queries must share a CUDA device")
    if keys.device != values.device or keys.device != queries.device:
        raise ValueError("keys, values, and queries must share a CUDA device")
    from .assoc_cuda import assoc_scan_cuda

    (keys, values, queries, r2, mean0, covariance0, batch, t, d, m, dtype,
     device) = _scan_inputs(keys, values, queries, observation_variances, initial_mean,
                            initial_covariance, denominator_floor, kernel_checks=True)
    if t == 0:
        if mean0 is None:
            mean0 = torch.zeros(*batch, d, m, device=device, dtype=dtype)
        if covariance0 is None:
            covariance0 = torch.eye(d, device=device, dtype=dtype).expand(*batch, d, d)
        return torch.empty(*batch, 0, m, device=device, dtype=dtype), mean0, covariance0
    return assoc_scan_cuda(keys, values, queries, r2, mean0, covariance0, batch=batch,
                           denominator_floor=float(denominator_floor))


__all__ = ["ReplaySSM", "associative_static_bayesian", "associative_static_bayesian_cuda"]
