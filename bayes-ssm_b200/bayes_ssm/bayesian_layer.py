"""Exact Bayesian Layer (arXiv:2605.31163) -- public API of the B200 build.

Same functions, arguments, defaults, validation and error messages as
catid/bayes-ssm ``bayes_ssm/bayesian_layer.py`` (``bayesian_layer`` :735-1182,
``BayesianLayer`` :1185-1274, ``make_*`` :1277-1343).

Execution:

* CUDA tensors with diagonal (or identity) dynamics, scalar isotropic process
  noise and ``(key_dim, value_dim)`` in {(1,8), (2,8), (4,8), (8,8)} run the
  hand-written sm_100a kernels through :mod:`.fused_cuda` whenever
  ``optimized=True`` (``replay_ssm=True`` selects the same kernels: their
  backward is the chunk replay).  Any batch shape is flattened to chains.
  If the kernel library cannot be loaded this raises -- there is no silent
  fallback.
* Everything else (CPU tensors, ``optimized=False``, dense transitions or
  process covariances, rotation dynamics, other dimensions) runs the dense
  PyTorch recurrence below: the reference's equation-level semantics, with
  gradients from autograd.  There is no Triton or Inductor path.
"""
from __future__ import annotations

import math
import weakref
from numbers import Real
from typing import Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn

_FLOAT8_DTYPES = tuple(
    dtype
    for name in ("float8_e4m3fn", "float8_e4m3fnuz", "float8_e5m2", "float8_e5m2fnuz")
    if (dtype := getattr(torch, name, None)) is not None
)


def _inv_softplus(value: float) -> float:
    if value <= 0 or not math.isfinite(value):
        raise ValueError("softplus initialization must be finite and positive")
    return math.log(math.expm1(value))


def _broadcastable(shape: torch.Size, target: torch.Size) -> bool:
    if len(shape) > len(target):
        return False
    return all(a == b or a == 1 for a, b in zip(reversed(shape), reversed(target)))


def _as_tensor(x, *, device, dtype, name: str) -> Tensor:
    if isinstance(x, Tensor):
        if not x.is_floating_point():
            raise TypeError(f"{name} must have a floating-point dtype")
        return x.to(device=device, dtype=dtype)
    try:
        result = torch.as_tensor(x, device=device, dtype=dtype)
    except (TypeError, ValueError):
        raise TypeError(f"{name} must be a real scalar, sequence, or tensor; got {type(x).__name__}") from None
    if not result.is_floating_point():
        raise TypeError(f"{name} must contain real values")
    return result


def _as_time_tensor(x, t: int, batch_shape: torch.Size, name: str, *, device, dtype) -> Tensor:
    x = _as_tensor(x, device=device, dtype=dtype, name=name)
    if x.ndim == 0:
        return x.expand(*batch_shape, t)
    if x.shape[-1] != t or not _broadcastable(x.shape[:-1], batch_shape):
        raise ValueError(
            f"{name} must be scalar or have shape [..., T={t}] broadcastable to "
            f"batch shape {tuple(batch_shape)}; got {tuple(x.shape)}"
        )
    return x


def _is_cuda_graph_capturing(x: Tensor) -> bool:
    if not x.is_cuda:
        return False
    try:
        return bool(torch.cuda.is_current_stream_capturing())
    except RuntimeError:
        return False


def _skip_host_checks(x: Tensor) -> bool:
    # Host-visible validation is illegal during CUDA graph capture and is
    # skipped under torch.compile tracing; inputs were validated in warm-up.
    return torch.compiler.is_compiling() or _is_cuda_graph_capturing(x)


_DEVICE_CHECK_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


def _device_flags(tensors) -> Optional[list]:
    """Check flags of CUDA tensors from the library's one-pass check kernel
    (one read-back for all of them), or None where the torch checks apply
    (CPU or non-contiguous tensors, other dtypes, no library)."""
    if not all(x.is_cuda and x.dtype in _DEVICE_CHECK_DTYPES and x.is_contiguous() for x in tensors):
        return None
    from . import _capi
    try:
        _capi.load()
    except _capi.ExtensionUnavailable:
        return None
    return _capi.check_values([x.detach() for x in tensors])


# Tensors whose value checks a producing kernel already computed while it
# wrote them (the fused mixer prologue): data pointer -> (weak reference to
# the producer's output, element count, dtype, version, device flag words,
# word index).  An entry counts only while that output is alive, unchanged
# (same version counter) and covers exactly the checked tensor; anything else
# is checked by the check kernel as usual.
_PRECHECKED: dict = {}


def _register_prechecked(tensors, flags: Tensor) -> None:
    """Record that ``flags[i]`` (an int32 device tensor) holds the CHECK_*
    flags of every value of ``tensors[i]``, as ``bssm_check_values`` would
    report them."""
    for key in [k for k, e in _PRECHECKED.items() if e[0]() is None]:
        del _PRECHECKED[key]
    for i, x in enumerate(tensors):
        _PRECHECKED[x.data_ptr()] = (weakref.ref(x), x.numel(), x.dtype, x._version, flags, i)


def _prechecked_word(x: Tensor):
    """(flags tensor, index) holding x's check flags, or None."""
    e = _PRECHECKED.get(x.data_ptr()) if x.is_cuda else None
    if e is None:
        return None
    ref, numel, dtype, version, flags, i = e
    src = ref()
    if (src is None or x.numel() != numel or x.dtype != dtype or not x.is_contiguous()
            or src._version != version or x._version != version):
        return None
    return flags, i


class _DeviceChecks:
    """The value checks of one ``bayesian_layer`` call, raised in the
    reference's order (bayesian_layer.py:798-985) but run together: checks of
    contiguous CUDA tensors are queued and flushed as one pass per tensor with
    a single read-back.  A flush happens before any check that must run on
    the host and when an exception leaves the ``with`` block (so a queued
    failure that precedes a host-side error is the one raised); otherwise the
    caller flushes -- on the kernel path right after the forward kernel is
    enqueued, so one read-back covers the checks and the kernel (whose outputs
    are discarded if a check fails)."""

    def __init__(self) -> None:
        self.items = []

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb) -> bool:
        if exc_type is not None:
            self.flush()
        return False

    def finite(self, x: Tensor, name: str) -> None:
        self._add(x, name, 0)

    def variance(self, x: Tensor, name: str, *, strictly_positive: bool) -> None:
        self._add(x, name, 2 if strictly_positive else 1)

    def _add(self, x: Tensor, name: str, kind: int) -> None:
        if _skip_host_checks(x):
            return
        if not (x.is_cuda and x.dtype in _DEVICE_CHECK_DTYPES and x.is_contiguous()):
            self.flush()
            self._run_now(x, name, kind)
            return
        self.items.append((x, name, kind, _prechecked_word(x)))

    @staticmethod
    def _run_now(x: Tensor, name: str, kind: int) -> None:
        if kind == 0:
            _check_finite(x, name)
        else:
            _validate_variance(x, name, strictly_positive=kind == 2)

    def flush(self) -> None:
        items, self.items = self.items, []
        if not items:
            return
        plain = [x for x, _, _, pre in items if pre is None]
        flags = _device_flags(plain) if plain else []
        if flags is None:
            for x, name, kind, _ in items:
                self._run_now(x, name, kind)
            return
        if len(plain) < len(items):  # words a producing kernel computed: one read-back per word buffer
            bufs = {}
            for _, _, _, p in items:
                if p is not None and id(p[0]) not in bufs:
                    bufs[id(p[0])] = p[0].tolist()
            plain_flags = iter(flags)
            flags = [bufs[id(p[0])][p[1]] if p is not None else next(plain_flags) for _, _, _, p in items]
        from ._capi import CHECK_NEGATIVE, CHECK_NONFINITE, CHECK_NOT_POSITIVE
        for (x, name, kind, _), f in zip(items, flags):
            if f & CHECK_NONFINITE:
                raise ValueError(f"{name} must contain only finite values")
            if kind == 2 and f & CHECK_NOT_POSITIVE:
                raise ValueError(f"{name} must be strictly positive")
            if kind == 1 and f & CHECK_NEGATIVE:
                raise ValueError(f"{name} must be nonnegative")


def _check_finite(x: Tensor, name: str) -> None:
    if _skip_host_checks(x):
        return
    flags = _device_flags([x])
    if flags is not None:
        from ._capi import CHECK_NONFINITE
        if flags[0] & CHECK_NONFINITE:
            raise ValueError(f"{name} must contain only finite values")
        return
    if x.numel() and not bool(torch.isfinite(x).all()):
        raise ValueError(f"{name} must contain only finite values")


def _validate_variance(x: Tensor, name: str, *, strictly_positive: bool) -> None:
    if not _skip_host_checks(x):
        flags = _device_flags([x])
        if flags is not None:  # the same checks in the same order, one pass
            from ._capi import CHECK_NEGATIVE, CHECK_NONFINITE, CHECK_NOT_POSITIVE
            if flags[0] & CHECK_NONFINITE:
                raise ValueError(f"{name} must contain only finite values")
            if strictly_positive and flags[0] & CHECK_NOT_POSITIVE:
                raise ValueError(f"{name} must be strictly positive")
            if not strictly_positive and flags[0] & CHECK_NEGATIVE:
                raise ValueError(f"{name} must be nonnegative")
            return
    _check_finite(x, name)
    if _skip_host_checks(x) or x.numel() == 0:
        return
    minimum = float(x.detach().min())
    if strictly_positive and minimum <= 0:
        raise ValueError(f"{name} must be strictly positive")
    if not strictly_positive and minimum < 0:
        raise ValueError(f"{name} must be nonnegative")


def _validate_covariance(x: Tensor, name: str, d: int) -> None:
    if x.shape[-2:] != (d, d):
        raise ValueError(f"{name} must end in {(d, d)}, got {tuple(x.shape)}")
    _check_finite(x, name)
    if _skip_host_checks(x) or not x.numel():
        return
    sym = (x + x.transpose(-1, -2)) * 0.5
    scale = max(1.0, float(sym.detach().abs().max()))
    if not torch.allclose(x, x.transpose(-1, -2), rtol=1e-5, atol=1e-6 * scale):
        raise ValueError(f"{name} must be symmetric")
    minimum = float(torch.linalg.eigvalsh(sym.detach()).min())
    if minimum < -1e-5 * scale:
        raise ValueError(f"{name} must be positive semidefinite")


def _dense_recurrence(keys: Tensor, values: Tensor, queries: Tensor, transitions: Tensor,
                      process_covariances: Tensor, observation_variances: Tensor, mean: Tensor,
                      covariance: Tensor, denominator_floor: float
                      ) -> Tuple[Tensor, Tensor, Tensor]:
    """Dense predict/update/read over every token (Eqs. 8-13 of the paper).

    The predicted covariance is symmetrised before it is used, as the
    reference's dense chunked oracle does (bayesian_layer.py:701-703), so the
    result depends on the initial covariance only through its symmetric part.
    """
    outputs = []
    for i in range(keys.shape[-2]):
        a = transitions[..., i, :, :]
        cov = a @ covariance @ a.transpose(-1, -2) + process_covariances[..., i, :, :]
        cov = (cov + cov.transpose(-1, -2)) * 0.5
        mean = a @ mean
        key = keys[..., i, :]
        u = (cov @ key.unsqueeze(-1)).squeeze(-1)
        s = observation_variances[..., i] + (key * u).sum(-1)
        beta = s.clamp_min(denominator_floor).reciprocal()
        e = values[..., i, :] - (mean.transpose(-1, -2) @ key.unsqueeze(-1)).squeeze(-1)
        mean = mean + beta[..., None, None] * u[..., :, None] * e[..., None, :]
        covariance = cov - beta[..., None, None] * u[..., :, None] * u[..., None, :]
        covariance = (covariance + covariance.transpose(-1, -2)) * 0.5
        outputs.append((mean.transpose(-1, -2) @ queries[..., i, :].unsqueeze(-1)).squeeze(-1))
    return torch.stack(outputs, dim=-2), mean, covariance


def _rotation_path(keys, values, queries, cosines, sines, process_variances, observation_variances, mean,
                   covariance, *, batch_shape, t, d, m, chunk_length, denominator_floor, pending_checks=None):
    """Flatten the batch to chains and run the rotation kernels."""
    from .rotation_cuda import rotation_bayesian

    n = 1
    for s_ in batch_shape:
        n *= int(s_)
    j = d // 2

    def chains(x, tail):
        return x.expand(*batch_shape, *tail).reshape(n, *tail).float()

    y, mt, pt = rotation_bayesian(
        chains(keys, (t, d)), chains(values, (t, m)), chains(queries, (t, d)), chains(cosines, (t, j)),
        chains(sines, (t, j)), chains(process_variances, (t, j)), chains(observation_variances, (t,)),
        None if mean is None else chains(mean, (d, m)), None if covariance is None else chains(covariance, (d, d)),
        chunk_length=chunk_length, denominator_floor=denominator_floor, _pending_checks=pending_checks)
    return (y.reshape(*batch_shape, t, m), mt.reshape(*batch_shape, d, m), pt.reshape(*batch_shape, d, d))


def _default_mean(mean, batch_shape, d, m, device, dtype):
    return torch.zeros(*batch_shape, d, m, device=device, dtype=dtype) if mean is None else mean


def _default_covariance(covariance, batch_shape, d, device, dtype):
    if covariance is not None:
        return covariance
    return torch.eye(d, device=device, dtype=dtype).expand(*batch_shape, d, d).clone()


def _fused_path(keys, values, queries, diagonal, process_variances, observation_variances,
                mean, covariance, *, batch_shape, t, d, m, chunk_length, denominator_floor,
                fixed_dynamics, kernel_dtype, pending_checks=None):
    """Flatten the batch to chains, run the CUDA kernels, restore the shape."""
    from .fused_cuda import fused_diagonal_bayesian

    n = 1
    for s in batch_shape:
        n *= int(s)
    dev = keys.device

    def chains(x, tail):
        return x.expand(*batch_shape, *tail).reshape(n, *tail)

    k = chains(keys.to(kernel_dtype), (t, d))
    v = chains(values.to(kernel_dtype), (t, m))
    q = chains(queries.to(kernel_dtype), (t, d))
    a = None if diagonal is None else chains(diagonal, (t, d))
    p = chains(process_variances, (t,))
    r = chains(observation_variances, (t,))
    m0 = None if mean is None else chains(mean, (d, m))
    c0 = None if covariance is None else chains(covariance, (d, d))
    if a is None:
        a = torch.ones((), device=dev, dtype=torch.float32).expand(n, t, d)
    y, mt, pt = fused_diagonal_bayesian(k, v, q, a, p, r, m0, c0, chunk_length=chunk_length,
                                        denominator_floor=denominator_floor,
                                        fixed_dynamics=fixed_dynamics, _pending_checks=pending_checks)
    return (y.reshape(*batch_shape, t, m), mt.reshape(*batch_shape, d, m),
            pt.reshape(*batch_shape, d, d))


def bayesian_layer(
    keys: Tensor,
    values: Tensor,
    queries: Tensor,
    *,
    transitions: Optional[Tensor] = None,
    transition_diagonals: Optional[Tensor] = None,
    rotation_radii: Optional[Tensor] = None,
    rotation_angles: Optional[Tensor] = None,
    process_variances: Optional[Tensor | Real] = None,
    process_covariances: Optional[Tensor] = None,
    observation_variances: Optional[Tensor | Real] = None,
    initial_mean: Optional[Tensor] = None,
    initial_covariance: Optional[Tensor] = None,
    denominator_floor: float = 1e-6,
    chunk_length: Optional[int] = None,
    optimized: bool = False,
    replay_ssm: bool = False,
    fixed_dynamics: bool = False,
) -> Tuple[Tensor, Tensor, Tensor]:
    """Run an exact Bayesian Layer over a sequence.

    Args (as in the reference): ``keys``/``queries`` ``[..., T, D]``, ``values``
    ``[..., T, m]``; ``transitions`` ``[..., T, D, D]`` (default identity) or
    ``transition_diagonals`` ``[..., T, D]`` or ``rotation_radii`` +
    ``rotation_angles`` ``[..., T, D/2]``; ``process_variances`` scalar or
    ``[..., T]`` (or ``process_covariances`` ``[..., T, D, D]``);
    ``observation_variances`` scalar or ``[..., T]`` (default 1);
    ``initial_mean`` ``[..., D, m]`` (default 0); ``initial_covariance``
    ``[..., D, D]`` (default I); ``denominator_floor`` (1e-6);
    ``chunk_length`` (boundary-checkpoint spacing; results do not depend on it);
    ``optimized`` selects the CUDA kernels where they apply; ``replay_ssm``
    requests the chunk-replay backward (the kernels' backward always is one);
    ``fixed_dynamics`` asserts ``A=0.97I, Q=0.1I, R=1`` and makes the kernels
    use those constants.

    BF16/FP16/FP8 inputs are promoted: the recurrent state, covariance and
    readouts are FP32.  Returns ``(readouts, final_mean, final_covariance)``.
    """
    if not all(isinstance(x, Tensor) for x in (keys, values, queries)):
        raise TypeError("keys, values and queries must be torch tensors")
    if keys.ndim < 2 or values.ndim < 2 or queries.ndim < 2:
        raise ValueError("keys, values and queries must have a time and feature dimension")
    if not all(x.is_floating_point() for x in (keys, values, queries)):
        raise TypeError("keys, values and queries must have floating-point dtype")
    if not (keys.device == values.device == queries.device):
        raise ValueError("keys, values and queries must be on the same device")
    if keys.shape[:-1] != queries.shape[:-1] or keys.shape[:-2] != values.shape[:-2]:
        raise ValueError("keys/queries batch and time dimensions must match values")
    t, d = keys.shape[-2:]
    m = values.shape[-1]
    if d <= 0 or m <= 0:
        raise ValueError("key and value dimensions must be positive")
    if values.shape[-2] != t:
        raise ValueError("values and keys must have the same sequence length")
    batch_shape = keys.shape[:-2]
    device, input_dtype = keys.device, keys.dtype
    low_precision = (torch.float16, torch.bfloat16, *_FLOAT8_DTYPES)
    dtype = torch.float32 if input_dtype in low_precision else input_dtype
    # BF16 projections may enter the kernels as BF16 (widened in registers);
    # every other path sees the promoted FP32 tensors.
    all_bf16 = keys.dtype == values.dtype == queries.dtype == torch.bfloat16
    raw_keys, raw_values, raw_queries = keys, values, queries
    # FP32 / BF16 / FP16 projections are checked as they are and widened only
    # where a path needs FP32 (widening keeps every value and its finiteness);
    # other low-precision dtypes are promoted first, as the reference does
    # (bayesian_layer.py:823-830).
    if not all(x.dtype in _DEVICE_CHECK_DTYPES for x in (keys, values, queries)):
        keys = keys.to(dtype)
        values = values.to(dtype)
        queries = queries.to(dtype)
    with _DeviceChecks() as chk:
        for x, name in ((keys, "keys"), (values, "values"), (queries, "queries")):
            chk.finite(x, name)
        if (rotation_radii is None) != (rotation_angles is None):
            raise ValueError("rotation_radii and rotation_angles must be supplied together")
        if transitions is not None and transition_diagonals is not None:
            raise ValueError("pass transitions or transition_diagonals, not both")
        if (rotation_radii is not None or rotation_angles is not None) and (
            transitions is not None or transition_diagonals is not None
        ):
            raise ValueError("rotation dynamics are mutually exclusive with transitions and transition_diagonals")
        if not isinstance(replay_ssm, bool):
            raise TypeError("replay_ssm must be a bool")
        if not isinstance(fixed_dynamics, bool):
            raise TypeError("fixed_dynamics must be a bool")

        diagonal = None
        identity_dynamics = False
        rotation = False
        if rotation_radii is not None:
            if d % 2:
                raise ValueError("rotational dynamics require an even key dimension")
            checked = []
            for name, value in (("rotation_radii", rotation_radii), ("rotation_angles", rotation_angles)):
                if not isinstance(value, Tensor) or value.ndim < 2:
                    raise ValueError(f"{name} must have shape [..., T={t}, D/2={d // 2}]")
                if not value.is_floating_point():
                    raise TypeError(f"{name} must have a floating-point dtype")
                if value.shape[-2:] != (t, d // 2):
                    raise ValueError(f"{name} must end in {(t, d // 2)}, got {tuple(value.shape)}")
                if not _broadcastable(value.shape[:-2], batch_shape):
                    raise ValueError(f"{name} batch dimensions are not broadcastable to input batch")
                value = value.to(device=device, dtype=dtype)
                chk.finite(value, name)
                checked.append(value)
            rotation_radii, rotation_angles = checked
            rotation = True
        elif transition_diagonals is not None:
            if not isinstance(transition_diagonals, Tensor) or transition_diagonals.ndim < 2:
                raise ValueError(f"transition_diagonals must have shape [..., T={t}, D={d}]")
            if not transition_diagonals.is_floating_point():
                raise TypeError("transition_diagonals must have a floating-point dtype")
            transition_diagonals = transition_diagonals.to(device=device, dtype=dtype)
            if transition_diagonals.shape[-2:] != (t, d):
                raise ValueError(f"transition_diagonals must end in {(t, d)}, got {tuple(transition_diagonals.shape)}")
            if not _broadcastable(transition_diagonals.shape[:-2], batch_shape):
                raise ValueError("transition_diagonals batch dimensions are not broadcastable to the input batch")
            chk.finite(transition_diagonals, "transition_diagonals")
            diagonal = transition_diagonals
        elif transitions is None:
            identity_dynamics = True
        else:
            if not isinstance(transitions, Tensor) or transitions.ndim < 3:
                raise ValueError(f"transitions must have shape [..., T={t}, D={d}, D={d}]")
            if not transitions.is_floating_point():
                raise TypeError("transitions must have a floating-point dtype")
            transitions = transitions.to(device=device, dtype=dtype)
            if transitions.shape[-3:] != (t, d, d):
                raise ValueError(f"transitions must end in {(t, d, d)}, got {tuple(transitions.shape)}")
            if not _broadcastable(transitions.shape[:-3], batch_shape):
                raise ValueError("transitions batch dimensions are not broadcastable to the input batch")
            chk.finite(transitions, "transitions")

        if rotation:
            if process_covariances is not None:
                raise ValueError("rotational dynamics require per-pair process_variances, not process_covariances")
            if process_variances is None:
                process_variances = torch.zeros(*batch_shape, t, d // 2, device=device, dtype=dtype)
            else:
                process_variances = _as_tensor(process_variances, device=device, dtype=dtype,
                                               name="process_variances")
                if process_variances.ndim == 0:
                    process_variances = process_variances.expand(*batch_shape, t, d // 2)
                elif process_variances.shape[-2:] == (t, d // 2) and _broadcastable(
                    process_variances.shape[:-2], batch_shape
                ):
                    process_variances = process_variances.expand(*batch_shape, t, d // 2)
                else:
                    raise ValueError(f"rotational process_variances must be scalar or end in {(t, d // 2)}")
                chk.variance(process_variances, "process_variances", strictly_positive=False)
        elif process_covariances is not None and process_variances is not None:
            raise ValueError("pass process_covariances or process_variances, not both")
        elif process_covariances is not None:
            if not isinstance(process_covariances, Tensor) or process_covariances.ndim < 3:
                raise ValueError(f"process_covariances must have shape [..., T={t}, D={d}, D={d}]")
            if not process_covariances.is_floating_point():
                raise TypeError("process_covariances must have a floating-point dtype")
            process_covariances = process_covariances.to(device=device, dtype=dtype)
            if process_covariances.shape[-3:] != (t, d, d):
                raise ValueError(f"process_covariances must end in {(t, d, d)}, got {tuple(process_covariances.shape)}")
            if not _broadcastable(process_covariances.shape[:-3], batch_shape):
                raise ValueError("process_covariances batch dimensions are not broadcastable to the input batch")
            chk.flush()
            _validate_covariance(process_covariances, "process_covariances", d)
        else:
            if process_variances is None:
                process_variances = 0.0
            process_variances = _as_time_tensor(process_variances, t, batch_shape, "process_variances",
                                                device=device, dtype=dtype)
            chk.variance(process_variances, "process_variances", strictly_positive=False)
        if observation_variances is None:
            observation_variances = 1.0
        observation_variances = _as_time_tensor(observation_variances, t, batch_shape,
                                                "observation_variances", device=device, dtype=dtype)
        chk.variance(observation_variances, "observation_variances", strictly_positive=True)

        user_mean = initial_mean is not None
        user_cov = initial_covariance is not None
        mean = covariance = None  # defaults (zeros, identity) are built only where used
        if initial_mean is not None:
            if not isinstance(initial_mean, Tensor) or initial_mean.ndim < 2:
                raise ValueError(f"initial_mean must have shape [..., D={d}, m={m}]")
            if not initial_mean.is_floating_point():
                raise TypeError("initial_mean must have a floating-point dtype")
            mean = initial_mean.to(device=device, dtype=dtype)
            if mean.shape[-2:] != (d, m) or not _broadcastable(mean.shape[:-2], batch_shape):
                raise ValueError("initial_mean has incompatible dimensions or batch shape")
            chk.finite(mean, "initial_mean")
            mean = mean.expand(*batch_shape, d, m)
        if initial_covariance is not None:
            if not isinstance(initial_covariance, Tensor) or initial_covariance.ndim < 2:
                raise ValueError(f"initial_covariance must have shape [..., D={d}, D={d}]")
            if not initial_covariance.is_floating_point():
                raise TypeError("initial_covariance must have a floating-point dtype")
            covariance = initial_covariance.to(device=device, dtype=dtype)
            if not _broadcastable(covariance.shape[:-2], batch_shape):
                raise ValueError("initial_covariance batch dimensions are not broadcastable to the input batch")
            chk.flush()
            _validate_covariance(covariance, "initial_covariance", d)
            covariance = covariance.expand(*batch_shape, d, d)

        if not isinstance(denominator_floor, Real) or not math.isfinite(float(denominator_floor)):
            raise ValueError("denominator_floor must be finite")
        if denominator_floor <= 0:
            raise ValueError("denominator_floor must be positive")
        if chunk_length is not None and (not isinstance(chunk_length, int) or isinstance(chunk_length, bool)
                                         or chunk_length <= 0):
            raise ValueError("chunk_length must be a positive integer or None")
        if t == 0:
            chk.flush()
            return (torch.empty(*batch_shape, 0, m, device=device, dtype=dtype),
                    _default_mean(mean, batch_shape, d, m, device, dtype),
                    _default_covariance(covariance, batch_shape, d, device, dtype))
        if chunk_length is None:
            chunk_length = t

    from .fused_cuda import kernel_supports
    from .rotation_cuda import SUPPORTED as ROTATION_SUPPORTED

    if (rotation and optimized and device.type == "cuda" and (d, m) in ROTATION_SUPPORTED
            and dtype in (torch.float32, torch.bfloat16)):
        # the reference's radius handling and make_rotation_dynamics' own
        # operations, so autograd reaches the radii and angles the same way:
        # one fused kernel pair for same-shape float32 tensors, else the ops
        from .rotation_cuda import coefficients_apply, rotation_coefficients
        if coefficients_apply(rotation_radii, rotation_angles):
            cosines, sines = rotation_coefficients(rotation_radii, rotation_angles)
        else:
            radius = rotation_radii.clamp_min(torch.finfo(dtype).tiny)
            radius = torch.where(radius <= 1.0, radius, torch.ones_like(radius))
            raw = torch.log(radius).exp()
            rho = torch.where(raw <= 1.0, raw, torch.ones_like(raw))
            cosines, sines = rho * rotation_angles.cos(), rho * rotation_angles.sin()
        return _rotation_path(keys, values, queries, cosines, sines,
                              process_variances, observation_variances, mean if user_mean else None,
                              covariance if user_cov else None, batch_shape=batch_shape, t=t, d=d, m=m,
                              chunk_length=chunk_length, denominator_floor=float(denominator_floor),
                              pending_checks=chk)

    kernel_path = (
        optimized
        and device.type == "cuda"
        and kernel_supports(d, m)
        and dtype in (torch.float32, torch.bfloat16)
        and not rotation
        and process_covariances is None
        and (diagonal is not None or identity_dynamics)
    )
    if kernel_path:
        kernel_dtype = torch.bfloat16 if all_bf16 and d != 64 else torch.float32
        src = (raw_keys, raw_values, raw_queries) if all_bf16 else (keys, values, queries)
        return _fused_path(
            *src, diagonal, process_variances, observation_variances,
            mean if user_mean else None, covariance if user_cov else None,
            batch_shape=batch_shape, t=t, d=d, m=m, chunk_length=chunk_length,
            denominator_floor=float(denominator_floor), fixed_dynamics=fixed_dynamics,
            kernel_dtype=kernel_dtype, pending_checks=chk)

    chk.flush()
    mean = _default_mean(mean, batch_shape, d, m, device, dtype)
    covariance = _default_covariance(covariance, batch_shape, d, device, dtype)
    # Dense PyTorch recurrence (reference semantics).
    if rotation:
        radius = rotation_radii.clamp_min(torch.finfo(dtype).tiny)
        radius = torch.where(radius <= 1.0, radius, torch.ones_like(radius))
        transitions = make_rotation_dynamics(torch.log(radius), rotation_angles)
        process_covariances = make_rotation_process_covariances(process_variances)
    else:
        eye = torch.eye(d, device=device, dtype=dtype)
        if diagonal is not None:
            transitions = torch.diag_embed(diagonal)
        elif identity_dynamics:
            transitions = eye.expand(*batch_shape, t, d, d)
        if process_covariances is None:
            process_covariances = process_variances[..., None, None] * eye
    return _dense_recurrence(keys.to(dtype), values.to(dtype), queries.to(dtype), transitions,
                             process_covariances, observation_variances, mean, covariance,
                             float(denominator_floor))


class BayesianLayer(nn.Module):
    """Convenience module with positive noise floors and initial covariance.

    Same constructor, buffers/parameters and forward as the reference
    (bayesian_layer.py:1185-1274).
    """

    def __init__(self, key_dim: int, value_dim: int, *, initial_covariance: float = 3.0,
                 process_variance: float = 0.05, observation_variance: float = 0.05,
                 learn_noise: bool = False, denominator_floor: float = 1e-6):
        super().__init__()
        if (not isinstance(key_dim, int) or isinstance(key_dim, bool) or not isinstance(value_dim, int)
                or isinstance(value_dim, bool)):
            raise TypeError("key_dim and value_dim must be integers")
        if key_dim <= 0 or value_dim <= 0:
            raise ValueError("key_dim and value_dim must be positive")
        for value, name, strictly_positive in (
            (initial_covariance, "initial_covariance", False),
            (process_variance, "process_variance", False),
            (observation_variance, "observation_variance", True),
        ):
            if not isinstance(value, Real) or not math.isfinite(float(value)):
                raise ValueError(f"{name} must be a finite real scalar")
            if strictly_positive and value <= 0:
                raise ValueError(f"{name} must be strictly positive")
            if not strictly_positive and value < 0:
                raise ValueError(f"{name} must be nonnegative")
        if learn_noise and process_variance <= 0:
            raise ValueError("process_variance must be positive when learn_noise=True")
        if not isinstance(denominator_floor, Real) or not math.isfinite(float(denominator_floor)):
            raise ValueError("denominator_floor must be finite")
        if denominator_floor <= 0:
            raise ValueError("denominator_floor must be positive")
        self.key_dim, self.value_dim = key_dim, value_dim
        self.denominator_floor = denominator_floor
        self.register_buffer("initial_covariance", torch.tensor(float(initial_covariance)))
        self._learn_noise = bool(learn_noise)
        process_raw = torch.tensor(_inv_softplus(float(max(process_variance, 1e-8))))
        observation_raw = torch.tensor(_inv_softplus(float(observation_variance)))
        if learn_noise:
            self._process_raw = nn.Parameter(process_raw)
            self._observation_raw = nn.Parameter(observation_raw)
        else:
            self.register_buffer("_process_raw", process_raw)
            self.register_buffer("_observation_raw", observation_raw)
        self.register_buffer("_process_is_zero", torch.tensor(process_variance == 0))

    @property
    def process_variance(self) -> Tensor:
        return torch.where(self._process_is_zero, self._process_raw * 0,
                           F.softplus(self._process_raw).clamp_min(1e-8))

    @property
    def observation_variance(self) -> Tensor:
        return F.softplus(self._observation_raw).clamp_min(1e-8)

    def forward(self, keys: Tensor, values: Tensor, queries: Tensor, *,
                transitions: Optional[Tensor] = None, chunk_length: Optional[int] = None,
                initial_mean: Optional[Tensor] = None, initial_covariance: Optional[Tensor] = None,
                optimized: bool = False):
        if not all(isinstance(x, Tensor) for x in (keys, values, queries)):
            raise TypeError("keys, values and queries must be torch tensors")
        if keys.ndim < 2 or values.ndim < 2 or queries.ndim < 2:
            raise ValueError("keys, values and queries must have a time and feature dimension")
        if keys.ndim >= 1 and keys.shape[-1] != self.key_dim:
            raise ValueError(f"keys last dimension must be key_dim={self.key_dim}")
        if values.ndim >= 1 and values.shape[-1] != self.value_dim:
            raise ValueError(f"values last dimension must be value_dim={self.value_dim}")
        if queries.ndim >= 1 and queries.shape[-1] != self.key_dim:
            raise ValueError(f"queries last dimension must be key_dim={self.key_dim}")
        if initial_covariance is None:
            d = keys.shape[-1]
            initial_covariance = torch.eye(d, device=keys.device, dtype=torch.float32) * \
                self.initial_covariance.to(device=keys.device, dtype=torch.float32)
        return bayesian_layer(
            keys, values, queries, transitions=transitions,
            process_variances=self.process_variance,
            observation_variances=self.observation_variance,
            initial_mean=initial_mean, initial_covariance=initial_covariance,
            denominator_floor=self.denominator_floor, chunk_length=chunk_length,
            optimized=optimized,
        )


def make_diagonal_dynamics(log_decay: Tensor) -> Tensor:
    """Build diagonal A_t from log radii, shape ``[..., T, D]`` -> ``[..., T,D,D]``."""
    raw_radius = log_decay.exp()
    radius = torch.where(raw_radius <= 1.0, raw_radius, torch.ones_like(raw_radius))
    return torch.diag_embed(radius)


def make_rotation_dynamics(log_radius: Tensor, angle: Tensor) -> Tensor:
    """Block-diagonal damped 2-D rotations ``[..., T, J]`` -> ``[..., T, 2J, 2J]``."""
    if not isinstance(log_radius, Tensor) or not isinstance(angle, Tensor):
        raise TypeError("log_radius and angle must be tensors")
    if log_radius.shape != angle.shape:
        raise ValueError("log_radius and angle must have the same shape")
    if not log_radius.is_floating_point() or not angle.is_floating_point():
        raise TypeError("log_radius and angle must have floating-point dtype")
    if log_radius.device != angle.device:
        raise ValueError("log_radius and angle must be on the same device")
    raw_radius = log_radius.exp()
    radius = torch.where(raw_radius <= 1.0, raw_radius, torch.ones_like(raw_radius))
    c, s = radius * angle.cos(), radius * angle.sin()
    j = angle.shape[-1]
    out = torch.zeros(*angle.shape[:-1], 2 * j, 2 * j, device=angle.device, dtype=angle.dtype)
    idx = torch.arange(j, device=angle.device)
    even = 2 * idx
    odd = even + 1
    out[..., even, even] = c
    out[..., odd, odd] = c
    out[..., even, odd] = -s
    out[..., odd, even] = s
    return out


def make_rotation_process_covariances(process_variance: Tensor) -> Tensor:
    """Rotation noise ``ell^2 diag(1, 0)`` per 2-D block: ``[..., T, J]`` -> ``[..., T, 2J, 2J]``."""
    if not isinstance(process_variance, Tensor):
        process_variance = torch.as_tensor(process_variance)
    if process_variance.ndim < 1:
        raise ValueError("process_variance must have a final block dimension")
    if not process_variance.is_floating_point():
        raise TypeError("process_variance must have a floating-point dtype")
    if not bool(torch.isfinite(process_variance).all()) or bool((process_variance < 0).any()):
        raise ValueError("process_variance must be finite and nonnegative")
    j = process_variance.shape[-1]
    zeros = torch.zeros_like(process_variance)
    diagonal = torch.stack((process_variance, zeros), dim=-1).reshape(*process_variance.shape[:-1], 2 * j)
    return torch.diag_embed(diagonal)


__all__ = ["bayesian_layer", "BayesianLayer", "make_diagonal_dynamics", "make_rotation_dynamics",
           "make_rotation_process_covariances"]
