"""BayesianMixer paper-feature prologue: projection rows -> recurrence inputs.

catid/bayes-ssm ``example/train_6layer.py`` builds the recurrence's inputs
from one fused projection per token (``BayesianMixer.forward``, :579-700, with
``fuse_paper_qkv`` / ``fuse_paper_projection`` and learned dynamics):

* a causal depthwise length-4 convolution over the Q/K/V channels
  (``CausalDepthwise4``, :160-191; ``nn.Conv1d`` with left padding 3 is the
  same map);
* SiLU on each stream, then per-head ``F.normalize`` of q and k (:629-639);
* process / observation variance ``softplus(noise + bias) + 1e-4`` (:665-666)
  and decay ``exp(-softplus(logit + bias))`` (:698);
* every stream permuted to chain-major ``[B*H, T, .]`` (:647-650, :699-701).

:func:`paper_prologue` does all of it in one sm_100a kernel on CUDA tensors
(``csrc/bssm_envelope.cu``), with a one-kernel backward that also sums the
convolution-weight and auxiliary-bias gradients deterministically.  On CPU
tensors it runs :func:`paper_prologue_torch`, the same op chain in PyTorch.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _capi

_DTYPES = {torch.float32: _capi.BSSM_F32, torch.bfloat16: _capi.BSSM_BF16}


def _widths(heads: int, key_dim: int, head_dim: int) -> tuple[int, int, int, int]:
    sw, w = heads * key_dim, heads * head_dim
    return sw, w, 2 * sw + w, sw + 2 * heads  # state width, width, conv channels, aux channels


def paper_prologue_torch(projected: Tensor, conv_weight: Tensor, aux_bias: Optional[Tensor], *, heads: int,
                         key_dim: int, head_dim: int):
    """The reference's op chain in PyTorch, computed in float32.

    Returns ``(keys, queries, values, decay, process, observation)`` shaped
    ``[B*H, T, D]``, ``[B*H, T, D]``, ``[B*H, T, head_dim]``, ``[B*H, T, D]``,
    ``[B*H, T]``, ``[B*H, T]``.
    """
    b, t, _ = projected.shape
    sw, w, c, aux_w = _widths(heads, key_dim, head_dim)
    x = projected.float()
    qkv = x[..., :c]
    aux = x[..., c:c + aux_w]
    if aux_bias is not None:
        aux = aux + aux_bias.float()
    taps = conv_weight.float().reshape(c, 4)
    padded = F.pad(qkv.transpose(1, 2), (3, 0))
    y = padded[..., :t] * taps[:, 0].view(1, -1, 1)
    y = y + padded[..., 1:t + 1] * taps[:, 1].view(1, -1, 1)
    y = y + padded[..., 2:t + 2] * taps[:, 2].view(1, -1, 1)
    y = y + padded[..., 3:t + 3] * taps[:, 3].view(1, -1, 1)
    q_in, k_in, v_in = y.transpose(1, 2).split((sw, sw, w), dim=-1)

    def heads_first(z, dim):
        return z.reshape(b, t, heads, dim).permute(0, 2, 1, 3).reshape(b * heads, t, dim)

    q = heads_first(F.normalize(F.silu(q_in).view(b, t, heads, key_dim), dim=-1), key_dim)
    k = heads_first(F.normalize(F.silu(k_in).view(b, t, heads, key_dim), dim=-1), key_dim)
    v = heads_first(F.silu(v_in), head_dim)
    noise = aux[..., sw:].view(b, t, heads, 2)
    process = (F.softplus(noise[..., 0]) + 1e-4).permute(0, 2, 1).reshape(b * heads, t)
    observation = (F.softplus(noise[..., 1]) + 1e-4).permute(0, 2, 1).reshape(b * heads, t)
    decay = heads_first(torch.exp(-F.softplus(aux[..., :sw])), key_dim)
    return k, q, v, decay, process, observation


def _rows(x: Tensor) -> int:
    """Row stride (elements) of a [B, T, P] tensor whose rows are evenly spaced."""
    if x.stride(-1) != 1 or (x.shape[0] > 1 and x.stride(0) != x.shape[1] * x.stride(1)):
        raise ValueError("projected must have unit channel stride and evenly spaced token rows")
    return x.stride(1)


class _PaperPrologue(torch.autograd.Function):
    @staticmethod
    def forward(ctx, projected, conv_weight, aux_bias, heads, key_dim, head_dim, out_dtype, check_flags):
        b, t, _ = projected.shape
        sw, w, c, aux_w = _widths(heads, key_dim, head_dim)
        dev = projected.device
        wt = conv_weight.detach().float().reshape(c, 4).contiguous()
        bias = None if aux_bias is None else aux_bias.detach().float().contiguous()
        n = b * heads
        keys = torch.empty(n, t, key_dim, device=dev, dtype=out_dtype)
        queries = torch.empty_like(keys)
        values = torch.empty(n, t, head_dim, device=dev, dtype=out_dtype)
        decay = torch.empty(n, t, key_dim, device=dev, dtype=torch.float32)
        process = torch.empty(n, t, device=dev, dtype=torch.float32)
        observation = torch.empty_like(process)
        stream = torch.cuda.current_stream(dev).cuda_stream
        with torch.cuda.device(dev):
            _capi.envelope_prologue(projected, _DTYPES[projected.dtype], b, t, heads, key_dim, head_dim,
                                    _rows(projected), wt, bias, keys, queries, values, _DTYPES[out_dtype], decay,
                                    process, observation, stream, check_flags=check_flags)
        ctx.save_for_backward(projected, wt, bias)
        ctx.dims = (heads, key_dim, head_dim, out_dtype, conv_weight.dtype,
                    None if aux_bias is None else aux_bias.dtype, tuple(conv_weight.shape))
        ctx.set_materialize_grads(False)
        return keys, queries, values, decay, process, observation

    @staticmethod
    def backward(ctx, gk, gq, gv, gd, gp, go):
        projected, wt, bias = ctx.saved_tensors
        heads, key_dim, head_dim, out_dtype, w_dtype, b_dtype, w_shape = ctx.dims
        b, t, p = projected.shape
        dev = projected.device

        def prep(g, dtype):
            return None if g is None else g.to(dtype).contiguous()

        gk, gq, gv = prep(gk, out_dtype), prep(gq, out_dtype), prep(gv, out_dtype)
        gd, gp, go = prep(gd, torch.float32), prep(gp, torch.float32), prep(go, torch.float32)
        gx = torch.empty(b, t, p, device=dev, dtype=projected.dtype)
        gw = torch.empty(wt.shape, device=dev, dtype=torch.float32)
        gb = None if bias is None else torch.empty_like(bias)
        ws = torch.empty(_capi.envelope_partial_floats(b, t, heads, key_dim, head_dim), device=dev,
                         dtype=torch.float32)
        stream = torch.cuda.current_stream(dev).cuda_stream
        with torch.cuda.device(dev):
            _capi.envelope_prologue_backward(projected, _DTYPES[projected.dtype], b, t, heads, key_dim, head_dim,
                                             _rows(projected), wt, bias, gk, gq, gv, _DTYPES[out_dtype], gd, gp, go,
                                             gx, p, gw, gb, ws, stream)
        gw = gw.reshape(w_shape).to(w_dtype)
        if gb is not None:
            gb = gb.to(b_dtype)
        return gx, gw, gb, None, None, None, None, None


def paper_prologue(projected: Tensor, conv_weight: Tensor, aux_bias: Optional[Tensor] = None, *, heads: int,
                   key_dim: int, head_dim: int, out_dtype: torch.dtype = torch.float32):
    """Recurrence inputs from the fused projection (see the module docstring).

    ``projected`` is ``[B, T, 2*H*D + H*head_dim + H*D + 2*H]``: the q, k and v
    streams, the decay logits and the per-head (process, observation) noise
    pairs.  ``conv_weight`` is the depthwise Conv1d weight ``[C, 1, 4]`` over
    the q/k/v channels; ``aux_bias`` is added to the auxiliary channels.
    ``out_dtype`` (float32 or bfloat16) is the dtype of keys, queries and
    values; decay and the variances are float32.  Gradients flow to
    ``projected``, ``conv_weight`` and ``aux_bias``.
    """
    if projected.ndim != 3:
        raise ValueError("projected must be [batch, tokens, channels]")
    sw, w, c, aux_w = _widths(heads, key_dim, head_dim)
    if projected.shape[-1] != c + aux_w:
        raise ValueError(f"projected must have {c + aux_w} channels (q, k, v, decay logits, noise), "
                         f"got {projected.shape[-1]}")
    if conv_weight.numel() != 4 * c:
        raise ValueError(f"conv_weight must be [{c}, 1, 4]")
    if aux_bias is not None and aux_bias.numel() != aux_w:
        raise ValueError(f"aux_bias must have {aux_w} entries")
    if not projected.is_cuda:
        return paper_prologue_torch(projected, conv_weight, aux_bias, heads=heads, key_dim=key_dim,
                                    head_dim=head_dim)
    if projected.dtype not in _DTYPES or out_dtype not in _DTYPES:
        raise TypeError("paper_prologue on CUDA takes float32 or bfloat16 projections and outputs")
    if key_dim < 2 or key_dim > 64 or key_dim & (key_dim - 1) or head_dim % 2:
        raise NotImplementedError("paper_prologue on CUDA needs key_dim a power of two in [2, 64] and an even "
                                  f"head_dim (got {key_dim}, {head_dim}); use paper_prologue_torch")
    # The kernel also computes bayesian_layer's value checks of what it writes
    # (finite keys, values, queries and decay; nonnegative process and
    # positive observation variances), so that layer need not read them again.
    check_flags = torch.zeros(6, device=projected.device, dtype=torch.int32)
    outs = _PaperPrologue.apply(projected, conv_weight, aux_bias, heads, key_dim, head_dim, out_dtype, check_flags)
    k, q, v, decay, process, observation = outs
    from .bayesian_layer import _register_prechecked
    _register_prechecked((k, v, q, decay, process, observation), check_flags)
    return outs


def read_epilogue_torch(read: Tensor, gate: Tensor, norm_weight: Tensor, *, heads: int,
                        eps: Optional[float] = None) -> Tensor:
    """The reference's readout in PyTorch (``train_6layer.py:719-729``): the
    reads permuted to ``[B, T, H, hd]`` and cast to the gate's dtype, then
    ``nn.RMSNorm(hd)`` (weight ``norm_weight``; ``eps=None`` is the dtype's
    machine epsilon, as ``nn.RMSNorm`` uses) times ``SiLU(gate)``, reshaped to
    ``[B, T, W]``."""
    bh, t, hd = read.shape
    b = bh // heads
    r = read.view(b, heads, t, hd).permute(0, 2, 1, 3).to(gate.dtype)
    normed = F.rms_norm(r, (hd,), norm_weight.to(gate.dtype), eps)
    return (normed * F.silu(gate.reshape(b, t, heads, hd))).reshape(b, t, heads * hd)


def _gate_rows(gate: Tensor) -> int:
    if gate.stride(-1) != 1 or (gate.shape[0] > 1 and gate.stride(0) != gate.shape[1] * gate.stride(1)):
        raise ValueError("gate must have unit channel stride and evenly spaced token rows")
    return gate.stride(1)


class _ReadEpilogue(torch.autograd.Function):
    @staticmethod
    def forward(ctx, read, gate, norm_weight, heads, eps):
        bh, t, hd = read.shape
        b = bh // heads
        dev = read.device
        w = norm_weight.detach().float().contiguous()
        out = torch.empty(b, t, heads * hd, device=dev, dtype=gate.dtype)
        stream = torch.cuda.current_stream(dev).cuda_stream
        with torch.cuda.device(dev):
            _capi.envelope_epilogue(read, _DTYPES[read.dtype], gate, _DTYPES[gate.dtype], _gate_rows(gate), w, eps, b,
                                    t, heads, hd, out, stream)
        ctx.save_for_backward(read, gate, w)
        ctx.dims = (heads, eps, norm_weight.dtype)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        read, gate, w = ctx.saved_tensors
        heads, eps, w_dtype = ctx.dims
        bh, t, hd = read.shape
        b = bh // heads
        dev = read.device
        go = grad_out.to(gate.dtype).contiguous()
        g_read = torch.empty_like(read)
        g_gate = torch.empty(b, t, heads * hd, device=dev, dtype=gate.dtype)
        g_w = torch.empty(hd, device=dev, dtype=torch.float32)
        ws = torch.empty(_capi.envelope_epilogue_partial_floats(b, t, heads, hd), device=dev, dtype=torch.float32)
        stream = torch.cuda.current_stream(dev).cuda_stream
        with torch.cuda.device(dev):
            _capi.envelope_epilogue_backward(read, _DTYPES[read.dtype], gate, _DTYPES[gate.dtype], _gate_rows(gate), w,
                                             eps, b, t, heads, hd, go, g_read, g_gate, heads * hd, g_w, ws, stream)
        return g_read, g_gate.view(gate.shape), g_w.to(w_dtype), None, None


def read_epilogue(read: Tensor, gate: Tensor, norm_weight: Tensor, *, heads: int,
                  eps: Optional[float] = None) -> Tensor:
    """The mixer's readout: ``read_norm(read) * SiLU(gate)`` as ``[B, T, W]``.

    ``read`` is the recurrence's ``[B*H, T, hd]`` output, ``gate`` the gate
    projection ``[B, T, W]`` (its rows may be a channel slice of a wider GEMM
    output), ``norm_weight`` the ``nn.RMSNorm(hd)`` weight.  The result has the
    gate's dtype, the dtype the reference casts the reads to.  On CUDA one
    sm_100a kernel does it (and one its backward); on CPU this runs
    :func:`read_epilogue_torch`.
    """
    if read.ndim != 3 or gate.ndim != 3:
        raise ValueError("read must be [B*H, T, hd] and gate [B, T, W]")
    bh, t, hd = read.shape
    if bh % heads or gate.shape != (bh // heads, t, heads * hd) or norm_weight.numel() != hd:
        raise ValueError("read, gate and norm_weight shapes do not agree")
    if eps is None:
        eps = torch.finfo(gate.dtype).eps
    if not read.is_cuda:
        return read_epilogue_torch(read, gate, norm_weight, heads=heads, eps=eps)
    if read.dtype not in _DTYPES or gate.dtype not in _DTYPES:
        raise TypeError("read_epilogue on CUDA takes float32 or bfloat16 tensors")
    if hd not in (8, 16, 32, 64):
        raise NotImplementedError(f"read_epilogue on CUDA needs head_dim 8, 16, 32 or 64 (got {hd}); "
                                  "use read_epilogue_torch")
    return _ReadEpilogue.apply(read.contiguous(), gate, norm_weight, heads, float(eps))


class _RmsNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        width = x.shape[-1]
        rows = x.numel() // width
        w = weight.detach().float().contiguous()
        out = torch.empty_like(x)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        with torch.cuda.device(x.device):
            _capi.rms_norm(x, _DTYPES[x.dtype], rows, width, w, eps, out, stream)
        ctx.save_for_backward(x, w)
        ctx.dims = (eps, weight.dtype)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, w = ctx.saved_tensors
        eps, w_dtype = ctx.dims
        width = x.shape[-1]
        rows = x.numel() // width
        go = grad_out.to(x.dtype).contiguous()
        gx = torch.empty_like(x)
        gw = torch.empty(width, device=x.device, dtype=torch.float32)
        ws = torch.empty(_capi.rms_norm_partial_floats(rows, width), device=x.device, dtype=torch.float32)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        with torch.cuda.device(x.device):
            _capi.rms_norm_backward(x, _DTYPES[x.dtype], rows, width, w, eps, go, gx, gw, ws, stream)
        return gx, gw.to(w_dtype), None


def rms_norm(x: Tensor, weight: Tensor, eps: Optional[float] = None) -> Tensor:
    """``nn.RMSNorm`` over the last dimension (the mixer's input norm): one
    sm_100a kernel for the forward and one for the backward on CUDA
    (float32 / bfloat16, width 256, 512, 768 or 1024); ``F.rms_norm``
    otherwise.  ``eps=None`` is the dtype's machine epsilon, as in
    ``nn.RMSNorm``."""
    if eps is None:
        eps = torch.finfo(x.dtype).eps
    width = x.shape[-1]
    if (not x.is_cuda or x.dtype not in _DTYPES or width % 256 or width > 1024 or weight.numel() != width):
        return F.rms_norm(x, (width,), weight, eps)
    return _RmsNorm.apply(x.contiguous(), weight, float(eps))


__all__ = ["paper_prologue", "paper_prologue_torch", "read_epilogue", "read_epilogue_torch", "rms_norm"]
