"""The BayesianMixer layer of catid/bayes-ssm's trainer, on this package's kernels.

``example/train_6layer.py:196-729`` defines ``BayesianMixer``; this is its
default production configuration: paper features, learned diagonal dynamics,
the fused Q/K/V + auxiliary projection (``fuse_paper_qkv``,
``fuse_paper_projection``) and a separate gate projection.  Parameter names,
shapes and initial values are the reference's (``:226-464``), so state dicts
load either way:

``norm`` (RMSNorm over the width), ``qkv_proj`` (bias-free Linear to
``2*H*D + W + H*D + 2*H`` rows: q, k, v, decay logits, noise pairs),
``aux_bias`` (the auxiliary rows' bias), ``qkv_conv`` (depthwise Conv1d weight
``[2*H*D + W, 1, 4]``, initialised to the identity tap), ``read_norm``
(RMSNorm over the head), ``g_proj`` and ``out_proj`` (bias-free Linears).

Forward (``:579-729``): RMSNorm -> projection GEMM -> the fused prologue
(:func:`bayes_ssm.envelope.paper_prologue`) -> :func:`bayesian_layer` on the
recurrence kernels -> the fused readout (:func:`bayes_ssm.envelope.read_epilogue`)
-> output GEMM.  The input RMSNorm is this package's kernel pair
(:func:`bayes_ssm.envelope.rms_norm`); the GEMMs are PyTorch's (cuBLAS).
``fused_envelope=False`` runs the norm, prologue and readout as the
reference's PyTorch ops instead, for comparison.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
from torch import Tensor, nn

from .bayesian_layer import bayesian_layer
from .envelope import paper_prologue, paper_prologue_torch, read_epilogue, read_epilogue_torch, rms_norm


class BayesianMixer(nn.Module):
    def __init__(self, width: int, heads: int, *, key_dim: Optional[int] = None, chunk_length: int = 64,
                 optimized: bool = True, bf16_state_io: bool = False, fused_envelope: bool = True,
                 dtype: torch.dtype = torch.bfloat16, device=None) -> None:
        super().__init__()
        if width % heads:
            raise ValueError("width must be divisible by heads")
        self.width, self.heads, self.head_dim = width, heads, width // heads
        self.key_dim = self.head_dim if key_dim is None else key_dim
        if not 0 < self.key_dim <= self.head_dim:
            raise ValueError("key_dim must be in [1, width // heads]")
        self.state_width = heads * self.key_dim
        self.chunk_length = chunk_length
        self.optimized = optimized
        # BF16 keys/queries/values at the state boundary (the recurrence still
        # computes in FP32); False keeps the reference's FP32 boundary
        self.bf16_state_io = bf16_state_io
        self.fused_envelope = fused_envelope
        self.qkv_core_width = 2 * self.state_width + width
        self.aux_width = self.state_width + 2 * heads
        kw = dict(dtype=dtype, device=device)
        self.norm = nn.RMSNorm(width, **kw)
        self.qkv_proj = nn.Linear(width, self.qkv_core_width + self.aux_width, bias=False, **kw)
        self.aux_bias = nn.Parameter(torch.zeros(self.aux_width, **kw))
        conv_channels = self.qkv_core_width
        self.qkv_conv = nn.Conv1d(conv_channels, conv_channels, kernel_size=4, groups=conv_channels, bias=False,
                                  **kw)
        self.out_proj = nn.Linear(width, width, bias=False, **kw)
        self.read_norm = nn.RMSNorm(self.head_dim, **kw)
        self.g_proj = nn.Linear(width, width, bias=False, **kw)
        with torch.no_grad():
            # identity causal filter (the last tap is the current token)
            self.qkv_conv.weight.zero_()
            self.qkv_conv.weight[:, 0, -1] = 1
            # decay half-lives over 32..4096 tokens: rho = exp(-softplus(raw))
            half_lives = torch.logspace(math.log10(32.0), math.log10(4096.0), self.state_width,
                                        device=self.aux_bias.device, dtype=torch.float32)
            raw = torch.log(torch.expm1(math.log(2.0) / half_lives))
            self.qkv_proj.weight[self.qkv_core_width:].zero_()
            self.aux_bias[:self.state_width].copy_(raw.to(dtype))
            self.aux_bias[self.state_width::2].fill_(math.log(math.expm1(0.1)))
            self.aux_bias[self.state_width + 1::2].fill_(math.log(math.expm1(1.0)))

    def forward(self, x: Tensor) -> Tensor:
        z = rms_norm(x, self.norm.weight, self.norm.eps) if self.fused_envelope else self.norm(x)
        projected = self.qkv_proj(z)
        kw = dict(heads=self.heads, key_dim=self.key_dim, head_dim=self.head_dim)
        if self.fused_envelope and projected.is_cuda:
            out_dtype = torch.bfloat16 if self.bf16_state_io else torch.float32
            k, q, v, decay, process, observation = paper_prologue(projected, self.qkv_conv.weight, self.aux_bias,
                                                                  out_dtype=out_dtype, **kw)
        else:
            k, q, v, decay, process, observation = paper_prologue_torch(projected, self.qkv_conv.weight,
                                                                        self.aux_bias, **kw)
        read, _, _ = bayesian_layer(k, v, q, transition_diagonals=decay, process_variances=process,
                                    observation_variances=observation, chunk_length=self.chunk_length,
                                    optimized=self.optimized)
        gate = self.g_proj(z)
        if self.fused_envelope and read.is_cuda:
            y = read_epilogue(read, gate, self.read_norm.weight, heads=self.heads, eps=self.read_norm.eps)
        else:
            eps = self.read_norm.eps if self.read_norm.eps is not None else torch.finfo(gate.dtype).eps
            y = read_epilogue_torch(read, gate, self.read_norm.weight, heads=self.heads, eps=eps)
        return self.out_proj(y)


__all__ = ["BayesianMixer"]
