"""The six-layer hybrid language model of catid/bayes-ssm's trainer, on this
package's kernels: the caller of the recurrence in BASELINE config 5.

Architecture (``example/train_6layer.py``): token embedding (``:823-824``,
N(0, 0.02)), six pre-norm residual blocks -- Bayesian mixer, Bayesian mixer,
causal GQA attention, Bayesian mixer, Bayesian mixer, causal GQA attention
(``SixLayerLM.block_kinds`` :797) -- each followed by a SwiGLU MLP
(``HybridBlock`` :744-790, ``SwiGLU`` :730-741), a final RMSNorm and the tied
head computed in FP32 (``:844-850``).  Module and parameter names follow the
reference so state dicts load either way.  Defaults are the reference's
(vocab 32,000, width 512, 64 heads, 4 KV heads, MLP width 8,448: about
101.94 M parameters), in BF16.

The Bayesian blocks are :class:`bayes_ssm.mixer.BayesianMixer` (fused
prologue, the recurrence kernels, fused readout); every RMSNorm is the
package's kernel pair (:func:`bayes_ssm.envelope.rms_norm`); attention is
PyTorch SDPA and the GEMMs are PyTorch's (cuBLAS).  :func:`train_step` is the
reference's step (``:1087-1099``): cross-entropy over the FP32 logits,
backward, gradient clipping, AdamW.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .envelope import rms_norm
from .mixer import BayesianMixer


class RMSNorm(nn.RMSNorm):
    """``nn.RMSNorm`` whose forward runs the package's kernels on CUDA."""

    def forward(self, x: Tensor) -> Tensor:
        return rms_norm(x, self.weight, self.eps)


class GQAAttention(nn.Module):
    """Causal grouped-query attention (``train_6layer.py:122-157``)."""

    def __init__(self, width: int, heads: int, kv_heads: int, *, dtype=torch.bfloat16, device=None) -> None:
        super().__init__()
        if width % heads or heads % kv_heads:
            raise ValueError("width must be divisible by heads; kv_heads must divide heads")
        self.width, self.heads, self.kv_heads = width, heads, kv_heads
        self.head_dim = width // heads
        kw = dict(dtype=dtype, device=device)
        self.norm = RMSNorm(width, **kw)
        self.q_proj = nn.Linear(width, width, bias=False, **kw)
        self.k_proj = nn.Linear(width, kv_heads * self.head_dim, bias=False, **kw)
        self.v_proj = nn.Linear(width, kv_heads * self.head_dim, bias=False, **kw)
        self.out_proj = nn.Linear(width, width, bias=False, **kw)

    def forward(self, x: Tensor) -> Tensor:
        z = self.norm(x)
        b, t, _ = z.shape
        q = self.q_proj(z).view(b, t, self.heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(z).view(b, t, self.kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(z).view(b, t, self.kv_heads, self.head_dim).transpose(1, 2)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        return self.out_proj(y.transpose(1, 2).reshape(b, t, self.width))


class SwiGLU(nn.Module):
    """``down(silu(gate(z)) * up(z))`` over the normed input (:730-741)."""

    def __init__(self, width: int, mlp_width: int, *, dtype=torch.bfloat16, device=None) -> None:
        super().__init__()
        kw = dict(dtype=dtype, device=device)
        self.norm = RMSNorm(width, **kw)
        self.gate = nn.Linear(width, mlp_width, bias=False, **kw)
        self.up = nn.Linear(width, mlp_width, bias=False, **kw)
        self.down = nn.Linear(mlp_width, width, bias=False, **kw)

    def forward(self, x: Tensor) -> Tensor:
        z = self.norm(x)
        return self.down(F.silu(self.gate(z)) * self.up(z))


class HybridBlock(nn.Module):
    def __init__(self, kind: str, width: int, heads: int, kv_heads: int, mlp_width: int, *, chunk_length: int,
                 key_dim: int | None, optimized: bool, dtype, device) -> None:
        super().__init__()
        self.kind = kind
        if kind == "bayesian":
            self.mixer = BayesianMixer(width, heads, key_dim=key_dim, chunk_length=chunk_length,
                                       optimized=optimized, dtype=dtype, device=device)
        elif kind == "fa":
            self.mixer = GQAAttention(width, heads, kv_heads, dtype=dtype, device=device)
        else:
            raise ValueError(f"unknown block kind {kind!r}")
        self.ffn = SwiGLU(width, mlp_width, dtype=dtype, device=device)

    def forward(self, x: Tensor) -> Tensor:
        x = x + self.mixer(x)
        return x + self.ffn(x)


class SixLayerLM(nn.Module):
    """Six blocks: Bayesian, Bayesian, FA-GQA, Bayesian, Bayesian, FA-GQA."""

    block_kinds = ("bayesian", "bayesian", "fa", "bayesian", "bayesian", "fa")

    def __init__(self, vocab_size: int = 32_000, width: int = 512, heads: int = 64, kv_heads: int = 4,
                 mlp_width: int = 8448, *, chunk_length: int = 64, key_dim: int | None = None,
                 optimized: bool = True, dtype: torch.dtype = torch.bfloat16, device=None) -> None:
        super().__init__()
        self.vocab_size, self.width = vocab_size, width
        self.embedding = nn.Embedding(vocab_size, width, dtype=dtype, device=device)
        nn.init.normal_(self.embedding.weight, mean=0.0, std=0.02)
        self.blocks = nn.ModuleList(
            HybridBlock(kind, width, heads, kv_heads, mlp_width, chunk_length=chunk_length, key_dim=key_dim,
                        optimized=optimized, dtype=dtype, device=device)
            for kind in self.block_kinds)
        self.final_norm = RMSNorm(width, dtype=dtype, device=device)

    def forward(self, tokens: Tensor) -> Tensor:
        x = self.embedding(tokens)
        for block in self.blocks:
            x = block(x)
        # the tied head runs in FP32 (:850)
        return self.final_norm(x).float() @ self.embedding.weight.float().t()


def parameter_count(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())


def make_optimizer(model: nn.Module, *, lr: float = 3e-4, weight_decay: float = 0.1) -> torch.optim.Optimizer:
    """AdamW(0.9, 0.95), fused on CUDA (:1063-1067)."""
    cuda = next(model.parameters()).is_cuda
    return torch.optim.AdamW(model.parameters(), lr=lr, betas=(0.9, 0.95), weight_decay=weight_decay, fused=cuda)


def train_step(model: nn.Module, optimizer: torch.optim.Optimizer, inputs: Tensor, targets: Tensor, *,
               vocab_size: int, grad_clip: float = 1.0) -> Tensor:
    """One optimisation step (:1087-1099); returns the loss (on the device)."""
    optimizer.zero_grad(set_to_none=False)
    logits = model(inputs)
    loss = F.cross_entropy(logits.reshape(-1, vocab_size), targets.reshape(-1))
    loss.backward()
    if grad_clip > 0:
        nn.utils.clip_grad_norm_(model.parameters(), grad_clip)
    optimizer.step()
    return loss.detach()


__all__ = ["SixLayerLM", "GQAAttention", "SwiGLU", "HybridBlock", "RMSNorm", "parameter_count", "make_optimizer",
           "train_step"]
