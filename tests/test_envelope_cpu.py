"""CPU: the BayesianMixer prologue's PyTorch op chain and its argument checks.

``paper_prologue_torch`` restates ``example/train_6layer.py:579-700``; here it
is checked against an independent restatement that uses ``nn.Conv1d`` with
left padding 3 (the reference's non-fast path, :474-480) and the reference's
own per-op order, so the CUDA parity tests have a pinned PyTorch reference.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from bayes_ssm.envelope import paper_prologue, paper_prologue_torch


def _inputs(b, t, h, d, hd, seed=0):
    g = torch.Generator().manual_seed(seed)
    sw, w = h * d, h * hd
    c, aux = 2 * sw + w, sw + 2 * h
    x = torch.randn(b, t, c + aux, generator=g)
    wt = torch.randn(c, 1, 4, generator=g) * 0.5
    bias = torch.randn(aux, generator=g) * 0.1
    return x, wt, bias


def _conv1d_reference(x, wt, bias, h, d, hd):
    b, t, _ = x.shape
    sw, w = h * d, h * hd
    c = 2 * sw + w
    conv = torch.nn.Conv1d(c, c, kernel_size=4, groups=c, bias=False)
    with torch.no_grad():
        conv.weight.copy_(wt)
    y = conv(F.pad(x[..., :c].transpose(1, 2), (3, 0))).transpose(1, 2)
    qi, ki, vi = y.split((sw, sw, w), dim=-1)
    q = F.normalize(F.silu(qi).view(b, t, h, d), dim=-1).permute(0, 2, 1, 3).reshape(b * h, t, d)
    k = F.normalize(F.silu(ki).view(b, t, h, d), dim=-1).permute(0, 2, 1, 3).reshape(b * h, t, d)
    v = F.silu(vi).view(b, t, h, hd).permute(0, 2, 1, 3).reshape(b * h, t, hd)
    aux = x[..., c:] + bias
    noise = aux[..., sw:].view(b, t, h, 2)
    proc = (F.softplus(noise[..., 0]) + 1e-4).permute(0, 2, 1).reshape(b * h, t)
    obs = (F.softplus(noise[..., 1]) + 1e-4).permute(0, 2, 1).reshape(b * h, t)
    dec = torch.exp(-F.softplus(aux[..., :sw])).view(b, t, h, d).permute(0, 2, 1, 3).reshape(b * h, t, d)
    return k, q, v, dec, proc, obs


@pytest.mark.parametrize("shape", [(2, 9, 3, 4, 6), (1, 5, 2, 8, 8), (3, 2, 1, 2, 2)])
def test_torch_chain_matches_conv1d_restatement(shape):
    b, t, h, d, hd = shape
    x, wt, bias = _inputs(b, t, h, d, hd, seed=t)
    got = paper_prologue_torch(x, wt, bias, heads=h, key_dim=d, head_dim=hd)
    want = _conv1d_reference(x, wt, bias, h, d, hd)
    for g, w_ in zip(got, want):
        assert g.shape == w_.shape
        torch.testing.assert_close(g, w_, rtol=1e-5, atol=1e-6)


def test_cpu_call_is_the_torch_chain_with_gradients():
    x, wt, bias = _inputs(2, 7, 2, 4, 4, seed=3)
    x.requires_grad_()
    wt.requires_grad_()
    out = paper_prologue(x, wt, bias, heads=2, key_dim=4, head_dim=4)
    ref = paper_prologue_torch(x, wt, bias, heads=2, key_dim=4, head_dim=4)
    for a, b in zip(out, ref):
        torch.testing.assert_close(a, b)
    sum(o.square().sum() for o in out).backward()
    assert x.grad is not None and wt.grad is not None and torch.isfinite(x.grad).all()


def test_argument_errors():
    x, wt, bias = _inputs(1, 4, 2, 4, 4)
    with pytest.raises(ValueError, match="channels"):
        paper_prologue(x[..., :-1], wt, bias, heads=2, key_dim=4, head_dim=4)
    with pytest.raises(ValueError, match="conv_weight"):
        paper_prologue(x, wt[:-1], bias, heads=2, key_dim=4, head_dim=4)
    with pytest.raises(ValueError, match="aux_bias"):
        paper_prologue(x, wt, bias[:-1], heads=2, key_dim=4, head_dim=4)
    with pytest.raises(ValueError, match="batch, tokens, channels"):
        paper_prologue(x[0], wt, bias, heads=2, key_dim=4, head_dim=4)


def test_read_epilogue_torch_matches_module_chain():
    """read_epilogue_torch is the reference's readout: nn.RMSNorm(hd) on the
    permuted, dtype-cast reads times SiLU(gate)."""
    from bayes_ssm.envelope import read_epilogue, read_epilogue_torch
    g = torch.Generator().manual_seed(9)
    b, t, h, hd = 2, 6, 3, 8
    read = torch.randn(b * h, t, hd, generator=g)
    gate = torch.randn(b, t, h * hd, generator=g)
    norm = torch.nn.RMSNorm(hd)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(hd, generator=g) + 0.5)
    want = (norm(read.view(b, h, t, hd).permute(0, 2, 1, 3)) * F.silu(gate.view(b, t, h, hd))).reshape(b, t, h * hd)
    got = read_epilogue_torch(read, gate, norm.weight, heads=h)
    torch.testing.assert_close(got, want)
    torch.testing.assert_close(read_epilogue(read, gate, norm.weight, heads=h), want)
    with pytest.raises(ValueError, match="shapes"):
        read_epilogue(read, gate[..., :-1], norm.weight, heads=h)
