"""CPU: the BayesianMixer layer's parameters and forward against the
reference module's op chain (``example/train_6layer.py:579-729``) written out
with ``nn.Conv1d`` and ``nn.RMSNorm`` on the same parameters."""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from bayes_ssm import bayesian_layer
from bayes_ssm.mixer import BayesianMixer


def test_parameter_names_shapes_and_init():
    m = BayesianMixer(64, 4, key_dim=8, dtype=torch.float32)
    shapes = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    sw, w, h = 32, 64, 4
    assert shapes == {"norm.weight": (w,), "qkv_proj.weight": (2 * sw + w + sw + 2 * h, w),
                      "aux_bias": (sw + 2 * h,), "qkv_conv.weight": (2 * sw + w, 1, 4),
                      "out_proj.weight": (w, w), "read_norm.weight": (w // h,), "g_proj.weight": (w, w)}
    assert torch.equal(m.qkv_conv.weight[:, 0, :3], torch.zeros(2 * sw + w, 3))
    assert torch.equal(m.qkv_conv.weight[:, 0, 3], torch.ones(2 * sw + w))
    assert torch.count_nonzero(m.qkv_proj.weight[2 * sw + w:]) == 0
    torch.testing.assert_close(F.softplus(m.aux_bias[sw::2]), torch.full((h,), 0.1))
    torch.testing.assert_close(F.softplus(m.aux_bias[sw + 1::2]), torch.full((h,), 1.0))
    rho = torch.exp(-F.softplus(m.aux_bias[:sw]))
    torch.testing.assert_close(rho[0], torch.tensor(0.5 ** (1 / 32.0)))


def _reference_forward(m, x):
    b, t, _ = x.shape
    h, hd, d, sw, w = m.heads, m.head_dim, m.key_dim, m.state_width, m.width
    z = m.norm(x)
    projected = m.qkv_proj(z)
    qkv = projected[..., :m.qkv_core_width]
    aux = projected[..., m.qkv_core_width:m.qkv_core_width + m.aux_width] + m.aux_bias
    conv = m.qkv_conv(F.pad(qkv.transpose(1, 2), (3, 0))).transpose(1, 2)
    qi, ki, vi = conv.split((sw, sw, w), dim=-1)
    q = F.normalize(F.silu(qi.float()).view(b, t, h, d), dim=-1).permute(0, 2, 1, 3).reshape(b * h, t, d)
    k = F.normalize(F.silu(ki.float()).view(b, t, h, d), dim=-1).permute(0, 2, 1, 3).reshape(b * h, t, d)
    v = F.silu(vi.float()).view(b, t, h, hd).permute(0, 2, 1, 3).reshape(b * h, t, hd)
    noise = aux[..., sw:].float().view(b, t, h, 2)
    proc = (F.softplus(noise[..., 0]) + 1e-4).permute(0, 2, 1).reshape(b * h, t)
    obs = (F.softplus(noise[..., 1]) + 1e-4).permute(0, 2, 1).reshape(b * h, t)
    dec = torch.exp(-F.softplus(aux[..., :sw].float())).view(b, t, h, d).permute(0, 2, 1, 3).reshape(b * h, t, d)
    read, _, _ = bayesian_layer(k, v, q, transition_diagonals=dec, process_variances=proc,
                                observation_variances=obs, chunk_length=m.chunk_length, optimized=False)
    read = m.read_norm(read.view(b, h, t, hd).permute(0, 2, 1, 3).to(x.dtype))
    gate = m.g_proj(z).view(b, t, h, hd)
    return m.out_proj((read * F.silu(gate)).reshape(b, t, w))


def test_forward_matches_reference_chain():
    torch.manual_seed(0)
    m = BayesianMixer(32, 4, key_dim=4, chunk_length=8, dtype=torch.float32)
    with torch.no_grad():  # move off the initial values so every path matters
        for p in m.parameters():
            p.add_(0.05 * torch.randn_like(p))
    x = torch.randn(2, 11, 32)
    torch.testing.assert_close(m(x), _reference_forward(m, x), rtol=1e-4, atol=1e-5)


def test_state_dict_round_trip():
    a = BayesianMixer(32, 4, key_dim=4, dtype=torch.float32)
    b = BayesianMixer(32, 4, key_dim=4, dtype=torch.float32)
    with torch.no_grad():
        for p in a.parameters():
            p.add_(torch.randn_like(p))
    b.load_state_dict(a.state_dict(), strict=True)
    x = torch.randn(1, 5, 32)
    torch.testing.assert_close(a(x), b(x))
    assert math.isfinite(float(b(x).detach().sum()))
