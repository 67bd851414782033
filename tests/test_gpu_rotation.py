"""GPU: the rotation-dynamics kernels (bssm_rotation.cu) through the public
API, against the reference's FP64 fixtures and against the API's own dense
path in FP64 on larger seeded cases (that path is pinned to the reference by
tests/test_rotation_cpu.py).  Tolerance: relative L2 <= 1e-5, cosine >=
0.99999 for every output and gradient, radii and angles included."""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from conftest import GOLDEN
from harness import assert_parity
from test_rotation_cpu import NAMES, run_fixture

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("rotation_*.npz")))
def test_rotation_kernels_match_reference_fixtures(name):
    from bayes_ssm import _capi
    g, (y, mt, pt), grads = run_fixture(name, device="cuda", dtype=torch.float32, optimized=True)
    assert_parity(y, g["out_y"], what="y")
    assert_parity(mt, g["out_MT"], what="M_T")
    assert_parity(pt, g["out_PT"], what="P_T")
    for x in NAMES:
        assert_parity(grads[x], g[f"grad_{x}"], what=f"grad {x}")
    _capi.stream_status(torch.cuda.current_stream().cuda_stream)


def _inputs(n, t, d, m, seed):
    g = torch.Generator().manual_seed(seed)
    j = d // 2
    return dict(k=F.normalize(torch.randn(n, t, d, generator=g), dim=-1),
                v=torch.randn(n, t, m, generator=g) / math.sqrt(m),
                q=F.normalize(torch.randn(n, t, d, generator=g), dim=-1),
                radii=0.85 + 0.2 * torch.rand(n, t, j, generator=g),  # some above 1: clamped
                angles=0.4 * torch.randn(n, t, j, generator=g),
                p=F.softplus(-3.0 + torch.randn(n, t, j, generator=g)),
                r=F.softplus(torch.randn(n, t, generator=g)) + 1e-3)


def _run(inp, device, dtype, chunk, optimized):
    import bayes_ssm
    leaves = {x: v.to(device=device, dtype=dtype).requires_grad_() for x, v in inp.items()}
    y, mt, pt = bayes_ssm.bayesian_layer(leaves["k"], leaves["v"], leaves["q"], rotation_radii=leaves["radii"],
                                         rotation_angles=leaves["angles"], process_variances=leaves["p"],
                                         observation_variances=leaves["r"], chunk_length=chunk,
                                         optimized=optimized)
    total = y.square().mean() + mt.square().mean() + pt.square().mean()
    return (y, mt, pt), dict(zip(leaves, torch.autograd.grad(total, list(leaves.values()))))


@pytest.mark.parametrize("d", (2, 4, 8))
@pytest.mark.parametrize("t,chunk", [(1, 1), (37, 16), (70, 64), (9, 4)])
def test_rotation_kernels_match_dense_path(d, t, chunk):
    inp = _inputs(5, t, d, 8, seed=10 * d + t)
    (y, mt, pt), g = _run(inp, "cuda", torch.float32, chunk, True)
    (y0, mt0, pt0), g0 = _run(inp, "cpu", torch.float64, chunk, False)
    assert_parity(y, y0.detach().numpy(), what="y")
    assert_parity(mt, mt0.detach().numpy(), what="M_T")
    assert_parity(pt, pt0.detach().numpy(), what="P_T")
    for x in g:
        want = g0[x].numpy()
        if abs(want).max() < 1e-12:
            # analytically zero (one token from the identity covariance and a
            # zero mean: the rotation has no effect): FP32 rounding only
            assert g[x].abs().max().item() < 1e-6, x
            continue
        assert_parity(g[x], want, what=f"grad {x}")


def test_rotation_batch_shape_and_bf16_promotion():
    inp = _inputs(6, 12, 4, 8, seed=3)
    shaped = {x: v.view(2, 3, *v.shape[1:]) for x, v in inp.items()}
    (y, _, _), _ = _run(shaped, "cuda", torch.float32, 5, True)
    (y1, _, _), _ = _run(inp, "cuda", torch.float32, 5, True)
    assert torch.equal(y.reshape(6, 12, 8), y1)
    import bayes_ssm
    leaves = {x: (v.cuda() if x not in "kvq" else v.cuda().bfloat16()) for x, v in inp.items()}
    yb, _, _ = bayes_ssm.bayesian_layer(leaves["k"], leaves["v"], leaves["q"], rotation_radii=leaves["radii"],
                                        rotation_angles=leaves["angles"], process_variances=leaves["p"],
                                        observation_variances=leaves["r"], chunk_length=5, optimized=True)
    yf, _, _ = bayes_ssm.bayesian_layer(leaves["k"].float(), leaves["v"].float(), leaves["q"].float(),
                                        rotation_radii=leaves["radii"], rotation_angles=leaves["angles"],
                                        process_variances=leaves["p"], observation_variances=leaves["r"],
                                        chunk_length=5, optimized=True)
    assert torch.equal(yb, yf)
