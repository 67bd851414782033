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


def test_rotation_coefficients_match_the_reference_chain():
    """The fused coefficient kernels against the reference's own operations
    (radii clamped to [tiny, 1], exp(log(radius)) clipped at 1, times cos and
    sin of the angles): values and both gradients, on radii below tiny, zero,
    negative, exactly 1, above 1 and ordinary, and angles of any size."""
    from bayes_ssm.rotation_cuda import coefficients_apply, rotation_coefficients
    g = torch.Generator().manual_seed(3)
    radii = 0.2 + 1.0 * torch.rand(4, 300, 4, generator=g)
    angles = 6.0 * torch.randn(4, 300, 4, generator=g)
    flat = radii.view(-1)
    flat[:6] = torch.tensor([0.0, -0.5, 1e-40, 1.0, 1.0000001, 3.0])
    radii, angles = radii.cuda(), angles.cuda()
    assert coefficients_apply(radii, angles)
    up_c = torch.randn(radii.shape, generator=g).cuda()
    up_s = torch.randn(radii.shape, generator=g).cuda()

    def reference(r, a):
        radius = r.clamp_min(torch.finfo(torch.float32).tiny)
        radius = torch.where(radius <= 1.0, radius, torch.ones_like(radius))
        raw = torch.log(radius).exp()
        rho = torch.where(raw <= 1.0, raw, torch.ones_like(raw))
        return rho * a.cos(), rho * a.sin()

    rk, ak = radii.clone().requires_grad_(), angles.clone().requires_grad_()
    rr, ar = radii.clone().requires_grad_(), angles.clone().requires_grad_()
    ck, sk = rotation_coefficients(rk, ak)
    cr, sr = reference(rr, ar)
    gk = torch.autograd.grad((ck, sk), (rk, ak), (up_c, up_s))
    gr = torch.autograd.grad((cr, sr), (rr, ar), (up_c, up_s))
    for name, a_, b_ in (("cos", ck, cr), ("sin", sk, sr), ("grad radii", gk[0], gr[0]), ("grad angles", gk[1], gr[1])):
        torch.testing.assert_close(a_, b_, rtol=1e-6, atol=1e-7, msg=name)
    # only the sine gradient given: the cosine's is taken as zero
    gk1 = torch.autograd.grad(rotation_coefficients(rk, ak)[1], (rk, ak), up_s)
    gr1 = torch.autograd.grad(reference(rr, ar)[1], (rr, ar), up_s)
    for a_, b_ in zip(gk1, gr1):
        torch.testing.assert_close(a_, b_, rtol=1e-6, atol=1e-7)
