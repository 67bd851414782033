"""CPU: rotation dynamics through the public API's dense path (FP64) against
the reference's own FP64 outputs and gradients (tests/golden/rotation_*.npz,
made by tests/golden/make_golden.py from bayes_ssm/bayesian_layer.py:254-340).
This pins the PyTorch reference the rotation kernels are checked against."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN

NAMES = ("k", "v", "q", "radii", "angles", "p", "r", "M0", "P0")


def run_fixture(name, device="cpu", dtype=torch.float64, optimized=False):
    import bayes_ssm
    with np.load(GOLDEN / f"{name}.npz") as z:
        g = {k: z[k] for k in z.files}
    ins = {x: torch.from_numpy(g[f"in_{x}"]).to(device=device, dtype=dtype).requires_grad_() for x in NAMES}
    y, mt, pt = bayes_ssm.bayesian_layer(
        ins["k"], ins["v"], ins["q"], rotation_radii=ins["radii"], rotation_angles=ins["angles"],
        process_variances=ins["p"], observation_variances=ins["r"], initial_mean=ins["M0"],
        initial_covariance=ins["P0"], chunk_length=int(g["chunk"]), optimized=optimized)
    if int(g["loss_all"]):
        total = y.square().mean() + mt.square().mean() + pt.square().mean()
    else:
        total = y.square().sum()
    grads = torch.autograd.grad(total, [ins[x] for x in NAMES])
    return g, (y, mt, pt), dict(zip(NAMES, grads))


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("rotation_*.npz")))
def test_dense_rotation_matches_reference(name):
    g, (y, mt, pt), grads = run_fixture(name)
    np.testing.assert_allclose(y.detach().numpy(), g["out_y"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(mt.detach().numpy(), g["out_MT"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(pt.detach().numpy(), g["out_PT"], rtol=1e-10, atol=1e-12)
    for x in NAMES:
        np.testing.assert_allclose(grads[x].numpy(), g[f"grad_{x}"], rtol=1e-9, atol=1e-11, err_msg=x)
