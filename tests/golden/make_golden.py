"""Generate the golden vectors that pin the CPU oracle to catid/bayes-ssm.

Run once in a container where the reference package is importable::

    PYTHONPATH=/path/to/bayes-ssm python tests/golden/make_golden.py

It runs the reference's own PyTorch implementation in FP64 and stores inputs,
outputs and autograd gradients as ``tests/golden/*.npz``.  Inputs are drawn in
FP32 and up-cast, so a FP32 kernel sees bit-identical values.  The fixtures are
committed; neither the tests nor the GPU box need the reference at run time.

Sources exercised (paths within the reference project):

* ``bayes_ssm/bayesian_layer.py:735`` ``bayesian_layer(..., transitions=diag_embed(a),
  optimized=False)`` -- the dense chunked oracle ``_run_chunked`` (:670-732).
* ``bayes_ssm/bayesian_layer.py:360`` ``_core_loop_fixed_diagonal`` -- the
  fixed-dynamics (0.97 / 0.1 / 1.0) core.
* ``bayes_ssm/replay_ssm.py:155`` ``associative_static_bayesian`` -- the
  information-form scan, and its observation-variance rejection (:243-248).
* ``bayes_ssm/bayesian_layer.py:254-340`` -- rotation dynamics (damped 2-D
  rotations per key pair, per-pair process noise), through the dense path
  (``--rotation-only`` regenerates just those fixtures).
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

from bayes_ssm.bayesian_layer import _core_loop_fixed_diagonal, bayesian_layer
from bayes_ssm.replay_ssm import associative_static_bayesian

OUT = Path(__file__).resolve().parent
F64 = torch.float64


def f32(x: torch.Tensor) -> torch.Tensor:
    """Round to FP32 and return as FP64 (exactly representable inputs)."""
    return x.to(torch.float32).to(F64)


def spd(g: torch.Generator, n: int, d: int, scale: float = 1.0) -> torch.Tensor:
    b = torch.randn(n, d, d, generator=g) / math.sqrt(d)
    p = scale * (torch.eye(d) + 0.5 * b @ b.transpose(-1, -2))
    p = f32(p)
    return 0.5 * (p + p.transpose(-1, -2))


def dense_case(name: str, *, seed: int, n: int, t: int, d: int, m: int, chunk: int,
               dist: str, init: str, loss: str, floor: float = 1e-6,
               zero_key_tokens: tuple[int, ...] = ()) -> None:
    g = torch.Generator().manual_seed(seed)
    if dist == "paper":
        # The dynamic paper-feature shapes: unit-norm k, q; sigmoid decay;
        # softplus noise (mixer: bayes_ssm example, BayesianMixer.forward).
        k = F.normalize(torch.randn(n, t, d, generator=g), dim=-1)
        q = F.normalize(torch.randn(n, t, d, generator=g), dim=-1)
        v = torch.randn(n, t, m, generator=g) / math.sqrt(m)
        a = torch.sigmoid(2.0 + torch.randn(n, t, d, generator=g))
        p = F.softplus(-4.0 + torch.randn(n, t, generator=g))
        r = F.softplus(torch.randn(n, t, generator=g)) + 1e-4
    else:  # the reference unit test's distributions
        k = torch.randn(n, t, d, generator=g)
        v = torch.randn(n, t, m, generator=g)
        q = torch.randn(n, t, d, generator=g)
        a = 0.8 + 0.15 * torch.rand(n, t, d, generator=g)
        p = 0.1 + 0.2 * torch.rand(n, t, generator=g)
        r = 0.2 + torch.rand(n, t, generator=g)
    for tok in zero_key_tokens:
        k[:, tok, :] = 0.0
        r[:, tok] = 1e-9  # below the floor: the clamp is active
    if init == "random":
        m0 = torch.randn(n, d, m, generator=g) * 0.3
        p0 = spd(g, n, d)
    else:
        m0 = torch.zeros(n, d, m)
        p0 = torch.eye(d).expand(n, d, d).clone()
    ins = {key: f32(val).requires_grad_() for key, val in
           dict(k=k, v=v, q=q, a=a, p=p, r=r, M0=m0, P0=p0).items()}
    y, mt, pt = bayesian_layer(
        ins["k"], ins["v"], ins["q"], transitions=torch.diag_embed(ins["a"]),
        process_variances=ins["p"], observation_variances=ins["r"],
        initial_mean=ins["M0"], initial_covariance=ins["P0"],
        denominator_floor=floor, chunk_length=chunk, optimized=False,
    )
    if loss == "all":
        total = y.square().mean() + mt.square().mean() + pt.square().mean()
    else:  # readout only: sum of squared readouts
        total = y.square().sum()
    names = ["k", "v", "q", "a", "p", "r", "M0", "P0"]
    grads = torch.autograd.grad(total, [ins[x] for x in names])
    # Gradients of the loss with respect to the three outputs, in closed form;
    # the kernel ABI takes these (gy, gM_T, gP_T) as its backward inputs.
    if loss == "all":
        gy = 2.0 * y.detach() / y.numel()
        gmt = 2.0 * mt.detach() / mt.numel()
        gpt = 2.0 * pt.detach() / pt.numel()
    else:
        gy = 2.0 * y.detach()
        gmt = torch.zeros_like(mt)
        gpt = torch.zeros_like(pt)
    arrays = {f"in_{x}": ins[x].detach().numpy() for x in names}
    arrays.update(out_y=y.detach().numpy(), out_MT=mt.detach().numpy(), out_PT=pt.detach().numpy(),
                  g_y=gy.numpy(), g_MT=gmt.numpy(), g_PT=gpt.numpy())
    arrays.update({f"grad_{x}": gr.numpy() for x, gr in zip(names, grads)})
    arrays.update(floor=np.array(floor), chunk=np.array(chunk), fixed=np.array(0))
    np.savez_compressed(OUT / f"{name}.npz", **arrays)
    print(name, {k_: v_.shape for k_, v_ in arrays.items() if v_.ndim})


def fixed_case(name: str, *, seed: int, n: int, t: int, d: int, m: int) -> None:
    g = torch.Generator().manual_seed(seed)
    k = f32(F.normalize(torch.randn(n, t, d, generator=g), dim=-1)).requires_grad_()
    q = f32(F.normalize(torch.randn(n, t, d, generator=g), dim=-1)).requires_grad_()
    v = f32(torch.randn(n, t, m, generator=g)).requires_grad_()
    m0 = f32(torch.randn(n, d, m, generator=g) * 0.3).requires_grad_()
    p0 = spd(g, n, d).requires_grad_()
    ones = torch.ones(n, t, d, dtype=F64)
    y, mt, pt = _core_loop_fixed_diagonal(k, v, q, ones, ones[..., 0], ones[..., 0], m0, p0, 1e-6)
    total = y.square().mean() + mt.square().mean() + pt.square().mean()
    grads = torch.autograd.grad(total, [k, v, q, m0, p0])
    arrays = dict(in_k=k.detach().numpy(), in_v=v.detach().numpy(), in_q=q.detach().numpy(),
                  in_M0=m0.detach().numpy(), in_P0=p0.detach().numpy(),
                  out_y=y.detach().numpy(), out_MT=mt.detach().numpy(), out_PT=pt.detach().numpy(),
                  g_y=(2.0 * y.detach() / y.numel()).numpy(),
                  g_MT=(2.0 * mt.detach() / mt.numel()).numpy(),
                  g_PT=(2.0 * pt.detach() / pt.numel()).numpy(),
                  grad_k=grads[0].numpy(), grad_v=grads[1].numpy(), grad_q=grads[2].numpy(),
                  grad_M0=grads[3].numpy(), grad_P0=grads[4].numpy(),
                  floor=np.array(1e-6), chunk=np.array(4), fixed=np.array(1))
    np.savez_compressed(OUT / f"{name}.npz", **arrays)
    print(name, "fixed")


def assoc_case(name: str, *, seed: int, n: int, t: int, d: int, m: int, init: str,
               dist: str) -> None:
    g = torch.Generator().manual_seed(seed)
    k = f32(torch.randn(n, t, d, generator=g) / math.sqrt(m))
    q = f32(torch.randn(n, t, d, generator=g) / math.sqrt(m))
    v = f32(torch.randn(n, t, m, generator=g))
    if dist == "config1":
        r = f32(0.5 + torch.rand(n, t, generator=g))
    else:
        r = f32(F.softplus(torch.randn(n, t, generator=g)) + 1e-2)
    if init == "random":
        m0 = f32(torch.randn(n, d, m, generator=g) * 0.3)
        p0 = spd(g, n, d)
    else:
        m0 = torch.zeros(n, d, m, dtype=F64)
        p0 = torch.eye(d, dtype=F64).expand(n, d, d).clone()
    y, mt, pt = associative_static_bayesian(k, v, q, observation_variances=r,
                                            initial_mean=m0, initial_covariance=p0)
    # The same quantity through the dense recurrence (A = I, Q = 0).
    kk, vv, qq, rr = (x.clone().requires_grad_() for x in (k, v, q, r))
    yd, mtd, ptd = bayesian_layer(kk, vv, qq, process_variances=0.0, observation_variances=rr,
                                  initial_mean=m0, initial_covariance=p0,
                                  chunk_length=t, optimized=False)
    total = yd.square().sum()
    gk, gv, gq, gr = torch.autograd.grad(total, [kk, vv, qq, rr])
    arrays = dict(in_k=k.numpy(), in_v=v.numpy(), in_q=q.numpy(), in_r=r.numpy(),
                  in_M0=m0.numpy(), in_P0=p0.numpy(),
                  out_y=y.numpy(), out_MT=mt.numpy(), out_PT=pt.numpy(),
                  dense_y=yd.detach().numpy(), dense_MT=mtd.detach().numpy(),
                  dense_PT=ptd.detach().numpy(),
                  dense_grad_k=gk.numpy(), dense_grad_v=gv.numpy(), dense_grad_q=gq.numpy(),
                  dense_grad_r=gr.numpy(), floor=np.array(1e-6))
    np.savez_compressed(OUT / f"{name}.npz", **arrays)
    print(name, "assoc", tuple(y.shape))


def rotation_case(name: str, *, seed: int, n: int, t: int, d: int, m: int, chunk: int, init: str,
                  loss: str) -> None:
    """``bayesian_layer(..., rotation_radii=, rotation_angles=, optimized=False)``:
    the reference's rotation dynamics (bayesian_layer.py:254-340 with
    make_rotation_dynamics / make_rotation_process_covariances)."""
    g = torch.Generator().manual_seed(seed)
    j = d // 2
    k = F.normalize(torch.randn(n, t, d, generator=g), dim=-1)
    q = F.normalize(torch.randn(n, t, d, generator=g), dim=-1)
    v = torch.randn(n, t, m, generator=g) / math.sqrt(m)
    radii = 0.8 + 0.19 * torch.rand(n, t, j, generator=g)
    angles = 0.5 * torch.randn(n, t, j, generator=g)
    p = F.softplus(-3.0 + torch.randn(n, t, j, generator=g))
    r = F.softplus(torch.randn(n, t, generator=g)) + 1e-2
    if init == "random":
        m0 = torch.randn(n, d, m, generator=g) * 0.3
        p0 = spd(g, n, d)
    else:
        m0 = torch.zeros(n, d, m)
        p0 = torch.eye(d).expand(n, d, d).clone()
    ins = {key: f32(val).requires_grad_() for key, val in
           dict(k=k, v=v, q=q, radii=radii, angles=angles, p=p, r=r, M0=m0, P0=p0).items()}
    y, mt, pt = bayesian_layer(
        ins["k"], ins["v"], ins["q"], rotation_radii=ins["radii"], rotation_angles=ins["angles"],
        process_variances=ins["p"], observation_variances=ins["r"], initial_mean=ins["M0"],
        initial_covariance=ins["P0"], chunk_length=chunk, optimized=False)
    if loss == "all":
        total = y.square().mean() + mt.square().mean() + pt.square().mean()
    else:
        total = y.square().sum()
    names = list(ins)
    grads = torch.autograd.grad(total, [ins[x] for x in names])
    arrays = {f"in_{x}": ins[x].detach().numpy() for x in names}
    arrays.update(out_y=y.detach().numpy(), out_MT=mt.detach().numpy(), out_PT=pt.detach().numpy())
    arrays.update({f"grad_{x}": gr.numpy() for x, gr in zip(names, grads)})
    arrays.update(chunk=np.array(chunk), loss_all=np.array(int(loss == "all")))
    np.savez_compressed(OUT / f"{name}.npz", **arrays)
    print(name, "rotation", tuple(y.shape))


def rotation_cases() -> None:
    rotation_case("rotation_d2m8_all", seed=500, n=2, t=11, d=2, m=8, chunk=4, init="random", loss="all")
    rotation_case("rotation_d4m8_all", seed=501, n=2, t=13, d=4, m=8, chunk=5, init="random", loss="all")
    rotation_case("rotation_d8m8_readout", seed=502, n=2, t=17, d=8, m=8, chunk=8, init="identity",
                  loss="readout")


def main() -> None:
    import sys
    torch.set_default_dtype(F64)
    if "--rotation-only" in sys.argv:
        rotation_cases()
        return
    dense_case("diag_d4m3_all", seed=44, n=2, t=7, d=4, m=3, chunk=3, dist="unit",
               init="random", loss="all")
    dense_case("diag_d3m2_all", seed=45, n=1, t=6, d=3, m=2, chunk=2, dist="unit",
               init="random", loss="all")
    for d in (1, 2, 4, 8):
        dense_case(f"paper_d{d}m8_all", seed=100 + d, n=3, t=13, d=d, m=8, chunk=4,
                   dist="paper", init="random", loss="all")
        dense_case(f"paper_d{d}m8_readout", seed=200 + d, n=2, t=21, d=d, m=8, chunk=8,
                   dist="paper", init="identity", loss="readout")
    dense_case("paper_d8m8_floor", seed=300, n=2, t=9, d=8, m=8, chunk=4, dist="paper",
               init="identity", loss="all", zero_key_tokens=(0, 4))
    fixed_case("fixed_d8m8", seed=400, n=2, t=11, d=8, m=8)
    fixed_case("fixed_d2m8", seed=401, n=2, t=11, d=2, m=8)
    assoc_case("assoc_config1", seed=0, n=1, t=16, d=4, m=4, init="identity", dist="config1")
    assoc_case("assoc_random_init", seed=1, n=2, t=9, d=4, m=3, init="random", dist="softplus")
    assoc_case("assoc_config2_slice", seed=2, n=4, t=64, d=16, m=16, init="identity",
               dist="softplus")
    rotation_cases()


if __name__ == "__main__":
    main()
