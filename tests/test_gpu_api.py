"""GPU: the public ``bayes_ssm`` API (autograd boundary) on the kernels, and
the static associative scan kernel, vs the FP64 oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from harness import assert_parity, make_inputs, to_np64
from oracle import oracle

pytestmark = pytest.mark.gpu


def _api(inp, **kw):
    import bayes_ssm
    return bayes_ssm.bayesian_layer(inp["k"], inp["v"], inp["q"], transition_diagonals=inp["a"],
                                    process_variances=inp["p"], observation_variances=inp["r"],
                                    **kw)


def _leaf(inp, device="cuda"):
    return {k: (None if v is None else v.detach().to(device).requires_grad_())
            for k, v in inp.items()}


@pytest.mark.parametrize("d", (1, 2, 4, 8))
def test_api_autograd_matches_oracle(d):
    inp = _leaf(make_inputs(12, 37, d, 8, seed=d, init="random"))
    y, mt, pt = _api(inp, initial_mean=inp["M0"], initial_covariance=inp["P0"], chunk_length=8,
                     optimized=True)
    loss = y.square().mean() + mt.square().mean() + pt.square().mean()
    names = ("k", "v", "q", "a", "p", "r", "M0", "P0")
    grads = torch.autograd.grad(loss, [inp[x] for x in names])
    ref = oracle.forward(*[to_np64(inp[x]) for x in names])
    assert_parity(y, ref[0], what="y")
    gy = 2 * ref[0] / ref[0].size
    gmt = 2 * ref[1] / ref[1].size
    gpt = 2 * ref[2] / ref[2].size
    rg = oracle.backward(*[to_np64(inp[x]) for x in names], gy, gmt, gpt)
    for x, g in zip(names, grads):
        assert_parity(g, rg[x], what=f"grad {x}")


def test_api_large_batch_default_kernels(monkeypatch):
    """At 4,096+ chains the default dispatch picks the thread-per-chain family
    (forward saving replay states, backward consuming them)."""
    monkeypatch.delenv("BSSM_KERNELS", raising=False)
    inp = make_inputs(4096, 24, 8, 8, seed=11, io_dtype=torch.bfloat16)
    leaf = _leaf(inp)
    y, _, _ = _api(leaf, chunk_length=16, optimized=True)
    names = ("k", "v", "q", "a", "p", "r")
    grads = torch.autograd.grad(y.square().mean(), [leaf[x] for x in names])
    ref = oracle.forward(*[to_np64(inp[x]) for x in names], None, None)
    assert_parity(y, ref[0], what="y")
    gy = 2 * ref[0] / ref[0].size
    rg = oracle.backward(*[to_np64(inp[x]) for x in names], None, None, gy, None, None)
    for x, g in zip(names, grads):
        assert_parity(g, rg[x], rel=4e-3 if x in ("k", "v", "q") else 1e-5, what=f"grad {x}")


def test_api_bf16_projection_path_equals_promoted_fp32():
    """BF16 k/q/v enter the kernel directly; same values as promoting first."""
    inp = make_inputs(16, 33, 8, 8, seed=3, io_dtype=torch.bfloat16)
    a = _leaf(inp)
    b = {k: (None if v is None else v.detach().clone().requires_grad_()) for k, v in a.items()}
    ya, _, _ = _api(a, chunk_length=16, optimized=True)
    yb, _, _ = _api({**b, "k": b["k"].float(), "v": b["v"].float(), "q": b["q"].float()},
                    chunk_length=16, optimized=True)
    assert torch.equal(ya, yb)
    ga = torch.autograd.grad(ya.square().sum(), [a["k"], a["v"], a["q"], a["a"]])
    gb = torch.autograd.grad(yb.square().sum(), [b["k"], b["v"], b["q"], b["a"]])
    for x, y in zip(ga, gb):
        assert x.dtype == y.dtype
        assert torch.equal(x, y)


def test_api_batch_shape_and_broadcast_noise():
    import bayes_ssm
    g = torch.Generator().manual_seed(0)
    k = torch.nn.functional.normalize(torch.randn(2, 3, 20, 4, generator=g), dim=-1).cuda()
    v = torch.randn(2, 3, 20, 8, generator=g).cuda()
    q = torch.nn.functional.normalize(torch.randn(2, 3, 20, 4, generator=g), dim=-1).cuda()
    a = torch.sigmoid(torch.randn(3, 20, 4, generator=g) + 2).cuda()
    y, mt, pt = bayes_ssm.bayesian_layer(k, v, q, transition_diagonals=a, process_variances=0.01,
                                         observation_variances=0.5, chunk_length=6, optimized=True)
    assert y.shape == (2, 3, 20, 8) and mt.shape == (2, 3, 4, 8) and pt.shape == (2, 3, 4, 4)
    ae = a.expand(2, 3, 20, 4).reshape(6, 20, 4)
    ref = oracle.forward(to_np64(k.reshape(6, 20, 4)), to_np64(v.reshape(6, 20, 8)),
                         to_np64(q.reshape(6, 20, 4)), to_np64(ae), np.full((6, 20), 0.01),
                         np.full((6, 20), 0.5))
    assert_parity(y.reshape(6, 20, 8), ref[0], what="y")


def test_replay_ssm_module_uses_kernels():
    import bayes_ssm
    from bayes_ssm import _capi
    mod = bayes_ssm.ReplaySSM(8, 8, chunk_length=16).cuda()
    inp = make_inputs(4, 40, 8, 8, seed=11)
    k, v, q, a = (inp[x].cuda().requires_grad_() for x in ("k", "v", "q", "a"))
    y, _, _ = mod(k, v, q, transition_diagonals=a)
    y.square().sum().backward()
    assert _capi._LIB is not None  # the C library served the call
    ref = oracle.forward(to_np64(k), to_np64(v), to_np64(q), to_np64(a), np.full((4, 40), 0.05),
                         np.full((4, 40), 0.2))
    assert_parity(y, ref[0], what="y")
    rg = oracle.backward(to_np64(k), to_np64(v), to_np64(q), to_np64(a), np.full((4, 40), 0.05),
                         np.full((4, 40), 0.2), None, None, 2 * ref[0])
    assert_parity(k.grad, rg["k"], what="grad k")
    assert_parity(a.grad, rg["a"], what="grad a")


def test_kernel_failure_is_loud():
    """An unsupported kernel call raises; nothing falls back silently."""
    from bayes_ssm.fused_cuda import fused_diagonal_bayesian
    k = torch.randn(2, 5, 3, device="cuda")
    with pytest.raises(ValueError, match="no kernel"):
        fused_diagonal_bayesian(k, torch.randn(2, 5, 8, device="cuda"), k, torch.ones(2, 5, 3, device="cuda"),
                                torch.zeros(2, 5, device="cuda"), torch.ones(2, 5, device="cuda"), None, None,
                                chunk_length=4, denominator_floor=1e-6)


# ----------------------------------------------------------------- assoc scan

def _scan_case(name):
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("name", ["assoc_config1", "assoc_random_init", "assoc_config2_slice"])
def test_assoc_scan_kernel_vs_reference_fixture(name):
    import bayes_ssm
    g = _scan_case(name)
    t = lambda x: torch.from_numpy(g[x]).float().cuda()
    with torch.no_grad():
        y, mt, pt = bayes_ssm.associative_static_bayesian_cuda(
            t("in_k"), t("in_v"), t("in_q"), observation_variances=t("in_r"),
            initial_mean=t("in_M0"), initial_covariance=t("in_P0"))
    assert_parity(y, g["out_y"], what="y")
    assert_parity(mt, g["out_MT"], what="M_T")
    assert_parity(pt, g["out_PT"], what="P_T")


def test_assoc_scan_config2_full_vs_oracle():
    """Config 2: B4 T64 H8 (32 chains), D = M = 16."""
    import bayes_ssm
    g = torch.Generator().manual_seed(2)
    n, t, d, m = 32, 64, 16, 16
    k = torch.randn(n, t, d, generator=g) / 4
    q = torch.randn(n, t, d, generator=g) / 4
    v = torch.randn(n, t, m, generator=g)
    r = torch.nn.functional.softplus(torch.randn(n, t, generator=g)) + 1e-2
    with torch.no_grad():
        y, mt, pt = bayes_ssm.associative_static_bayesian_cuda(k.cuda(), v.cuda(), q.cuda(),
                                                               observation_variances=r.cuda())
    ry, rmt, rpt = oracle.assoc_scan(to_np64(k), to_np64(v), to_np64(q), to_np64(r))
    assert_parity(y, ry, what="y")
    assert_parity(mt, rmt, what="M_T")
    assert_parity(pt, rpt, what="P_T")
    # and the scan equals the dense recurrence it replaces
    dy = oracle.forward(to_np64(k), to_np64(v), to_np64(q), None, None, to_np64(r))[0]
    assert_parity(y, dy, what="y vs dense")


def test_assoc_scan_rejects_small_variance_on_gpu():
    import bayes_ssm
    k = torch.randn(2, 8, 4, device="cuda")
    r = torch.full((2, 8), 0.5, device="cuda")
    r[1, 3] = 1e-9
    with pytest.raises(ValueError, match="denominator_floor"):
        bayes_ssm.associative_static_bayesian_cuda(k, torch.randn(2, 8, 3, device="cuda"), k,
                                                   observation_variances=r)


@pytest.mark.parametrize("bad", [float("nan"), float("inf"), float("-inf"), 0.0, -1.0, 9.9e-7, "scalar"])
def test_assoc_scan_variance_errors_match_eager(bad):
    """The kernel flags the observation variances the eager scan rejects
    (non-finite, or below the floor; any chain, any token, scalar broadcast)
    and accepts the floor itself and the largest finite float."""
    import bayes_ssm
    g = torch.Generator().manual_seed(5)
    k = (torch.randn(3, 21, 4, generator=g) / 2).cuda()
    v = torch.randn(3, 21, 5, generator=g).cuda()
    if bad == "scalar":
        r = 5e-7
    else:
        r = torch.full((3, 21), 0.5, device="cuda")
        r[2, 20] = bad
    for fn in (bayes_ssm.associative_static_bayesian, bayes_ssm.associative_static_bayesian_cuda):
        with torch.no_grad(), pytest.raises(ValueError, match="denominator_floor"):
            fn(k, v, k, observation_variances=r)
    # accepted boundary values (a variance at the floor makes the precision
    # ~1e5 and both FP32 scans ill-conditioned: acceptance only, no parity)
    ok = torch.full((3, 21), 0.5, device="cuda")
    ok[0, 0], ok[1, 7] = 1e-6, torch.finfo(torch.float32).max
    with torch.no_grad():
        y, _, _ = bayes_ssm.associative_static_bayesian_cuda(k, v, k, observation_variances=ok)
    assert torch.isfinite(y).all()


def test_assoc_scan_default_state_equals_explicit():
    """Omitting the initial state (identity covariance, zero mean; not built
    on the CUDA path) gives the same result as passing it explicitly, and
    T = 0 returns the defaults."""
    import bayes_ssm
    g = torch.Generator().manual_seed(6)
    k = (torch.randn(2, 3, 17, 8, generator=g) / 3).cuda()
    v = torch.randn(2, 3, 17, 6, generator=g).cuda()
    r = (torch.rand(2, 3, 17, generator=g) + 0.1).cuda()
    with torch.no_grad():
        a = bayes_ssm.associative_static_bayesian_cuda(k, v, k, observation_variances=r)
        b = bayes_ssm.associative_static_bayesian_cuda(
            k, v, k, observation_variances=r, initial_mean=torch.zeros(2, 3, 8, 6, device="cuda"),
            initial_covariance=torch.eye(8, device="cuda"))
        for x, y in zip(a, b):
            assert x.shape == y.shape
            assert float((x - y).norm()) <= 1e-5 * float(y.norm())
        y0, m0, p0 = bayes_ssm.associative_static_bayesian_cuda(k[..., :0, :], v[..., :0, :], k[..., :0, :])
    assert y0.shape == (2, 3, 0, 6)
    assert torch.equal(m0, torch.zeros(2, 3, 8, 6, device="cuda"))
    assert torch.equal(p0, torch.eye(8, device="cuda").expand(2, 3, 8, 8))


@pytest.mark.parametrize("dtype", (torch.float32, torch.bfloat16, torch.float16))
def test_check_values_flags_match_torch(dtype):
    """The one-pass input check (C ABI) agrees with torch's isfinite / sign
    tests, on aligned and unaligned views and ragged lengths."""
    from bayes_ssm import _capi
    base = (torch.rand(1003, device="cuda") + 0.5).to(dtype)

    def want(x):
        xf = x.float()
        return ((_capi.CHECK_NONFINITE if bool((~torch.isfinite(xf)).any()) else 0)
                | (_capi.CHECK_NOT_POSITIVE if bool((xf <= 0).any()) else 0)
                | (_capi.CHECK_NEGATIVE if bool((xf < 0).any()) else 0))

    for pos, val in ((None, None), (3, float("nan")), (1002, float("inf")), (500, 0.0), (7, -1.0),
                     (64, float("-inf")), (0, -0.0)):
        x = base.clone()
        if pos is not None:
            x[pos] = val
        views = (x, x[1:], x[:997], x[5:13], x[:0])
        got = _capi.check_values(list(views))
        assert got == [want(v) for v in views], (pos, val, got)


@pytest.mark.parametrize("dtype", (torch.float32, torch.bfloat16, torch.float16))
def test_check_values_flags_large_tensor(dtype):
    """Tensors far larger than one pass of the check kernel's grid, where each
    thread keeps four loads in flight: a bad value planted early, in the
    middle, near the end of the four-load loop, in its remainder and in the
    scalar tail is found (and nothing is flagged without one)."""
    from bayes_ssm import _capi
    n = 40_000_003  # not a multiple of a 16-byte vector either
    x = torch.ones(n, device="cuda", dtype=dtype)
    assert _capi.check_values([x]) == [0]
    for pos, val, flag in ((17, float("nan"), _capi.CHECK_NONFINITE), (n // 2, -2.0, _capi.CHECK_NEGATIVE),
                           (n - 1_000_000, 0.0, _capi.CHECK_NOT_POSITIVE), (n - 40_000, float("inf"), _capi.CHECK_NONFINITE),
                           (n - 1, -1.0, _capi.CHECK_NEGATIVE)):
        y = x.clone()
        y[pos] = val
        got = _capi.check_values([y])[0]
        assert got & flag, (pos, val, got)


@pytest.mark.parametrize("dtype", (torch.float32, torch.bfloat16, torch.float16))
def test_api_validation_errors_on_gpu(dtype):
    """CUDA inputs raise the reference's validation errors, first failing
    check first (keys before values, finiteness before sign)."""
    import bayes_ssm
    inp = make_inputs(4, 12, 4, 8, seed=9)
    base = {k: (None if v is None else v.cuda()) for k, v in inp.items()}
    for key in ("k", "v", "q"):
        base[key] = base[key].to(dtype)

    def call(**over):
        x = {**base, **over}
        return bayes_ssm.bayesian_layer(x["k"], x["v"], x["q"], transition_diagonals=x["a"],
                                        process_variances=x["p"], observation_variances=x["r"],
                                        chunk_length=4, optimized=True)

    def poked(name, value, idx=(1, 2)):
        t = base[name].clone()
        t[idx] = value
        return t

    call()
    with pytest.raises(ValueError, match="^keys must contain only finite values$"):
        call(k=poked("k", float("nan")), v=poked("v", float("inf")))
    with pytest.raises(ValueError, match="^values must contain only finite values$"):
        call(v=poked("v", float("inf")))
    with pytest.raises(ValueError, match="^queries must contain only finite values$"):
        call(q=poked("q", float("-inf")))
    with pytest.raises(ValueError, match="^transition_diagonals must contain only finite values$"):
        call(a=poked("a", float("nan")))
    with pytest.raises(ValueError, match="^process_variances must be nonnegative$"):
        call(p=poked("p", -1e-3))
    with pytest.raises(ValueError, match="^process_variances must contain only finite values$"):
        call(p=poked("p", float("nan")))
    with pytest.raises(ValueError, match="^observation_variances must be strictly positive$"):
        call(r=poked("r", 0.0))
    # a value check that precedes a host-side check wins, as in the reference
    with pytest.raises(ValueError, match="^keys must contain only finite values$"):
        call(k=poked("k", float("nan")), r=base["r"][:, :5])
    with pytest.raises(ValueError, match="^observation_variances must be scalar or have shape"):
        call(r=base["r"][:, :5])
