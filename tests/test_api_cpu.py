"""Host-side API behaviour on CPU tensors (no GPU): the public ``bayes_ssm``
functions keep the reference's signatures, validation errors and dense
semantics.  The CPU dense recurrence is compared with the reference's FP64
golden vectors (the same fixtures that pin the oracle)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bayes_ssm
from bayes_ssm import bayesian_layer
from conftest import GOLDEN


def _load(name):
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("name", ["diag_d4m3_all", "paper_d8m8_all", "paper_d2m8_all", "paper_d8m8_floor"])
def test_cpu_dense_path_matches_reference_fixture(name):
    g = _load(name)
    ins = {k: torch.from_numpy(g[f"in_{k}"]).requires_grad_() for k in ("k", "v", "q", "a", "p", "r", "M0", "P0")}
    y, mt, pt = bayesian_layer(ins["k"], ins["v"], ins["q"], transition_diagonals=ins["a"],
                               process_variances=ins["p"], observation_variances=ins["r"],
                               initial_mean=ins["M0"], initial_covariance=ins["P0"],
                               chunk_length=int(g["chunk"]), denominator_floor=float(g["floor"]))
    for got, key in ((y, "out_y"), (mt, "out_MT"), (pt, "out_PT")):
        np.testing.assert_allclose(got.detach().numpy(), g[key], rtol=1e-10, atol=1e-11)
    loss = (y * torch.from_numpy(g["g_y"])).sum() + (mt * torch.from_numpy(g["g_MT"])).sum() + \
        (pt * torch.from_numpy(g["g_PT"])).sum()
    grads = torch.autograd.grad(loss, list(ins.values()))
    for key, gr in zip(ins, grads):
        np.testing.assert_allclose(gr.numpy(), g[f"grad_{key}"], rtol=1e-9, atol=1e-10, err_msg=key)


def test_public_surface_matches_reference():
    assert set(bayes_ssm.__all__) == {
        "BayesianLayer", "bayesian_layer", "make_diagonal_dynamics", "make_rotation_dynamics",
        "make_rotation_process_covariances", "ReplaySSM", "associative_static_bayesian",
        "associative_static_bayesian_cuda"}


@pytest.mark.parametrize("kwargs,exc,msg", [
    (dict(observation_variances=0.0), ValueError, "strictly positive"),
    (dict(process_variances=-1.0), ValueError, "nonnegative"),
    (dict(denominator_floor=0.0), ValueError, "positive"),
    (dict(chunk_length=0), ValueError, "chunk_length"),
    (dict(transitions=torch.eye(4).expand(5, 4, 4), transition_diagonals=torch.ones(5, 4)), ValueError, "not both"),
    (dict(rotation_radii=torch.ones(5, 2)), ValueError, "together"),
    (dict(initial_covariance=torch.tensor([[1.0, 2.0, 0, 0], [0, 1.0, 0, 0], [0, 0, 1.0, 0], [0, 0, 0, 1.0]])),
     ValueError, "symmetric"),
    (dict(initial_covariance=-torch.eye(4)), ValueError, "positive semidefinite"),
    (dict(replay_ssm=1), TypeError, "replay_ssm"),
])
def test_validation_errors(kwargs, exc, msg):
    k = torch.randn(5, 4)
    with pytest.raises(exc, match=msg):
        bayesian_layer(k, torch.randn(5, 3), k, **kwargs)


def test_non_finite_inputs_rejected():
    k = torch.randn(5, 4)
    k[2, 1] = float("nan")
    with pytest.raises(ValueError, match="finite"):
        bayesian_layer(k, torch.randn(5, 3), torch.randn(5, 4))


def test_empty_sequence_returns_initial_state():
    k = torch.randn(3, 0, 4)
    y, m, p = bayesian_layer(k, torch.randn(3, 0, 2), k)
    assert y.shape == (3, 0, 2)
    assert torch.equal(m, torch.zeros(3, 4, 2))
    assert torch.equal(p, torch.eye(4).expand(3, 4, 4))


def test_low_precision_inputs_promote_to_fp32():
    k = torch.randn(2, 6, 4).to(torch.bfloat16)
    y, m, p = bayesian_layer(k, torch.randn(2, 6, 3).to(torch.bfloat16), k)
    assert y.dtype == m.dtype == p.dtype == torch.float32


def test_identity_and_diagonal_ones_agree():
    g = torch.Generator().manual_seed(3)
    k, q = torch.randn(2, 9, 4, generator=g), torch.randn(2, 9, 4, generator=g)
    v = torch.randn(2, 9, 3, generator=g)
    a = bayesian_layer(k, v, q, process_variances=0.1, chunk_length=4)
    b = bayesian_layer(k, v, q, transition_diagonals=torch.ones(2, 9, 4), process_variances=0.1, chunk_length=2)
    for x, y in zip(a, b):
        torch.testing.assert_close(x, y, rtol=1e-6, atol=1e-6)


def test_rotation_dynamics_dense_path_runs():
    g = torch.Generator().manual_seed(4)
    k, q = torch.randn(1, 5, 4, generator=g), torch.randn(1, 5, 4, generator=g)
    v = torch.randn(1, 5, 2, generator=g)
    radius = torch.rand(1, 5, 2, generator=g) * 0.2 + 0.7
    angle = torch.randn(1, 5, 2, generator=g) * 0.2
    y, _, _ = bayesian_layer(k, v, q, rotation_radii=radius, rotation_angles=angle, process_variances=0.1)
    y2, _, _ = bayesian_layer(k, v, q, transitions=bayes_ssm.make_rotation_dynamics(radius.log(), angle),
                              process_covariances=bayes_ssm.make_rotation_process_covariances(
                                  torch.full((1, 5, 2), 0.1)))
    torch.testing.assert_close(y, y2)


def test_bayesian_layer_module_and_replay_module_cpu():
    layer = bayes_ssm.BayesianLayer(4, 3, learn_noise=True)
    k = torch.randn(2, 7, 4)
    y, m, p = layer(k, torch.randn(2, 7, 3), k)
    y.sum().backward()
    assert layer._process_raw.grad is not None
    rep = bayes_ssm.ReplaySSM(4, 3, process_variance=0.0)
    k2 = torch.randn(2, 7, 4, dtype=torch.float64)
    v2 = torch.randn(2, 7, 3, dtype=torch.float64)
    ya, ma, pa = rep(k2, v2, k2)
    yb, mb, pb = rep.associative_scan(k2, v2, k2)
    torch.testing.assert_close(ya, yb, rtol=1e-8, atol=1e-9)
    with pytest.raises(ValueError, match="process_variance=0"):
        bayes_ssm.ReplaySSM(4, 3).associative_scan(k2, v2, k2)


def test_assoc_scan_cpu_matches_reference_fixture():
    g = _load("assoc_random_init")
    t = lambda x: torch.from_numpy(g[x])
    y, mt, pt = bayes_ssm.associative_static_bayesian(t("in_k"), t("in_v"), t("in_q"),
                                                      observation_variances=t("in_r"),
                                                      initial_mean=t("in_M0"),
                                                      initial_covariance=t("in_P0"))
    np.testing.assert_allclose(y.numpy(), g["out_y"], rtol=1e-9, atol=1e-10)
    np.testing.assert_allclose(pt.numpy(), g["out_PT"], rtol=1e-9, atol=1e-10)


def test_assoc_scan_rejects_variance_below_floor():
    k = torch.randn(1, 4, 2)
    with pytest.raises(ValueError, match="denominator_floor"):
        bayes_ssm.associative_static_bayesian(k, torch.randn(1, 4, 2), k,
                                              observation_variances=torch.tensor([1.0, 1e-9, 1.0, 1.0]))


def test_assoc_scan_cuda_requires_cuda_tensors():
    k = torch.randn(1, 4, 2)
    with pytest.raises(ValueError, match="CUDA"):
        bayes_ssm.associative_static_bayesian_cuda(k, torch.randn(1, 4, 2), k)


def test_queued_checks_merge_precomputed_words_in_order(monkeypatch):
    """The queued value checks take a producing kernel's precomputed words for
    some tensors and the check kernel's flags for the rest, and raise the
    first failure in the reference's order (host logic; the flag sources are
    faked on CPU)."""
    import sys

    bl = sys.modules["bayes_ssm.bayesian_layer"]
    calls = []

    def fake_device_flags(tensors):
        calls.append(len(tensors))
        return [int(x.flatten()[0].item()) for x in tensors]  # each fake tensor carries its flags

    monkeypatch.setattr(bl, "_device_flags", fake_device_flags)
    words = torch.tensor([0, 0, 1, 0, 0, 0], dtype=torch.int32)  # queries not finite

    def run(entries):
        chk = bl._DeviceChecks()
        chk.items = list(entries)
        chk.flush()

    keys, values = torch.zeros(2), torch.zeros(2)
    # every item precomputed: no check-kernel call, queries' word raises
    with pytest.raises(ValueError, match="queries must contain only finite values"):
        run([(keys, "keys", 0, (words, 0)), (values, "values", 0, (words, 1)), (keys, "queries", 0, (words, 2))])
    assert calls == []
    # mixed: a plain tensor earlier in the order fails first
    bad_obs = torch.tensor([float(bayes_ssm._capi.CHECK_NOT_POSITIVE)])
    with pytest.raises(ValueError, match="observation_variances must be strictly positive"):
        run([(keys, "keys", 0, (words, 0)), (bad_obs, "observation_variances", 2, None),
             (keys, "queries", 0, (words, 2))])
    assert calls == [1]
    # a negative-variance word on a kind-1 check
    words2 = torch.tensor([0, 0, 0, 0, bayes_ssm._capi.CHECK_NEGATIVE, 0], dtype=torch.int32)
    with pytest.raises(ValueError, match="process_variances must be nonnegative"):
        run([(keys, "process_variances", 1, (words2, 4)), (torch.zeros(1), "observation_variances", 2, None)])
    # all clear
    run([(keys, "keys", 0, (torch.zeros(6, dtype=torch.int32), 0)), (torch.zeros(1), "values", 0, None)])


def test_prechecked_registry_ignores_cpu_tensors():
    import sys

    bl = sys.modules["bayes_ssm.bayesian_layer"]
    x = torch.zeros(4)
    bl._register_prechecked((x,), torch.zeros(1, dtype=torch.int32))
    assert bl._prechecked_word(x) is None  # words only stand for CUDA outputs
