"""GPU: a bounded in-kernel wait that gives up is reported, never silent.

The probe kernel waits with a short poll limit on a barrier phase that
nothing completes -- the way a recurrence kernel's wait would run out -- so
nothing faults or hangs.  The status check must then raise once, and a
following check must pass (each give-up is reported once).
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_give_up_raises_once():
    from bayes_ssm import _capi
    sp = torch.cuda.current_stream().cuda_stream
    before = _capi.wait_timeouts()
    _capi.wait_probe(256, sp)
    with pytest.raises(_capi.WaitTimeout, match="1 bounded wait"):
        _capi.stream_status(sp)
    assert _capi.wait_timeouts() == before + 1
    _capi.stream_status(sp)  # already reported: no error now


def test_api_raises_after_a_give_up():
    """A give-up pending on the device makes the next public call raise rather
    than return outputs."""
    import bayes_ssm
    from bayes_ssm import _capi
    sp = torch.cuda.current_stream().cuda_stream
    k = torch.nn.functional.normalize(torch.randn(4, 16, 8, device="cuda"), dim=-1)
    v = torch.randn(4, 16, 8, device="cuda")
    _capi.wait_probe(256, sp)
    with pytest.raises(_capi.WaitTimeout):
        bayes_ssm.bayesian_layer(k, v, k, transition_diagonals=torch.full_like(k, 0.9),
                                 process_variances=0.01, observation_variances=1.0, chunk_length=8,
                                 optimized=True)
    y, _, _ = bayes_ssm.bayesian_layer(k, v, k, transition_diagonals=torch.full_like(k, 0.9),
                                       process_variances=0.01, observation_variances=1.0, chunk_length=8,
                                       optimized=True)
    assert torch.isfinite(y).all()
