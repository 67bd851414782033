"""The allocation-free backward entry point (bssm_backward_chunked_noalloc).

Callers that cannot allocate device memory when they call the backward (a
host whose allocator owns the device budget, a serving loop that cannot take
an allocation's device-wide synchronisation, an FFI host with no device
allocator) use this entry point: its phase-A scratch is a static device array
inside the library instead of a caller workspace.  Checked here: it matches
the workspace-taking entry point on two calls in a row (the shared array keeps
the previous call's contents, which must not matter), and a problem larger
than the array is refused.  The file is named to be collected last.
"""
from __future__ import annotations

import pytest
import torch

from harness import assert_parity, capi_backward, capi_forward, io_code, make_inputs

pytestmark = pytest.mark.gpu


def _noalloc(inp, fwd, gy, *, chunks, n, t, d=8, m=8, fixed=False):
    from bayes_ssm import _capi
    dev = torch.device("cuda")
    k, v, q = (inp[x].cuda().contiguous() for x in ("k", "v", "q"))
    a, p, r = (inp[x].cuda().contiguous() for x in ("a", "p", "r"))
    gk, gv, gq = torch.empty_like(k), torch.empty_like(v), torch.empty_like(q)
    gd = torch.empty(n, t, d, device=dev)
    gp = torch.empty(n, t, device=dev)
    gr = torch.empty(n, t, device=dev)
    gm0 = torch.empty(n, d, m, device=dev)
    gc0 = torch.empty(n, d, d, device=dev)
    _capi.backward_chunked_noalloc(d, m, io_code(k.dtype), fixed, True, True, k, v, q, a, p, r, None,
                                   None, fwd["bm"], fwd["bc"], gy.cuda(), None, None, gk, gv, gq, gd,
                                   gp, gr, gm0, gc0, n, t, chunks, 1e-6,
                                   torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return dict(k=gk, v=gv, q=gq, a=gd, p=gp, r=gr, M0=gm0, P0=gc0)


def test_noalloc_backward_matches_workspace_backward_twice():
    from bayes_ssm import _capi
    n, t, chunks = 96, 130, 64  # 15 phase-A states per chunk: scratch is used
    assert _capi.workspace_bytes(8, 8, n, t, chunks) > 0
    gy = torch.randn(n, t, 8, generator=torch.Generator().manual_seed(5))
    for seed in (1, 2):  # two calls in a row, different inputs
        inp = make_inputs(n, t, 8, 8, seed=seed, io_dtype=torch.bfloat16)
        fwd = capi_forward(inp, chunks=chunks, replay_states=False)
        want = capi_backward(inp, fwd, gy, None, None, chunks=chunks)
        got = _noalloc(inp, fwd, gy, chunks=chunks, n=n, t=t)
        for key in want:
            assert_parity(got[key], want[key].float().cpu().numpy(), what=f"noalloc grad {key}")


@pytest.mark.parametrize("d,m,n", [(1, 8, 24), (2, 8, 24), (4, 8, 24), (8, 8, 24), (64, 64, 3)])
@pytest.mark.parametrize("dtype", (torch.float32, torch.bfloat16))
@pytest.mark.parametrize("fixed", (False, True))
def test_noalloc_every_shape_family_and_dynamics(d, m, n, dtype, fixed):
    """Every key dimension (each with its own scratch layout), FP32 and BF16
    projections and fixed dynamics, two calls in a row; chunk 64 so the
    scratch is used."""
    from bayes_ssm import _capi
    if d == 64 and dtype == torch.bfloat16:
        pytest.skip("(64, 64) takes float32 projections only")
    t, chunks = 70, 64
    assert _capi.workspace_bytes(d, m, n, t, chunks) > 0
    gy = torch.randn(n, t, m, generator=torch.Generator().manual_seed(7))
    for seed in (3, 4):
        inp = make_inputs(n, t, d, m, seed=seed, io_dtype=dtype)
        fwd = capi_forward(inp, chunks=chunks, fixed=fixed, replay_states=False)
        want = capi_backward(inp, fwd, gy, None, None, chunks=chunks, fixed=fixed)
        got = _noalloc(inp, fwd, gy, chunks=chunks, n=n, t=t, d=d, m=m, fixed=fixed)
        for key in want:
            assert_parity(got[key], want[key].float().cpu().numpy(), what=f"noalloc d{d} grad {key}")


def test_noalloc_backward_rejects_problems_larger_than_the_scratch():
    from bayes_ssm import _capi
    cap = _capi.load().bssm_backward_noalloc_max_scratch_bytes()
    n = cap // (15 * 128 * 4) + 1  # one chain more than fits at chunk 64
    assert _capi.workspace_bytes(8, 8, n, 512, 64) > cap
    fake = 1 << 20  # never dereferenced: the size check comes first
    with pytest.raises(_capi.KernelError, match="static scratch"):
        _capi.load()
        rc = _capi.load().bssm_backward_chunked_noalloc(
            8, 8, 0, 0, 0, 0, *([fake] * 21), n, 512, 64, 1e-6, None)
        _capi.check(rc, "bssm_backward_chunked_noalloc")
