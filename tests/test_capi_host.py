"""CPU-side checks of the C ABI: the library loads and exports every symbol
the header declares; argument validation fails loudly without a GPU."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "bayes_ssm_b200.h"


def _declared_symbols() -> set[str]:
    text = HEADER.read_text()
    names = set(re.findall(r"\b(bssm_[a-z0-9_]+)\s*\(", text))
    # expand the per-dimension macro declarations
    macro = re.search(r"#define BSSM_DECLARE_DIM\(DN\)(.*?)\n\n", text, re.S).group(1)
    templ = set(re.findall(r"bssm_d##DN##_([a-z_]+)\s*\(", macro))
    for dn in re.findall(r"BSSM_DECLARE_DIM\((\d+)\)", text):
        names |= {f"bssm_d{dn}_{t}" for t in templ}
    names.discard("bssm_d")
    return {n for n in names if not n.startswith("bssm_d##")}


@pytest.fixture(scope="module")
def lib():
    from bayes_ssm import _build, _capi
    _build.build()
    return _capi.load()


def test_library_exports_every_declared_symbol(lib):
    declared = _declared_symbols()
    assert len(declared) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", str(Path(lib._name))], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (bssm_\w+)", out))
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_version_and_last_error(lib):
    assert lib.bssm_version() >= 10000
    assert isinstance(lib.bssm_last_error(), bytes)


def test_unsupported_shape_rejected_without_gpu(lib):
    from bayes_ssm import _capi
    fwd_nulls = [None] * 13 + [None, 0]
    rc = lib.bssm_forward_chunked_ex(3, 8, 0, 0, *fwd_nulls, 1, 1, 1, 1e-6, None)
    assert rc == 2
    assert b"no kernel" in lib.bssm_last_error()
    rc = lib.bssm_forward_chunked_ex(8, 8, 0, 0, *fwd_nulls, 1, 1, 0, 1e-6, None)
    assert rc == 1 and b"chunks" in lib.bssm_last_error()
    rc = lib.bssm_forward_chunked_ex(8, 8, 0, 0, *fwd_nulls, 1, 1, 4, -1.0, None)
    assert rc == 1 and b"floor" in lib.bssm_last_error()
    rc = lib.bssm_forward_chunked_ex(8, 8, 7, 0, *fwd_nulls, 1, 1, 4, 1e-6, None)
    assert rc == 2
    with pytest.raises(_capi.KernelError):
        _capi.check(rc, "probe")


def test_null_pointers_rejected_without_gpu(lib):
    rc = lib.bssm_forward_chunked_ex(8, 8, 0, 0, *([None] * 13), None, 0, 4, 10, 4, 1e-6, None)
    assert rc == 1 and b"null" in lib.bssm_last_error()
    bwd_nulls = [None] * 10 + [None, 0] + [None] * 11
    rc = lib.bssm_backward_chunked_ex(8, 8, 0, 0, 1, 1, *bwd_nulls, None, 0, 4, 10, 4, 1e-6, None)
    assert rc == 1


def _gains_floats(n, t, d):
    """Per-token gains after the states: u [N,T,D], then the signed gain
    scales [N,T], each part padded to 4 floats."""
    r4 = lambda x: (x + 3) // 4 * 4
    return r4(n * t * d) + r4(n * t)


def _group_chains(n):
    """States are stored per group of 32 chains (structure of arrays)."""
    return (n + 31) // 32 * 32


def test_replay_states_size_formula(lib):
    # chunks <= 4: no state between boundary checkpoints, only the gains
    assert lib.bssm_replay_states_bytes(8, 8, 100, 512, 4) == _gains_floats(100, 512, 8) * 4
    # D8M8, chunk 64: 15 states per chunk, 8 chunks; 64 mean + 36 packed
    # covariance floats each
    assert lib.bssm_replay_states_bytes(8, 8, 64, 512, 64) == (64 * 8 * 15 * (64 + 36) + _gains_floats(64, 512, 8)) * 4
    # a partial group of chains is padded to 32
    assert lib.bssm_replay_states_bytes(8, 8, 10, 512, 64) == (32 * 8 * 15 * 100 + _gains_floats(10, 512, 8)) * 4
    # D4M8: 32 + 10 floats, padded to 44
    assert lib.bssm_replay_states_bytes(4, 8, 2, 64, 64) == (_group_chains(2) * 1 * 15 * 44 + _gains_floats(2, 64, 4)) * 4
    # partial last chunk: slots are sized by the full chunk length; D2: 16 + 3 -> 20
    assert lib.bssm_replay_states_bytes(2, 8, 3, 70, 32) == (_group_chains(3) * 3 * 7 * 20 + _gains_floats(3, 70, 2)) * 4
    # D1: 8 + 1 floats per state, padded to 12
    assert lib.bssm_replay_states_bytes(1, 8, 5, 64, 64) == (_group_chains(5) * 1 * 15 * 12 + _gains_floats(5, 64, 1)) * 4


def test_workspace_size_formula(lib):
    # chunks <= sub-chunk length: no phase-A workspace
    assert lib.bssm_backward_workspace_bytes(8, 8, 100, 512, 4) == 0
    # D8: 16 floats per lane, 8 lanes, (64/4 - 1) saved states per chain
    assert lib.bssm_backward_workspace_bytes(8, 8, 10, 512, 64) == 10 * 15 * 8 * 16 * 4
    assert lib.bssm_backward_workspace_bytes(3, 8, 10, 512, 64) == 0


def test_assoc_scan_limits_without_gpu(lib):
    rc = lib.bssm_assoc_scan_ex(33, 8, *([None] * 10), 1, 1, 1e-6, None)
    assert rc == 2 and b"key_dim" in lib.bssm_last_error()


def test_misaligned_pointer_rejected_before_launch(lib):
    """A 4-byte-offset pointer is refused on the host; no kernel is launched
    (fake addresses are never dereferenced)."""
    good = 0x10000
    ptrs = [good + 0x1000 * i for i in range(13)]
    ptrs[0] += 4  # keys: misaligned
    rc = lib.bssm_forward_chunked_ex(8, 8, 0, 0, *ptrs, None, 0, 2, 16, 8, 1e-6, None)
    assert rc == 3 and b"16-byte" in lib.bssm_last_error()


def test_d64_and_rotation_host_checks_without_gpu(lib):
    from bayes_ssm import _capi
    _capi.load()
    # (64, 64): float32 only; no replay states; the workspace holds 64 KB per
    # saved 2-token sub-chunk state and chain
    fwd_nulls = [None] * 13 + [None, 0]
    rc = lib.bssm_forward_chunked_ex(64, 64, 1, 0, *fwd_nulls, 1, 1, 1, 1e-6, None)
    assert rc == 2 and b"float32" in lib.bssm_last_error()
    assert lib.bssm_replay_states_bytes(64, 64, 4, 512, 64) == 0
    assert lib.bssm_backward_workspace_bytes(64, 64, 3, 512, 64) == 3 * 31 * 2 * 16 * 256 * 4
    # rotation: (2|4|8, 8) only, workspace (D + M) floats per lane and saved state
    assert lib.bssm_rotation_workspace_bytes(8, 8, 10, 512, 64) == 10 * 15 * 8 * 16 * 4
    assert lib.bssm_rotation_workspace_bytes(1, 8, 10, 512, 64) == 0
    rc = lib.bssm_rotation_forward_chunked(1, 8, *([None] * 14), 1, 1, 1, 1e-6, None)
    assert rc == 2 and b"rotation" in lib.bssm_last_error()
    rc = lib.bssm_rotation_forward_chunked(8, 8, *([None] * 14), 1, 4, 4, 1e-6, None)
    assert rc == 1 and b"null" in lib.bssm_last_error()
    rc = lib.bssm_rotation_backward_chunked(8, 8, 0, *([None] * 22), 0, 1, 4, 0, 1e-6, None)
    assert rc == 1 and b"chunks" in lib.bssm_last_error()
