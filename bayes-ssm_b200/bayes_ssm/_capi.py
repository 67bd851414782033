"""ctypes binding of ``libbayes_ssm_b200.so`` (the C ABI in include/bayes_ssm_b200.h).

The library is built in-tree (``bayes_ssm/_build.py``) and loaded once.  A
missing or unloadable library raises :class:`ExtensionUnavailable`; there is
no fallback path for CUDA tensors.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

PKG_ROOT = Path(__file__).resolve().parents[1]
LIB_PATH = Path(os.environ.get("BAYES_SSM_B200_LIB", PKG_ROOT / "lib" / "libbayes_ssm_b200.so"))

BSSM_OK = 0
BSSM_F32 = 0
BSSM_BF16 = 1
BSSM_F16 = 2
CHECK_NONFINITE, CHECK_NOT_POSITIVE, CHECK_NEGATIVE = 1, 2, 4
SUPPORTED = ((1, 8), (2, 8), (4, 8), (8, 8), (64, 64))

_LIB: Optional[ctypes.CDLL] = None
_LOAD_ERROR: Optional[BaseException] = None


class ExtensionUnavailable(RuntimeError):
    """The CUDA library could not be loaded."""


class KernelError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


_vp, _l, _i, _d, _sz = ctypes.c_void_p, ctypes.c_long, ctypes.c_int, ctypes.c_double, ctypes.c_size_t

_SIGNATURES = {
    "bssm_last_error": ([], ctypes.c_char_p),
    "bssm_version": ([], _i),
    "bssm_forward_chunked_ex": ([_i, _i, _i, _i] + [_vp] * 13 + [_vp, _sz, _l, _l, _i, _d, _vp], _i),
    "bssm_replay_states_bytes": ([_i, _i, _l, _l, _i], _sz),
    "bssm_backward_workspace_bytes": ([_i, _i, _l, _l, _i], _sz),
    "bssm_backward_chunked_ex": ([_i, _i, _i, _i, _i, _i] + [_vp] * 10 + [_vp, _sz] + [_vp] * 11
                                 + [_vp, _sz, _l, _l, _i, _d, _vp], _i),
    "bssm_assoc_scan_ex": ([_i, _i] + [_vp] * 10 + [_l, _l, _d, _vp], _i),
    "bssm_backward_noalloc_max_scratch_bytes": ([], _sz),
    "bssm_backward_chunked_noalloc": ([_i, _i, _i, _i, _i, _i] + [_vp] * 21 + [_l, _l, _i, _d, _vp], _i),
    "bssm_check_values": ([_vp, _l, _i, _vp, _vp], _i),
    "bssm_envelope_partial_floats": ([_l, _l, _i, _i, _i], _l),
    "bssm_envelope_prologue": ([_vp, _i, _l, _l, _i, _i, _i, _l] + [_vp] * 5 + [_i] + [_vp] * 5, _i),
    "bssm_envelope_prologue_backward": ([_vp, _i, _l, _l, _i, _i, _i, _l] + [_vp] * 5 + [_i] + [_vp] * 4
                                        + [_l, _vp, _vp, _vp, _l, _vp], _i),
    "bssm_envelope_epilogue_partial_floats": ([_l, _l, _i, _i], _l),
    "bssm_rms_norm": ([_vp, _i, _l, _i, _vp, ctypes.c_float, _vp, _vp], _i),
    "bssm_rms_norm_partial_floats": ([_l, _i], _l),
    "bssm_rms_norm_backward": ([_vp, _i, _l, _i, _vp, ctypes.c_float, _vp, _vp, _vp, _vp, _l, _vp], _i),
    "bssm_envelope_epilogue": ([_vp, _i, _vp, _i, _l, _vp, ctypes.c_float, _l, _l, _i, _i, _vp, _vp], _i),
    "bssm_envelope_epilogue_backward": ([_vp, _i, _vp, _i, _l, _vp, ctypes.c_float, _l, _l, _i, _i, _vp, _vp, _vp,
                                         _l, _vp, _vp, _l, _vp], _i),
    "bssm_rotation_workspace_bytes": ([_i, _i, _l, _l, _i], _sz),
    "bssm_rotation_forward_chunked": ([_i, _i] + [_vp] * 14 + [_l, _l, _i, _d, _vp], _i),
    "bssm_rotation_backward_chunked": ([_i, _i, _i] + [_vp] * 22 + [_sz, _l, _l, _i, _d, _vp], _i),
    "bssm_rotation_coefficients": ([_vp, _vp, _l, _vp, _vp, _vp], _i),
    "bssm_rotation_coefficients_backward": ([_vp, _vp, _vp, _vp, _l, _vp, _vp, _vp], _i),
    "bssm_debug_wait_timeouts": ([], ctypes.c_uint),
    "bssm_stream_status": ([_vp], _i),
    "bssm_debug_wait_probe": ([_i, _vp], _i),
    "bssm_debug_fma_probe": ([_vp, _i, _i, _vp], _i),
    "bssm_debug_fma_probe_flops": ([_i, _i], _l),
    "bssm_debug_last_family": ([], _i),
}


def load() -> ctypes.CDLL:
    """Load the library (once) and declare the prototypes used here."""
    global _LIB, _LOAD_ERROR
    if _LIB is not None:
        return _LIB
    if _LOAD_ERROR is not None:
        raise ExtensionUnavailable(str(_LOAD_ERROR)) from _LOAD_ERROR
    try:
        if not LIB_PATH.exists():
            raise FileNotFoundError(
                f"{LIB_PATH} is missing; build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "or `python bayes-ssm_b200/bayes_ssm/_build.py`")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
    except BaseException as exc:  # remember the failure; every later call raises it
        _LOAD_ERROR = exc
        raise ExtensionUnavailable(f"cannot load {LIB_PATH}: {exc}") from exc
    _LIB = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != BSSM_OK:
        msg = load().bssm_last_error().decode(errors="replace")
        raise KernelError(f"{what} failed (status {rc}): {msg}")


def ptr(t) -> Optional[int]:
    """Device pointer of a tensor (None passes NULL)."""
    return None if t is None else t.data_ptr()


def forward_chunked(key_dim, value_dim, io_dtype, fixed, keys, values, queries, decay, process,
                    observation, mean0, cov0, out, mean_final, cov_final, bmean, bcov, n, t,
                    chunks, floor, stream, replay_states=None) -> None:
    lib = load()
    rs_bytes = 0 if replay_states is None else replay_states.numel() * replay_states.element_size()
    rc = lib.bssm_forward_chunked_ex(
        key_dim, value_dim, io_dtype, int(fixed), ptr(keys), ptr(values), ptr(queries), ptr(decay),
        ptr(process), ptr(observation), ptr(mean0), ptr(cov0), ptr(out), ptr(mean_final),
        ptr(cov_final), ptr(bmean), ptr(bcov), ptr(replay_states), rs_bytes, n, t, chunks,
        float(floor), stream)
    check(rc, "bssm_forward_chunked_ex")


def replay_states_bytes(key_dim, value_dim, n, t, chunks) -> int:
    return int(load().bssm_replay_states_bytes(key_dim, value_dim, n, t, chunks))


def workspace_bytes(key_dim, value_dim, n, t, chunks) -> int:
    return int(load().bssm_backward_workspace_bytes(key_dim, value_dim, n, t, chunks))


def backward_chunked(key_dim, value_dim, io_dtype, fixed, need_dynamics, need_initial, keys, values,
                     queries, decay, process, observation, mean0, cov0, bmean, bcov, gy, gmf, gcf,
                     gk, gv, gq, gd, gp, gr, gm0, gc0, workspace, workspace_nbytes, n, t, chunks,
                     floor, stream, replay_states=None) -> None:
    lib = load()
    rs_bytes = 0 if replay_states is None else replay_states.numel() * replay_states.element_size()
    rc = lib.bssm_backward_chunked_ex(
        key_dim, value_dim, io_dtype, int(fixed), int(need_dynamics), int(need_initial), ptr(keys),
        ptr(values), ptr(queries), ptr(decay), ptr(process), ptr(observation), ptr(mean0), ptr(cov0),
        ptr(bmean), ptr(bcov), ptr(replay_states), rs_bytes, ptr(gy), ptr(gmf), ptr(gcf), ptr(gk),
        ptr(gv), ptr(gq), ptr(gd), ptr(gp), ptr(gr), ptr(gm0), ptr(gc0), ptr(workspace),
        workspace_nbytes, n, t, chunks, float(floor), stream)
    check(rc, "bssm_backward_chunked_ex")


def assoc_scan(key_dim, value_dim, keys, values, queries, observation, mean0, cov0, out, mean_final,
               cov_final, status, n, t, floor, stream) -> None:
    lib = load()
    rc = lib.bssm_assoc_scan_ex(key_dim, value_dim, ptr(keys), ptr(values), ptr(queries),
                                ptr(observation), ptr(mean0), ptr(cov0), ptr(out), ptr(mean_final),
                                ptr(cov_final), ptr(status), n, t, float(floor), stream)
    check(rc, "bssm_assoc_scan_ex")


def rotation_workspace_bytes(key_dim, value_dim, n, t, chunks) -> int:
    return int(load().bssm_rotation_workspace_bytes(key_dim, value_dim, n, t, chunks))


def rotation_forward(key_dim, value_dim, keys, values, queries, cosines, sines, process, observation, mean0, cov0,
                     out, mean_final, cov_final, bmean, bcov, n, t, chunks, floor, stream) -> None:
    rc = load().bssm_rotation_forward_chunked(
        key_dim, value_dim, ptr(keys), ptr(values), ptr(queries), ptr(cosines), ptr(sines), ptr(process),
        ptr(observation), ptr(mean0), ptr(cov0), ptr(out), ptr(mean_final), ptr(cov_final), ptr(bmean), ptr(bcov),
        n, t, chunks, float(floor), stream)
    check(rc, "bssm_rotation_forward_chunked")


def rotation_backward(key_dim, value_dim, need_initial, keys, values, queries, cosines, sines, process,
                      observation, bmean, bcov, gy, gmf, gcf, gk, gv, gq, gcos, gsin, gproc, gobs, gm0, gc0,
                      workspace, workspace_nbytes, n, t, chunks, floor, stream) -> None:
    rc = load().bssm_rotation_backward_chunked(
        key_dim, value_dim, int(need_initial), ptr(keys), ptr(values), ptr(queries), ptr(cosines), ptr(sines),
        ptr(process), ptr(observation), ptr(bmean), ptr(bcov), ptr(gy), ptr(gmf), ptr(gcf), ptr(gk), ptr(gv),
        ptr(gq), ptr(gcos), ptr(gsin), ptr(gproc), ptr(gobs), ptr(gm0), ptr(gc0), ptr(workspace), workspace_nbytes,
        n, t, chunks, float(floor), stream)
    check(rc, "bssm_rotation_backward_chunked")


def rotation_coefficients(radii, angles, cosines, sines, stream) -> None:
    rc = load().bssm_rotation_coefficients(ptr(radii), ptr(angles), radii.numel(), ptr(cosines), ptr(sines), stream)
    check(rc, "bssm_rotation_coefficients")


def rotation_coefficients_backward(radii, angles, grad_cosines, grad_sines, grad_radii, grad_angles, stream) -> None:
    rc = load().bssm_rotation_coefficients_backward(ptr(radii), ptr(angles), ptr(grad_cosines), ptr(grad_sines),
                                                    radii.numel(), ptr(grad_radii), ptr(grad_angles), stream)
    check(rc, "bssm_rotation_coefficients_backward")


def backward_chunked_noalloc(key_dim, value_dim, io_dtype, fixed, need_dynamics, need_initial, keys,
                             values, queries, decay, process, observation, mean0, cov0, bmean, bcov,
                             gy, gmf, gcf, gk, gv, gq, gd, gp, gr, gm0, gc0, n, t, chunks, floor,
                             stream) -> None:
    """The allocation-free backward (static device scratch; see the header)."""
    lib = load()
    rc = lib.bssm_backward_chunked_noalloc(
        key_dim, value_dim, io_dtype, int(fixed), int(need_dynamics), int(need_initial), ptr(keys),
        ptr(values), ptr(queries), ptr(decay), ptr(process), ptr(observation), ptr(mean0), ptr(cov0),
        ptr(bmean), ptr(bcov), ptr(gy), ptr(gmf), ptr(gcf), ptr(gk), ptr(gv), ptr(gq), ptr(gd),
        ptr(gp), ptr(gr), ptr(gm0), ptr(gc0), n, t, chunks, float(floor), stream)
    check(rc, "bssm_backward_chunked_noalloc")


def check_values(tensors) -> list[int]:
    """Flags (CHECK_*) of each contiguous CUDA tensor in ``tensors`` (float32,
    bfloat16 or float16), from one pass per tensor on the current stream and
    one read-back for all of them."""
    import torch
    codes = {torch.float32: BSSM_F32, torch.bfloat16: BSSM_BF16, torch.float16: BSSM_F16}
    lib = load()
    dev = tensors[0].device
    flags = torch.zeros(len(tensors), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for i, x in enumerate(tensors):
        check(lib.bssm_check_values(ptr(x), x.numel(), codes[x.dtype], flags.data_ptr() + 4 * i, stream),
              "check_values")
    return [int(f) for f in flags.tolist()]


def wait_timeouts() -> int:
    """Bounded in-kernel waits that gave up since load (0 in a healthy run)."""
    return int(load().bssm_debug_wait_timeouts())


class WaitTimeout(KernelError):
    """A bounded wait inside a recurrence kernel gave up: outputs are wrong."""


BSSM_ERR_TIMEOUT = 6


def stream_status(stream) -> None:
    """Synchronise ``stream`` and raise :class:`WaitTimeout` if a bounded
    in-kernel wait on this device gave up since the previous check (each
    give-up is reported once), :class:`KernelError` on a CUDA error."""
    lib = load()
    rc = lib.bssm_stream_status(stream)
    if rc == BSSM_ERR_TIMEOUT:
        raise WaitTimeout(lib.bssm_last_error().decode(errors="replace"))
    check(rc, "bssm_stream_status")


def fma_probe(out, blocks, iters, stream) -> int:
    """Enqueue the FP32 FMA throughput probe; returns its flop count."""
    lib = load()
    check(lib.bssm_debug_fma_probe(ptr(out), int(blocks), int(iters), stream), "bssm_debug_fma_probe")
    return int(lib.bssm_debug_fma_probe_flops(int(blocks), int(iters)))


def wait_probe(limit, stream) -> None:
    """Diagnostic: make one bounded wait give up (see the C header)."""
    check(load().bssm_debug_wait_probe(int(limit), stream), "bssm_debug_wait_probe")


FAMILIES = {0: None, 1: "chain", 2: "staged", 3: "v1", 4: "tile64"}


def last_family() -> str | None:
    """Kernel family of this thread's last forward/backward call."""
    return FAMILIES[int(load().bssm_debug_last_family())]


def envelope_partial_floats(batch, tokens, heads, key_dim, head_dim) -> int:
    return int(load().bssm_envelope_partial_floats(batch, tokens, heads, key_dim, head_dim))


def envelope_prologue(projected, in_dtype, batch, tokens, heads, key_dim, head_dim, row_stride, conv_weight,
                      aux_bias, keys, queries, values, out_dtype, decay, process, observation, stream,
                      check_flags=None) -> None:
    """``check_flags``: None, or a zeroed int32 tensor of 6 words that receives
    the CHECK_* flags of keys, values, queries, decay, process, observation."""
    rc = load().bssm_envelope_prologue(ptr(projected), in_dtype, batch, tokens, heads, key_dim, head_dim,
                                       row_stride, ptr(conv_weight), ptr(aux_bias), ptr(keys), ptr(queries),
                                       ptr(values), out_dtype, ptr(decay), ptr(process), ptr(observation),
                                       ptr(check_flags), stream)
    check(rc, "bssm_envelope_prologue")


def envelope_prologue_backward(projected, in_dtype, batch, tokens, heads, key_dim, head_dim, row_stride,
                               conv_weight, aux_bias, gk, gq, gv, out_dtype, gdecay, gprocess, gobservation,
                               gprojected, grad_row_stride, gconv_weight, gaux_bias, workspace, stream) -> None:
    rc = load().bssm_envelope_prologue_backward(
        ptr(projected), in_dtype, batch, tokens, heads, key_dim, head_dim, row_stride, ptr(conv_weight),
        ptr(aux_bias), ptr(gk), ptr(gq), ptr(gv), out_dtype, ptr(gdecay), ptr(gprocess), ptr(gobservation),
        ptr(gprojected), grad_row_stride, ptr(gconv_weight), ptr(gaux_bias), ptr(workspace),
        0 if workspace is None else workspace.numel(), stream)
    check(rc, "bssm_envelope_prologue_backward")


def envelope_epilogue_partial_floats(batch, tokens, heads, head_dim) -> int:
    return int(load().bssm_envelope_epilogue_partial_floats(batch, tokens, heads, head_dim))


def envelope_epilogue(read, read_dtype, gate, gate_dtype, gate_row_stride, norm_weight, eps, batch, tokens, heads,
                      head_dim, out, stream) -> None:
    rc = load().bssm_envelope_epilogue(ptr(read), read_dtype, ptr(gate), gate_dtype, gate_row_stride,
                                       ptr(norm_weight), float(eps), batch, tokens, heads, head_dim, ptr(out), stream)
    check(rc, "bssm_envelope_epilogue")


def envelope_epilogue_backward(read, read_dtype, gate, gate_dtype, gate_row_stride, norm_weight, eps, batch, tokens,
                               heads, head_dim, grad_out, grad_read, grad_gate, grad_gate_row_stride,
                               grad_norm_weight, workspace, stream) -> None:
    rc = load().bssm_envelope_epilogue_backward(
        ptr(read), read_dtype, ptr(gate), gate_dtype, gate_row_stride, ptr(norm_weight), float(eps), batch, tokens,
        heads, head_dim, ptr(grad_out), ptr(grad_read), ptr(grad_gate), grad_gate_row_stride, ptr(grad_norm_weight),
        ptr(workspace), 0 if workspace is None else workspace.numel(), stream)
    check(rc, "bssm_envelope_epilogue_backward")


def rms_norm(x, dtype, rows, width, weight, eps, out, stream) -> None:
    check(load().bssm_rms_norm(ptr(x), dtype, rows, width, ptr(weight), float(eps), ptr(out), stream), "bssm_rms_norm")


def rms_norm_partial_floats(rows, width) -> int:
    return int(load().bssm_rms_norm_partial_floats(rows, width))


def rms_norm_backward(x, dtype, rows, width, weight, eps, grad_out, grad_x, grad_weight, workspace, stream) -> None:
    rc = load().bssm_rms_norm_backward(ptr(x), dtype, rows, width, ptr(weight), float(eps), ptr(grad_out),
                                       ptr(grad_x), ptr(grad_weight), ptr(workspace),
                                       0 if workspace is None else workspace.numel(), stream)
    check(rc, "bssm_rms_norm_backward")
