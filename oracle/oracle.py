"""ctypes front end for the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module, and only to check or to time the reference algorithm
on the host.  The shipped package never imports it.

The restated algorithm and its reference citations are documented in
``oracle/bayes_oracle.c``.  Arrays are numpy, row-major, with the layouts
listed there; ``precision`` selects the FP64 checker or the FP32 build.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle_bayes.so"
_LIB: Optional[ctypes.CDLL] = None


class OracleError(RuntimeError):
    pass


def build() -> Path:
    """Compile the oracle shared library in place (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def _lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            build()
        _LIB = ctypes.CDLL(str(LIB_PATH))
        for sfx in ("_f64", "_f32"):
            getattr(_LIB, "oracle_num_threads" + sfx).restype = ctypes.c_int
    return _LIB


def num_threads() -> int:
    return int(_lib().oracle_num_threads_f64())


_CODES = {-1: "bad arguments", -2: "observation variance below the floor or non-finite",
          -3: "out of memory", -4: "Cholesky failure (precision not positive definite)"}


def _prep(x, dtype):
    if x is None:
        return None, None
    arr = np.ascontiguousarray(x, dtype=dtype)
    return arr, arr.ctypes.data_as(ctypes.c_void_p)


def _real(precision: str):
    if precision == "f64":
        return np.float64, ctypes.c_double, "_f64"
    if precision == "f32":
        return np.float32, ctypes.c_float, "_f32"
    raise ValueError(precision)


def forward(k, v, q, a=None, p=None, r=None, M0=None, P0=None, *, floor=1e-6,
            fixed=False, precision="f64"):
    """Return (y [n,t,m], M_T [n,d,m], P_T [n,d,d])."""
    dt, creal, sfx = _real(precision)
    n, t, d = np.shape(k)
    m = np.shape(v)[-1]
    keep = [_prep(x, dt) for x in (k, v, q, a, p, r, M0, P0)]
    y = np.zeros((n, t, m), dt)
    mt = np.zeros((n, d, m), dt)
    pt = np.zeros((n, d, d), dt)
    fn = getattr(_lib(), "oracle_forward" + sfx)
    rc = fn(ctypes.c_long(n), ctypes.c_long(t), ctypes.c_int(d), ctypes.c_int(m),
            *[ptr for _, ptr in keep], creal(floor), ctypes.c_int(int(fixed)),
            y.ctypes.data_as(ctypes.c_void_p), mt.ctypes.data_as(ctypes.c_void_p),
            pt.ctypes.data_as(ctypes.c_void_p))
    if rc:
        raise OracleError(_CODES.get(rc, str(rc)))
    return y, mt, pt


def backward(k, v, q, a=None, p=None, r=None, M0=None, P0=None, gy=None, gMT=None, gPT=None,
             *, floor=1e-6, fixed=False, precision="f64"):
    """Return dict of gradients: k, v, q, a, p, r, M0, P0."""
    dt, creal, sfx = _real(precision)
    n, t, d = np.shape(k)
    m = np.shape(v)[-1]
    keep = [_prep(x, dt) for x in (k, v, q, a, p, r, M0, P0)]
    gkeep = [_prep(x, dt) for x in (gy, gMT, gPT)]
    out = dict(k=np.zeros((n, t, d), dt), v=np.zeros((n, t, m), dt), q=np.zeros((n, t, d), dt),
               a=np.zeros((n, t, d), dt), p=np.zeros((n, t), dt), r=np.zeros((n, t), dt),
               M0=np.zeros((n, d, m), dt), P0=np.zeros((n, d, d), dt))
    fn = getattr(_lib(), "oracle_backward" + sfx)
    rc = fn(ctypes.c_long(n), ctypes.c_long(t), ctypes.c_int(d), ctypes.c_int(m),
            *[ptr for _, ptr in keep], creal(floor), ctypes.c_int(int(fixed)),
            *[ptr for _, ptr in gkeep],
            *[out[x].ctypes.data_as(ctypes.c_void_p) for x in ("k", "v", "q", "a", "p", "r", "M0", "P0")])
    if rc:
        raise OracleError(_CODES.get(rc, str(rc)))
    return out


def assoc_scan(k, v, q, r=None, M0=None, P0=None, *, floor=1e-6, precision="f64"):
    """Return (y, M_T, P_T) of the static information-form scan."""
    dt, creal, sfx = _real(precision)
    n, t, d = np.shape(k)
    m = np.shape(v)[-1]
    keep = [_prep(x, dt) for x in (k, v, q, r, M0, P0)]
    y = np.zeros((n, t, m), dt)
    mt = np.zeros((n, d, m), dt)
    pt = np.zeros((n, d, d), dt)
    fn = getattr(_lib(), "oracle_assoc_scan" + sfx)
    rc = fn(ctypes.c_long(n), ctypes.c_long(t), ctypes.c_int(d), ctypes.c_int(m),
            *[ptr for _, ptr in keep], creal(floor),
            y.ctypes.data_as(ctypes.c_void_p), mt.ctypes.data_as(ctypes.c_void_p),
            pt.ctypes.data_as(ctypes.c_void_p))
    if rc:
        raise OracleError(_CODES.get(rc, str(rc)))
    return y, mt, pt


def set_threads(n: int) -> None:
    """Set the OpenMP thread count for subsequent oracle calls (before first use)."""
    os.environ["OMP_NUM_THREADS"] = str(int(n))
