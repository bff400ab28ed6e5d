"""ctypes front of the CPU oracle (sem_oracle.cpp).  Test infrastructure only.

`local` / `assembled` call the exact-order parity build (libsem_oracle.so);
`assembled_omp` calls the OpenMP build that bench.py times as the CPU port.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import build as _build

_build.build()
_exact = C.CDLL(str(_build.ORACLE))
_fast = C.CDLL(str(_build.CPU))

_POINT_ORDER = ("xix", "xiy", "xiz", "etax", "etay", "etaz", "gamx", "gamy", "gamz",
                "jac", "l2m", "mu")


def _pp(arrs):
    return (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


def _check_dtype(dt, arrays):
    for a in arrays:
        assert a.dtype == dt and a.flags.c_contiguous, (a.dtype, dt)


def _cfun(lib, name):
    f = getattr(lib, name)
    f.restype = None
    return f


def local(nelem, ngll, u, arrays, H, Hw, w, dtype):
    """Element-local operator: u[c] and the result are [E*N^3] per component."""
    dt = np.dtype(dtype)
    P = ngll ** 3
    m = [np.ascontiguousarray(arrays[n], dtype=dt) for n in _POINT_ORDER]
    uu = [np.ascontiguousarray(x, dtype=dt) for x in u]
    f = [np.zeros(nelem * P, dtype=dt) for _ in range(3)]
    ops = [np.ascontiguousarray(x, dtype=dt) for x in (H, Hw, w)]
    name = "oracle_sem3d_local_f32" if dt == np.float32 else "oracle_sem3d_local_f64"
    _cfun(_exact, name)(C.c_int64(nelem), C.c_int(ngll), _pp(uu), _pp(m), ops[0].ctypes.data_as(C.c_void_p),
                        ops[1].ctypes.data_as(C.c_void_p), ops[2].ctypes.data_as(C.c_void_p), _pp(f))
    return f


def assembled(nelem, ngll, nglob, ibool, u, arrays, H, Hw, w, dtype):
    """Assembled operator: gather u[c][nglob] through ibool, scatter-add in element order."""
    dt = np.dtype(dtype)
    m = [np.ascontiguousarray(arrays[n], dtype=dt) for n in _POINT_ORDER]
    uu = [np.ascontiguousarray(x, dtype=dt) for x in u]
    f = [np.zeros(nglob, dtype=dt) for _ in range(3)]
    ib = np.ascontiguousarray(ibool, dtype=np.int32)
    ops = [np.ascontiguousarray(x, dtype=dt) for x in (H, Hw, w)]
    name = "oracle_sem3d_assembled_f32" if dt == np.float32 else "oracle_sem3d_assembled_f64"
    _cfun(_exact, name)(C.c_int64(nelem), C.c_int(ngll), C.c_int64(nglob), ib.ctypes.data_as(C.c_void_p),
                        _pp(uu), _pp(m), ops[0].ctypes.data_as(C.c_void_p),
                        ops[1].ctypes.data_as(C.c_void_p), ops[2].ctypes.data_as(C.c_void_p), _pp(f))
    return f


SEM2D_POINT_ORDER = ("xix", "xiz", "gamx", "gamz", "jac", "l2m", "mu")


def sem2d_local(nelem, ngll, u, arrays, H, Hw, w, dtype):
    """2D elastic P-SV element-local operator: u[c] and the result are [E*N^2] (c = 0, 1)."""
    dt = np.dtype(dtype)
    m = [np.ascontiguousarray(arrays[n], dtype=dt) for n in SEM2D_POINT_ORDER]
    uu = [np.ascontiguousarray(x, dtype=dt) for x in u]
    f = [np.zeros(nelem * ngll * ngll, dtype=dt) for _ in range(2)]
    ops = [np.ascontiguousarray(x, dtype=dt) for x in (H, Hw, w)]
    name = "oracle_sem2d_local_f32" if dt == np.float32 else "oracle_sem2d_local_f64"
    _cfun(_exact, name)(C.c_int64(nelem), C.c_int(ngll), _pp(uu), _pp(m),
                        ops[0].ctypes.data_as(C.c_void_p), ops[1].ctypes.data_as(C.c_void_p),
                        ops[2].ctypes.data_as(C.c_void_p), _pp(f))
    return f


ACOUSTIC_ORDER = ("xix", "xiz", "gamx", "gamz", "jac", "rho")


def sem2d_acoustic(nelem, ngll, nglob, ibool, u, arrays, H, Hw, w, dtype):
    """2D acoustic assembled operator (scalar u[nglob] -> f[nglob])."""
    dt = np.dtype(dtype)
    m = [np.ascontiguousarray(arrays[n], dtype=dt) for n in ACOUSTIC_ORDER]
    uu = np.ascontiguousarray(u, dtype=dt)
    f = np.zeros(nglob, dtype=dt)
    ib = np.ascontiguousarray(ibool, dtype=np.int32)
    ops = [np.ascontiguousarray(x, dtype=dt) for x in (H, Hw, w)]
    name = "oracle_sem2d_acoustic_f64" if dt == np.float64 else "oracle_sem2d_acoustic_f32"
    _cfun(_exact, name)(C.c_int64(nelem), C.c_int(ngll), C.c_int64(nglob),
                        ib.ctypes.data_as(C.c_void_p), uu.ctypes.data_as(C.c_void_p), _pp(m),
                        ops[0].ctypes.data_as(C.c_void_p), ops[1].ctypes.data_as(C.c_void_p),
                        ops[2].ctypes.data_as(C.c_void_p), f.ctypes.data_as(C.c_void_p))
    return f


def colouring(nelem, ngll, nglob, ibool):
    """(ncolours, colour_start[ncol+1], colour_elems[E]) of a greedy element colouring."""
    col = np.empty(nelem, dtype=np.int32)
    fn = _exact.oracle_colour_elements
    fn.restype = C.c_int
    ib = np.ascontiguousarray(ibool, dtype=np.int32)
    n = fn(C.c_int64(nelem), C.c_int(ngll), C.c_int64(nglob), ib.ctypes.data_as(C.c_void_p),
           col.ctypes.data_as(C.c_void_p))
    if n < 0:
        raise RuntimeError("colouring needs more than 64 colours")
    order = np.argsort(col, kind="stable").astype(np.int64)
    counts = np.bincount(col, minlength=n)
    start = np.zeros(n + 1, dtype=np.int64)
    start[1:] = np.cumsum(counts)
    return n, start, order, col


class AssembledCPU:
    """The timed CPU port: colour-parallel OpenMP assembled operator."""

    def __init__(self, nelem, ngll, nglob, ibool, arrays, H, Hw, w, dtype):
        self.dt = np.dtype(dtype)
        self.nelem, self.ngll, self.nglob = nelem, ngll, nglob
        self.ib = np.ascontiguousarray(ibool, dtype=np.int32)
        self.m = [np.ascontiguousarray(arrays[n], dtype=self.dt) for n in _POINT_ORDER]
        self.ops = [np.ascontiguousarray(x, dtype=self.dt) for x in (H, Hw, w)]
        self.ncol, self.start, self.order, _ = colouring(nelem, ngll, nglob, self.ib)
        self._mp = _pp(self.m)
        name = ("oracle_sem3d_assembled_omp_f32" if self.dt == np.float32
                else "oracle_sem3d_assembled_omp_f64")
        self.fn = _cfun(_fast, name)

    def __call__(self, u, f):
        uu = [np.ascontiguousarray(x, dtype=self.dt) for x in u]
        self.fn(C.c_int64(self.nelem), C.c_int(self.ngll), C.c_int64(self.nglob),
                self.ib.ctypes.data_as(C.c_void_p), _pp(uu), self._mp,
                self.ops[0].ctypes.data_as(C.c_void_p), self.ops[1].ctypes.data_as(C.c_void_p),
                self.ops[2].ctypes.data_as(C.c_void_p), _pp(f), C.c_int(self.ncol),
                self.start.ctypes.data_as(C.c_void_p), self.order.ctypes.data_as(C.c_void_p))
        return f


def num_threads() -> int:
    fn = _fast.oracle_num_threads
    fn.restype = C.c_int
    return fn()


def host_cores() -> int:
    """Cores this process may run on (its CPU affinity set)."""
    import os
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def set_num_threads(n: int) -> int:
    """Threads of the OpenMP CPU port (ignores OMP_NUM_THREADS); returns the count now in use."""
    fn = _fast.oracle_set_num_threads
    fn.restype = None
    fn(C.c_int(int(n)))
    return num_threads()


def rel_l2(a, b) -> float:
    """Relative L2 error of a against reference b over all components."""
    a = np.concatenate([np.asarray(x, dtype=np.float64).ravel() for x in a])
    b = np.concatenate([np.asarray(x, dtype=np.float64).ravel() for x in b])
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))
