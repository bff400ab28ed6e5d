"""Inputs of the 2D elastic P-SV operator (element-local, NGLL 8, f32).

Two fills, both [E][j][i] per array:
* `reference_fill_2d`: the reference benchmark's own deterministic fill,
  restated (benchmarks/sem_stiffness/bench_sem_stiffness.cpp:1306-1331):
  v(e,j,i) = (((e + 3j + 5i + salt) mod 7) + 1) / 8 with salts u0 0, u1 1,
  xix 2, xiz 3, gamx 4, gamz 5, l2m 6, mu 7, jac 8 (:1476-1484);
  H(a,b) = (((3a + 2b) mod 5) - 2) / 2, w(a) = 1/2 + (a mod 3) / 8,
  Hw(a,b) = w(a) H(a,b).
* `synthetic_2d`: seeded splitmix64 fields with the 3D configuration's
  distributions (inverse Jacobian U[0.5,1.5) + 1 on xix and gamz, jac
  U[0.5,2), lambda U[1,3), mu U[0.5,2), l2m = lambda + 2 mu, u N(0,1)) and the
  true GLL operators.
"""
from __future__ import annotations

import numpy as np

from . import abi

N2D = 8
ARRAYS = abi.SEM2D_ARRAYS


def reference_fill_2d(nelem: int):
    N = N2D
    e = np.arange(nelem)[:, None, None]
    j = np.arange(N)[None, :, None]
    i = np.arange(N)[None, None, :]

    def fill(salt):
        return ((((e + 3 * j + 5 * i + salt) % 7) + 1).astype(np.float32) * np.float32(0.125)).reshape(-1)

    salts = {"u0": 0, "u1": 1, "xix": 2, "xiz": 3, "gamx": 4, "gamz": 5, "l2m": 6, "mu": 7, "jac": 8}
    vals = {k: fill(v) for k, v in salts.items()}
    a = np.arange(N)
    w = (np.float32(0.5) + np.float32(0.125) * (a % 3).astype(np.float32)).astype(np.float32)
    H = ((((3 * a[:, None] + 2 * a[None, :]) % 5) - 2).astype(np.float32) * np.float32(0.5)).astype(np.float32)
    Hw = (w[:, None] * H).astype(np.float32)
    arrays = {k: vals[k] for k in ARRAYS}
    return [vals["u0"], vals["u1"]], arrays, H.astype(np.float64), Hw.astype(np.float64), w.astype(np.float64)


def synthetic_2d(nelem: int, seed: int = 0x2D5EED, dtype=np.float32):
    dt = np.dtype(dtype)
    N = N2D
    npts = nelem * N * N
    _, w, H, Hw = abi.gll_operators(N)
    arrays = {}
    for r, name in enumerate(("xix", "xiz", "gamx", "gamz")):
        a = abi.synth_fill(npts, np.float64, seed + 3 + r, "uniform", 0.5, 1.5)
        if name in ("xix", "gamz"):
            a += 1.0
        arrays[name] = a.astype(dt)
    arrays["jac"] = abi.synth_fill(npts, dt, seed + 12, "uniform", 0.5, 2.0)
    lam = abi.synth_fill(npts, dt, seed + 13, "uniform", 1.0, 3.0)
    mu = abi.synth_fill(npts, dt, seed + 14, "uniform", 0.5, 2.0)
    arrays["l2m"] = (lam + dt.type(2) * mu).astype(dt)
    arrays["mu"] = mu
    u = [abi.synth_fill(npts, dt, seed + c, "normal", 0.0, 1.0) for c in range(2)]
    return u, arrays, H, Hw, w


def structured_ibool_2d(nex: int, nez: int, ngll: int) -> np.ndarray:
    """Shared-node numbering of an nex x nez quad mesh: element e = ez*nex + ex,
    node(e, j, i) = (ez (N-1) + j) nx + ex (N-1) + i, nx = nex (N-1) + 1."""
    n1 = ngll - 1
    nx = nex * n1 + 1
    e = np.arange(nex * nez)
    ex, ez = e % nex, e // nex
    j = np.arange(ngll)[None, :, None]
    i = np.arange(ngll)[None, None, :]
    ib = (ez[:, None, None] * n1 + j) * nx + ex[:, None, None] * n1 + i
    return ib.reshape(-1).astype(np.int32)


def acoustic_problem(nex: int = 128, nez: int = 128, ngll: int = 5, dtype=np.float64,
                     seed: int = 0xAC0571C):
    """The first configuration: structured quads, GLL operators, seeded fields:
    xix, xiz, gamx, gamz U[0.5,1.5); jac U[0.5,2); rho, kappa U[1,3); u N(0,1)
    per global node.  Returns (u, arrays, ibool, nglob, H, Hw, w)."""
    dt = np.dtype(dtype)
    P = ngll * ngll
    E = nex * nez
    _, w, H, Hw = abi.gll_operators(ngll)
    arrays = {}
    for r, name in enumerate(("xix", "xiz", "gamx", "gamz")):
        arrays[name] = abi.synth_fill(E * P, dt, seed + 1 + r, "uniform", 0.5, 1.5)
    arrays["jac"] = abi.synth_fill(E * P, dt, seed + 5, "uniform", 0.5, 2.0)
    arrays["rho"] = abi.synth_fill(E * P, dt, seed + 6, "uniform", 1.0, 3.0)
    arrays["kappa"] = abi.synth_fill(E * P, dt, seed + 7, "uniform", 1.0, 3.0)
    n1 = ngll - 1
    nglob = (nex * n1 + 1) * (nez * n1 + 1)
    u = abi.synth_fill(nglob, dt, seed, "normal", 0.0, 1.0)
    return u, arrays, structured_ibool_2d(nex, nez, ngll), nglob, H, Hw, w
