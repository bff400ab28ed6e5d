"""Synthetic SEM 3D elastic problems (host arrays) and their device upload.

Inputs follow the configuration of the hot path's benchmark: a structured
nex x ney x nez hexahedral mesh, GLL operators computed (not drawn), and one
splitmix64 seed per array:

  array            seed            distribution
  u0, u1, u2       seed + 0..2     Normal(0, 1) per global node (or per point)
  xix .. gmz       seed + 3..11    Uniform[0.5, 1.5), + 1.0 on xix, etay, gamz
  jac              seed + 12       Uniform[0.5, 2.0)
  lambda           seed + 13       Uniform[1, 3)
  mu               seed + 14       Uniform[0.5, 2)
  l2m = lambda + 2 mu, evaluated in the working dtype.

The reference's own benchmark fills (deterministic sin/cos,
benchmarks/sem_stiffness_3d/bench_sem3d_levelgraph.cpp:588-598,767-779) are
available through `reference_fill_problem` for the pin against the reference.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import abi

DEFAULT_SEED = 0x5EED2026


@dataclass
class Sem3dProblem:
    ngll: int
    nelem: int
    dtype: np.dtype
    H: np.ndarray
    Hw: np.ndarray
    w: np.ndarray
    arrays: dict  # POINT_ARRAYS name -> [E*P]
    u: list  # 3 arrays: [nglob] (assembled) or [E*P]
    ibool: np.ndarray | None = None
    nglob: int = 0
    mesh: tuple = field(default_factory=tuple)

    @property
    def assembled(self) -> bool:
        return self.ibool is not None

    @property
    def npoints(self) -> int:
        return self.nelem * self.ngll ** 3

    def plan(self) -> abi.Sem3dPlan:
        return abi.Sem3dPlan(self.dtype, self.ngll, self.nelem, self.H, self.Hw, self.w,
                             nglob=self.nglob, assembled=self.assembled)


def point_arrays(npts: int, dtype, seed: int = DEFAULT_SEED, first: int = 0) -> dict:
    """The per-point arrays of points [first, first + npts) of a problem."""
    dt = np.dtype(dtype)
    out = {}
    for r, name in enumerate(abi.POINT_ARRAYS[:9]):
        a = abi.synth_fill(npts, np.float64, seed + 3 + r, "uniform", 0.5, 1.5, first=first)
        if name in ("xix", "etay", "gamz"):
            a += 1.0
        out[name] = a.astype(dt)
    out["jac"] = abi.synth_fill(npts, dt, seed + 12, "uniform", 0.5, 2.0, first=first)
    lam = abi.synth_fill(npts, dt, seed + 13, "uniform", 1.0, 3.0, first=first)
    mu = abi.synth_fill(npts, dt, seed + 14, "uniform", 0.5, 2.0, first=first)
    out["l2m"] = (lam + dt.type(2) * mu).astype(dt)
    out["mu"] = mu
    return out


def structured_problem(nex: int, ney: int, nez: int, ngll: int = 5, dtype=np.float32,
                       assembled: bool = True, seed: int = DEFAULT_SEED) -> Sem3dProblem:
    dt = np.dtype(dtype)
    _, w, H, Hw = abi.gll_operators(ngll)
    E = nex * ney * nez
    P = ngll ** 3
    arrays = point_arrays(E * P, dt, seed)
    if assembled:
        ibool = abi.structured_ibool(nex, ney, nez, ngll).reshape(-1)
        n1 = ngll - 1
        nglob = (nex * n1 + 1) * (ney * n1 + 1) * (nez * n1 + 1)
        u = [abi.synth_fill(nglob, dt, seed + c, "normal", 0.0, 1.0) for c in range(3)]
    else:
        ibool, nglob = None, 0
        u = [abi.synth_fill(E * P, dt, seed + c, "normal", 0.0, 1.0) for c in range(3)]
    return Sem3dProblem(ngll, E, dt, H, Hw, w, arrays, u, ibool, nglob, (nex, ney, nez))


def reference_fill_problem(nelem: int, ngll: int = 5) -> Sem3dProblem:
    """The reference benchmark's deterministic inputs, element-local, float32.

    fill(): v(e,k,j,i) = 0.1 sin(0.7 (s+1) (e % 11) + 0.3 k + 0.17 j + 0.11 i) + 0.6
    with s = 0..14 in the order u0,u1,u2,xix,xiy,xiz,etx,ety,etz,gmx,gmy,gmz,l2m,mu,jac;
    H(a,b) = 0.3 sin(1.3 a + 0.7 b) + 0.1 [a == b]; w(a) = 0.2 + 0.05 a;
    Hw(a,b) = H(b,a) w(b)   (bench_sem3d_levelgraph.cpp:588-598, 757-780).
    Evaluated in float32 with the same operation order as the reference (C sinf).
    """
    N = ngll
    e = np.arange(nelem, dtype=np.int64)[:, None, None, None]
    k = np.arange(N)[None, :, None, None]
    j = np.arange(N)[None, None, :, None]
    i = np.arange(N)[None, None, None, :]
    f32 = np.float32

    def fill(s):
        arg = (f32(0.7) * f32(s + 1) * (e % 11).astype(f32) + f32(0.3) * k.astype(f32)
               + f32(0.17) * j.astype(f32) + f32(0.11) * i.astype(f32)).astype(f32)
        return (f32(0.1) * np.sin(arg).astype(f32) + f32(0.6)).astype(f32).reshape(-1)

    names = ["u0", "u1", "u2", "xix", "xiy", "xiz", "etax", "etay", "etaz", "gamx", "gamy",
             "gamz", "l2m", "mu", "jac"]
    vals = {n: fill(s) for s, n in enumerate(names)}
    a = np.arange(N)
    w = (f32(0.2) + f32(0.05) * a.astype(f32)).astype(f32)
    H = (f32(0.3) * np.sin(f32(1.3) * a[:, None].astype(f32) + f32(0.7) * a[None, :].astype(f32))
         .astype(f32) + f32(0.1) * (a[:, None] == a[None, :]).astype(f32)).astype(f32)
    Hw = (H.T * w[None, :]).astype(f32)
    arrays = {n: vals[n] for n in abi.POINT_ARRAYS}
    u = [vals["u0"], vals["u1"], vals["u2"]]
    return Sem3dProblem(N, nelem, np.dtype(f32), H.astype(np.float64), Hw.astype(np.float64),
                        w.astype(np.float64), arrays, u)


def to_device(prob: Sem3dProblem, device="cuda"):
    """Upload a problem: returns (u, f, arrays, ibool) torch tensors on `device`."""
    import torch
    arrays = {n: torch.from_numpy(a).to(device) for n, a in prob.arrays.items()}
    u = [torch.from_numpy(x).to(device) for x in prob.u]
    n_out = prob.nglob if prob.assembled else prob.npoints
    f = [torch.zeros(n_out, dtype=u[0].dtype, device=device) for _ in range(3)]
    ibool = torch.from_numpy(prob.ibool).to(device) if prob.assembled else None
    return u, f, arrays, ibool
