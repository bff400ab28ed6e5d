"""Generate the golden vectors in this folder from the REFERENCE's own code.

Test infrastructure.  Run where the reference tree is mounted, after
`python -m oracle.build_ref` has compiled the reference sources into
oracle/_ref/ (libref_sem3d.so: bench_sem3d_levelgraph.cpp's fill() and host
reference(); libref_sem2d.so: bench_sem_stiffness.cpp's fill_field(),
fill_operators() and host_reference()):

    python tests/golden/make_golden.py

Writes
  sem3d_ref_fill_E6.npz  the 3D program's 15 fill() inputs for E=6 (NGLL 5),
                         the operators it builds, and its host reference's
                         three force components;
  sem2d_ref_fill_E5.npz  the 2D program's nine fill_field() inputs for E=5
                         (NGLL 8), its fill_operators() H, Hw, w, and its
                         host_reference() f0, f1.
The tests (tests/test_golden_cpu.py, tests/test_golden_gpu.py) only read these
files; nothing at run time needs the reference tree.
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
REF = ROOT / "oracle" / "_ref"

NAMES3 = ["u0", "u1", "u2", "xix", "xiy", "xiz", "etax", "etay", "etaz", "gamx", "gamy", "gamz",
          "l2m", "mu", "jac"]
NAMES2 = ["u0", "u1", "xix", "xiz", "gamx", "gamz", "l2m", "mu", "jac"]


def _pp(arrs):
    return (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


def _vp(a):
    return a.ctypes.data_as(C.c_void_p)


def golden_3d(E=6):
    sys.path.insert(0, str(ROOT))
    from tensoroperations_b200.sem3d import reference_fill_problem
    lib = C.CDLL(str(REF / "libref_sem3d.so"))
    N = 5
    P = N ** 3
    ins = [np.empty(E * P, np.float32) for _ in NAMES3]
    assert lib.ref_sem3d_fill(E, _pp(ins)) == N
    # the operators the reference builds (:767-776), evaluated in f32
    p = reference_fill_problem(1)
    H, Hw, w = (np.ascontiguousarray(x, dtype=np.float32) for x in (p.H, p.Hw, p.w))
    r = [np.empty(E * P, np.float32) for _ in range(3)]
    lib.ref_sem3d_reference(C.c_int(E), _pp(ins), _vp(H), _vp(Hw), _vp(w), _vp(r[0]), _vp(r[1]),
                            _vp(r[2]))
    np.savez_compressed(HERE / f"sem3d_ref_fill_E{E}.npz", E=E, ngll=N, H=H, Hw=Hw, w=w,
                        **dict(zip(NAMES3, ins)), f0=r[0], f1=r[1], f2=r[2])


def golden_2d(E=5):
    lib = C.CDLL(str(REF / "libref_sem2d.so"))
    N = lib.ref_sem2d_ngll()
    ins = [np.empty(E * N * N, np.float32) for _ in NAMES2]
    H = np.empty(N * N, np.float32)
    Hw = np.empty(N * N, np.float32)
    w = np.empty(N, np.float32)
    assert lib.ref_sem2d_fill(E, _pp(ins), _vp(H), _vp(Hw), _vp(w)) == N
    f0 = np.empty(E * N * N, np.float32)
    f1 = np.empty(E * N * N, np.float32)
    lib.ref_sem2d_reference(E, _pp(ins), _vp(H), _vp(Hw), _vp(w), _vp(f0), _vp(f1))
    np.savez_compressed(HERE / f"sem2d_ref_fill_E{E}.npz", E=E, ngll=N, H=H, Hw=Hw, w=w,
                        **dict(zip(NAMES2, ins)), f0=f0, f1=f1)


if __name__ == "__main__":
    golden_3d()
    golden_2d()
    print(sorted(p.name for p in HERE.glob("*.npz")))
