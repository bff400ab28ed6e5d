"""Pin the CPU oracle to the reference's own code (no GPU).

oracle/_ref/libref_sem3d.so is the reference benchmark source
benchmarks/sem_stiffness_3d/bench_sem3d_levelgraph.cpp compiled from where it
lies (oracle/build_ref.py): its fill() makes the reference's deterministic
inputs and its reference() is the reference's own host loop of the SEM 3D
operator (:600-663).  The oracle's f32 element-local entry point restates that
loop with the same operation order, so on identical inputs the two must agree
BIT FOR BIT; the fp64 restatement must agree to f32 rounding.

The library is built here (where the reference tree is mounted) and shipped
with the repository; without it these tests skip.
"""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle import sem as osem
from tensoroperations_b200.sem3d import reference_fill_problem

LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libref_sem3d.so"
N = 5
P = N ** 3
NAMES = ["u0", "u1", "u2", "xix", "xiy", "xiz", "etax", "etay", "etaz", "gamx", "gamy", "gamz",
         "l2m", "mu", "jac"]

pytestmark = pytest.mark.skipif(not LIB.exists(), reason="oracle/_ref not built (no reference tree)")


def _lib():
    lib = C.CDLL(str(LIB))
    lib.ref_sem3d_fill.restype = C.c_int
    lib.ref_sem3d_reference.restype = None
    return lib


def _ptrs(arrs):
    return (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


def reference_inputs(E):
    lib = _lib()
    out = [np.empty(E * P, dtype=np.float32) for _ in range(15)]
    assert lib.ref_sem3d_fill(E, _ptrs(out)) == N
    return dict(zip(NAMES, out))


def reference_operators():
    # bench_sem3d_levelgraph.cpp:767-776, evaluated once in f32 (any H pins the
    # operator; these are the benchmark's own values up to sinf rounding)
    p = reference_fill_problem(1)
    return tuple(np.ascontiguousarray(x, dtype=np.float32) for x in (p.H, p.Hw, p.w))


def reference_operator(E, inputs, H, Hw, w):
    lib = _lib()
    H, Hw, w = (np.ascontiguousarray(x, dtype=np.float32) for x in (H, Hw, w))
    inputs = {n: np.ascontiguousarray(inputs[n], dtype=np.float32) for n in NAMES}
    r = [np.empty(E * P, dtype=np.float32) for _ in range(3)]
    lib.ref_sem3d_reference(C.c_int(E), _ptrs([inputs[n] for n in NAMES]),
                            H.ctypes.data_as(C.c_void_p), Hw.ctypes.data_as(C.c_void_p),
                            w.ctypes.data_as(C.c_void_p), r[0].ctypes.data_as(C.c_void_p),
                            r[1].ctypes.data_as(C.c_void_p), r[2].ctypes.data_as(C.c_void_p))
    return r


def test_reference_fill_matches_the_python_restatement():
    E = 37
    got = reference_inputs(E)
    mine = reference_fill_problem(E)
    for n in NAMES:
        src = mine.u[int(n[1])] if n in ("u0", "u1", "u2") else mine.arrays[n]
        np.testing.assert_allclose(got[n], src, rtol=2e-7, atol=0)


@pytest.mark.parametrize("E", [1, 11, 40])
def test_oracle_f32_is_bit_exact_with_the_reference_host_loop(E):
    inp = reference_inputs(E)
    H, Hw, w = reference_operators()
    ref = reference_operator(E, inp, H, Hw, w)
    arrays = {n: inp[n] for n in NAMES[3:]}
    got = osem.local(E, N, [inp["u0"], inp["u1"], inp["u2"]], arrays, H, Hw, w, np.float32)
    for c in range(3):
        assert np.array_equal(got[c], ref[c]), (c, np.max(np.abs(got[c] - ref[c])))


def test_oracle_f64_agrees_with_the_reference_host_loop():
    E = 40
    inp = reference_inputs(E)
    H, Hw, w = reference_operators()
    ref = reference_operator(E, inp, H, Hw, w)
    arrays = {n: inp[n].astype(np.float64) for n in NAMES[3:]}
    u = [inp[n].astype(np.float64) for n in ("u0", "u1", "u2")]
    got = osem.local(E, N, u, arrays, H.astype(np.float64), Hw.astype(np.float64),
                     w.astype(np.float64), np.float64)
    assert osem.rel_l2(ref, got) < 1e-6


def test_oracle_matches_reference_on_synthetic_random_inputs():
    """The pin on this build's own seeded inputs and true GLL operators."""
    from tensoroperations_b200.sem3d import structured_problem
    p = structured_problem(3, 2, 2, ngll=5, dtype=np.float32, assembled=False, seed=77)
    inp = {"u0": p.u[0], "u1": p.u[1], "u2": p.u[2], **p.arrays}
    H, Hw, w = (x.astype(np.float32) for x in (p.H, p.Hw, p.w))
    ref = reference_operator(p.nelem, inp, H, Hw, w)
    got = osem.local(p.nelem, N, p.u, p.arrays, H, Hw, w, np.float32)
    for c in range(3):
        assert np.array_equal(got[c], ref[c])
