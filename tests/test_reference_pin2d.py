"""Pin the 2D CPU oracle to the reference's own 2D code (no GPU).

oracle/_ref/libref_sem2d.so is benchmarks/sem_stiffness/bench_sem_stiffness.cpp
compiled host-only from where it lies (oracle/build_ref.py, oracle/ref_pin2d.cpp):
its fill_field() / fill_operators() make the reference's deterministic inputs
and its host_reference() (:1335-1385) is the reference's own host loop of the
2D P-SV operator.  The oracle's f32 restatement (sem2d_local) follows that loop
operation for operation, so on identical inputs the two agree BIT FOR BIT; the
Python restatement of the fill (sem2d.reference_fill_2d) must reproduce the
reference's inputs exactly.

The library is built here (where the reference tree is mounted) and shipped
with the repository; without it these tests skip.
"""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle import sem as osem
from tensoroperations_b200.sem2d import reference_fill_2d

LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libref_sem2d.so"
NAMES = ["u0", "u1", "xix", "xiz", "gamx", "gamz", "l2m", "mu", "jac"]

pytestmark = pytest.mark.skipif(not LIB.exists(), reason="oracle/_ref not built (no reference tree)")


def _lib():
    return C.CDLL(str(LIB))


def _pp(arrs):
    return (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


def reference_inputs(E):
    lib = _lib()
    N = lib.ref_sem2d_ngll()
    out = [np.empty(E * N * N, dtype=np.float32) for _ in range(9)]
    H = np.empty(N * N, np.float32)
    Hw = np.empty(N * N, np.float32)
    w = np.empty(N, np.float32)
    assert lib.ref_sem2d_fill(E, _pp(out), H.ctypes.data_as(C.c_void_p),
                              Hw.ctypes.data_as(C.c_void_p), w.ctypes.data_as(C.c_void_p)) == N
    return N, dict(zip(NAMES, out)), H, Hw, w


def reference_operator(E, ins, H, Hw, w):
    lib = _lib()
    N = lib.ref_sem2d_ngll()
    arrs = [np.ascontiguousarray(ins[n], dtype=np.float32) for n in NAMES]
    f0 = np.empty(E * N * N, np.float32)
    f1 = np.empty(E * N * N, np.float32)
    lib.ref_sem2d_reference(E, _pp(arrs), H.ctypes.data_as(C.c_void_p), Hw.ctypes.data_as(C.c_void_p),
                            w.ctypes.data_as(C.c_void_p), f0.ctypes.data_as(C.c_void_p),
                            f1.ctypes.data_as(C.c_void_p))
    return f0, f1


def test_reference_2d_fill_matches_the_python_restatement():
    E = 37
    N, ins, H, Hw, w = reference_inputs(E)
    u, arrays, H2, Hw2, w2 = reference_fill_2d(E)
    assert N == 8
    np.testing.assert_array_equal(ins["u0"], u[0])
    np.testing.assert_array_equal(ins["u1"], u[1])
    for n in ("xix", "xiz", "gamx", "gamz", "l2m", "mu", "jac"):
        np.testing.assert_array_equal(ins[n], arrays[n])
    np.testing.assert_array_equal(H, H2.astype(np.float32).reshape(-1))
    np.testing.assert_array_equal(Hw, Hw2.astype(np.float32).reshape(-1))
    np.testing.assert_array_equal(w, w2.astype(np.float32))


@pytest.mark.parametrize("E", [1, 7, 64])
def test_oracle_2d_f32_is_bit_exact_with_the_reference_host_loop(E):
    N, ins, H, Hw, w = reference_inputs(E)
    r0, r1 = reference_operator(E, ins, H, Hw, w)
    arrays = {n: ins[n] for n in NAMES[2:]}
    f = osem.sem2d_local(E, N, [ins["u0"], ins["u1"]], arrays, H, Hw, w, np.float32)
    np.testing.assert_array_equal(f[0], r0)
    np.testing.assert_array_equal(f[1], r1)


def test_oracle_2d_on_random_inputs_matches_the_reference_host_loop():
    rng = np.random.default_rng(7)
    E = 19
    N, _, H, Hw, w = reference_inputs(1)
    ins = {n: rng.uniform(0.5, 1.5, E * N * N).astype(np.float32) for n in NAMES}
    r0, r1 = reference_operator(E, ins, H, Hw, w)
    arrays = {n: ins[n] for n in NAMES[2:]}
    f = osem.sem2d_local(E, N, [ins["u0"], ins["u1"]], arrays, H, Hw, w, np.float32)
    np.testing.assert_array_equal(f[0], r0)
    np.testing.assert_array_equal(f[1], r1)
