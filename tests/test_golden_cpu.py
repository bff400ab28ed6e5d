"""The CPU oracle against golden vectors made by the reference's own code (no GPU).

tests/golden/*.npz were written by tests/golden/make_golden.py from the
reference benchmarks compiled from their own sources (oracle/_ref):
  sem3d_ref_fill_E6.npz  bench_sem3d_levelgraph.cpp fill() inputs and its host
                         reference() output (NGLL 5, f32, element-local);
  sem2d_ref_fill_E5.npz  bench_sem_stiffness.cpp fill_field()/fill_operators()
                         inputs and its host_reference() output (NGLL 8, f32).
The oracle's f32 restatements follow those loops operation for operation, so
they must reproduce the golden outputs BIT FOR BIT; the Python restatements of
the fills must reproduce the golden inputs (the 3D fill calls sinf, so to
within 2e-7 relative; the 2D fill is integer arithmetic, exactly).  These tests
need no reference tree and no oracle/_ref build.
"""
from pathlib import Path

import numpy as np

from oracle import sem as osem
from tensoroperations_b200.sem2d import reference_fill_2d
from tensoroperations_b200.sem3d import reference_fill_problem

GOLD = Path(__file__).resolve().parent / "golden"
NAMES3 = ["u0", "u1", "u2", "xix", "xiy", "xiz", "etax", "etay", "etaz", "gamx", "gamy", "gamz",
          "l2m", "mu", "jac"]
NAMES2 = ["u0", "u1", "xix", "xiz", "gamx", "gamz", "l2m", "mu", "jac"]


def load3():
    return dict(np.load(GOLD / "sem3d_ref_fill_E6.npz"))


def load2():
    return dict(np.load(GOLD / "sem2d_ref_fill_E5.npz"))


def test_golden_3d_oracle_bit_exact():
    g = load3()
    E, N = int(g["E"]), int(g["ngll"])
    arrays = {n: g[n] for n in NAMES3[3:]}
    got = osem.local(E, N, [g["u0"], g["u1"], g["u2"]], arrays, g["H"], g["Hw"], g["w"], np.float32)
    for c in range(3):
        np.testing.assert_array_equal(got[c], g[f"f{c}"])


def test_golden_3d_fill_restatement():
    g = load3()
    p = reference_fill_problem(int(g["E"]))
    for n in NAMES3:
        mine = p.u[int(n[1])] if n in ("u0", "u1", "u2") else p.arrays[n]
        np.testing.assert_allclose(mine, g[n], rtol=2e-7, atol=0)
    np.testing.assert_allclose(p.H.astype(np.float32), g["H"], rtol=2e-7, atol=1e-8)


def test_golden_3d_oracle_f64_close():
    g = load3()
    E, N = int(g["E"]), int(g["ngll"])
    arrays = {n: g[n].astype(np.float64) for n in NAMES3[3:]}
    got = osem.local(E, N, [g[n].astype(np.float64) for n in ("u0", "u1", "u2")], arrays,
                     g["H"].astype(np.float64), g["Hw"].astype(np.float64),
                     g["w"].astype(np.float64), np.float64)
    assert osem.rel_l2([g["f0"], g["f1"], g["f2"]], got) < 1e-6


def test_golden_2d_oracle_bit_exact():
    g = load2()
    E, N = int(g["E"]), int(g["ngll"])
    arrays = {n: g[n] for n in NAMES2[2:]}
    got = osem.sem2d_local(E, N, [g["u0"], g["u1"]], arrays, g["H"], g["Hw"], g["w"], np.float32)
    np.testing.assert_array_equal(got[0], g["f0"])
    np.testing.assert_array_equal(got[1], g["f1"])


def test_golden_2d_fill_restatement():
    g = load2()
    u, arrays, H, Hw, w = reference_fill_2d(int(g["E"]))
    np.testing.assert_array_equal(u[0], g["u0"])
    np.testing.assert_array_equal(u[1], g["u1"])
    for n in NAMES2[2:]:
        np.testing.assert_array_equal(arrays[n], g[n])
    np.testing.assert_array_equal(H.astype(np.float32).reshape(-1), g["H"])
    np.testing.assert_array_equal(Hw.astype(np.float32).reshape(-1), g["Hw"])
    np.testing.assert_array_equal(w.astype(np.float32), g["w"])


def test_planted_error_is_caught():
    """A one-ulp change in one golden output must fail the bit-exact comparison."""
    g = load3()
    E, N = int(g["E"]), int(g["ngll"])
    arrays = {n: g[n] for n in NAMES3[3:]}
    got = osem.local(E, N, [g["u0"], g["u1"], g["u2"]], arrays, g["H"], g["Hw"], g["w"], np.float32)
    bad = got[1].copy()
    bad[17] = np.nextafter(bad[17], np.float32(np.inf))
    assert not np.array_equal(bad, g["f1"])
