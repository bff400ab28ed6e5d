"""The CPU oracle checked against the mathematics and against itself (no GPU).

Known answers used to trust the restatement before it judges the CUDA path:
  * GLL operators: weights integrate polynomials of degree <= 2N-3 exactly, the
    derivative matrix differentiates degree <= N-1 polynomials exactly;
  * rigid translation is in the kernel of the stiffness operator (H rows sum
    to zero), so K u = 0 for a constant u;
  * with the standard hprimewgll Hw(q,i) = H(q,i) w(q) the assembled operator
    is symmetric: v.K u == u.K v;
  * the assembled operator equals the scatter of the element-local one;
  * f32 and f64 restatements agree within f32 rounding;
  * the OpenMP colour-parallel port equals the serial oracle.
The bit-exact pin against the reference's own compiled host loop lives in
tests/test_reference_pin.py.
"""
import numpy as np
import pytest

from oracle import sem as osem
from tensoroperations_b200 import abi
from tensoroperations_b200.sem3d import structured_problem


@pytest.mark.parametrize("n", [2, 3, 5, 8])
def test_gll_quadrature_and_derivative_exact(n):
    x, w, H, Hw = abi.gll_operators(n)
    assert np.all(np.diff(x) > 0) and x[0] == -1.0 and x[-1] == 1.0
    np.testing.assert_allclose(x, -x[::-1], atol=1e-14)
    for deg in range(0, 2 * n - 2):  # GLL exact up to degree 2N-3
        exact = (1 - (-1) ** (deg + 1)) / (deg + 1)
        assert abs(np.dot(w, x ** deg) - exact) < 1e-13
    for deg in range(0, n):
        np.testing.assert_allclose(H @ (x ** deg), deg * x ** max(deg - 1, 0) if deg else 0 * x,
                                   atol=1e-11)
    np.testing.assert_allclose(Hw, H * w[:, None], atol=0)


def _small(assembled=True, dtype=np.float64, mesh=(3, 2, 4)):
    return structured_problem(*mesh, ngll=5, dtype=dtype, assembled=assembled, seed=1234)


def test_f32_restatement_matches_f64():
    p64 = _small(assembled=False, dtype=np.float64)
    p32 = _small(assembled=False, dtype=np.float32)
    f64 = osem.local(p64.nelem, 5, p64.u, p64.arrays, p64.H, p64.Hw, p64.w, np.float64)
    f32 = osem.local(p32.nelem, 5, p32.u, p32.arrays, p32.H, p32.Hw, p32.w, np.float32)
    assert osem.rel_l2(f32, f64) < 2e-6


def test_assembled_is_scatter_of_local():
    p = _small(assembled=True)
    fa = osem.assembled(p.nelem, 5, p.nglob, p.ibool, p.u, p.arrays, p.H, p.Hw, p.w, np.float64)
    uloc = [u[p.ibool] for u in p.u]
    floc = osem.local(p.nelem, 5, uloc, p.arrays, p.H, p.Hw, p.w, np.float64)
    ref = [np.zeros(p.nglob) for _ in range(3)]
    for c in range(3):
        np.add.at(ref[c], p.ibool, floc[c])
    assert osem.rel_l2(fa, ref) < 1e-14


def test_rigid_translation_is_in_the_kernel():
    p = _small(assembled=True)
    u = [np.full(p.nglob, v) for v in (1.0, -2.0, 0.5)]
    f = osem.assembled(p.nelem, 5, p.nglob, p.ibool, u, p.arrays, p.H, p.Hw, p.w, np.float64)
    scale = osem.assembled(p.nelem, 5, p.nglob, p.ibool, p.u, p.arrays, p.H, p.Hw, p.w,
                           np.float64)
    assert max(np.abs(x).max() for x in f) < 1e-11 * max(np.abs(x).max() for x in scale)


def test_assembled_operator_is_symmetric():
    p = _small(assembled=True)
    rng = np.random.default_rng(7)
    v = [rng.standard_normal(p.nglob) for _ in range(3)]
    Ku = osem.assembled(p.nelem, 5, p.nglob, p.ibool, p.u, p.arrays, p.H, p.Hw, p.w, np.float64)
    Kv = osem.assembled(p.nelem, 5, p.nglob, p.ibool, v, p.arrays, p.H, p.Hw, p.w, np.float64)
    vKu = sum(np.dot(a, b) for a, b in zip(v, Ku))
    uKv = sum(np.dot(a, b) for a, b in zip(p.u, Kv))
    assert abs(vKu - uKv) < 1e-11 * abs(vKu)


def test_linearity():
    p = _small(assembled=True)
    rng = np.random.default_rng(3)
    v = [rng.standard_normal(p.nglob) for _ in range(3)]
    args = (p.nelem, 5, p.nglob, p.ibool)
    Ku = osem.assembled(*args, p.u, p.arrays, p.H, p.Hw, p.w, np.float64)
    Kv = osem.assembled(*args, v, p.arrays, p.H, p.Hw, p.w, np.float64)
    Kw = osem.assembled(*args, [2.0 * a - 3.0 * b for a, b in zip(p.u, v)], p.arrays, p.H, p.Hw,
                        p.w, np.float64)
    assert osem.rel_l2(Kw, [2.0 * a - 3.0 * b for a, b in zip(Ku, Kv)]) < 1e-13


def test_structured_colouring_is_valid_and_uses_8_colours():
    p = _small(assembled=True, mesh=(4, 3, 2))
    n, start, order, col = osem.colouring(p.nelem, 5, p.nglob, p.ibool)
    assert n == 8
    ib = p.ibool.reshape(p.nelem, -1)
    for c in range(n):
        nodes = ib[order[start[c]:start[c + 1]]].ravel()
        assert len(np.unique(nodes)) == len(nodes)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_openmp_port_matches_serial_oracle(dtype):
    p = _small(assembled=True, dtype=dtype, mesh=(4, 3, 5))
    ref = osem.assembled(p.nelem, 5, p.nglob, p.ibool, p.u, p.arrays, p.H, p.Hw, p.w, dtype)
    cpu = osem.AssembledCPU(p.nelem, 5, p.nglob, p.ibool, p.arrays, p.H, p.Hw, p.w, dtype)
    out = cpu(p.u, [np.empty(p.nglob, dtype=dtype) for _ in range(3)])
    assert osem.rel_l2(out, ref) < (1e-5 if dtype == np.float32 else 1e-13)
