"""The C ABI library on a host without a GPU: it loads, exports every function
the public header declares, and its host-side validation and utilities behave.
No compute call is made here."""
import ctypes as C

import numpy as np
import pytest

from tensoroperations_b200 import abi


def test_library_loads_and_abi_version_matches_header():
    text = abi.HEADER.read_text()
    ver = int(text.split("#define TO_ABI_VERSION")[1].split()[0])
    assert abi.lib.to_abi_version() == ver


def test_every_declared_function_is_exported():
    names = abi.header_functions()
    assert "to_sem3d_apply" in names and len(names) >= 10
    missing = [n for n in names if not hasattr(abi.lib, n)]
    assert not missing, missing


def test_status_strings():
    assert abi.status_name(abi.TO_OK) == "TO_OK"
    assert abi.status_name(abi.TO_ERR_ALIGNMENT) == "TO_ERR_ALIGNMENT"
    assert abi.status_name(999) == "TO_ERR_UNKNOWN"


def _ops(n=5):
    _, w, H, Hw = abi.gll_operators(n)
    return H, Hw, w


def test_plan_validation_errors():
    H, Hw, w = _ops()
    with pytest.raises(abi.ToError) as e:
        abi.Sem3dPlan(np.float32, 3, 10, *_ops(3))
    assert e.value.status == abi.TO_ERR_UNSUPPORTED
    with pytest.raises(abi.ToError) as e:
        abi.Sem3dPlan(np.float32, 5, 10, H, Hw, w, nglob=0, assembled=True)
    assert e.value.status == abi.TO_ERR_INVALID_ARGUMENT
    with pytest.raises(abi.ToError) as e:
        abi.Sem3dPlan(np.float32, 5, -1, H, Hw, w)
    assert e.value.status == abi.TO_ERR_INVALID_ARGUMENT
    d = abi.Sem3dDesc()
    d.dtype, d.ngll, d.nelem = 7, 5, 1
    h = C.c_void_p()
    assert abi.lib.to_sem3d_plan_create(C.byref(d), C.byref(h)) == abi.TO_ERR_INVALID_ARGUMENT
    assert b"dtype" in abi.lib.to_last_error()
    assert abi.lib.to_sem3d_apply(None, None, 0, None) == abi.TO_ERR_INVALID_ARGUMENT


def test_apply_rejects_null_and_misaligned_pointers_before_any_launch():
    H, Hw, w = _ops()
    plan = abi.Sem3dPlan(np.float32, 5, 4, H, Hw, w)
    fl = abi.Sem3dFields()
    with pytest.raises(abi.ToError) as e:
        plan.apply(fl)
    assert e.value.status == abi.TO_ERR_INVALID_ARGUMENT
    bogus = 0x1000  # never dereferenced: alignment is checked first
    for c in range(3):
        fl.u[c] = bogus
        fl.f[c] = bogus
    for n in abi.POINT_ARRAYS:
        setattr(fl, n, bogus)
    fl.xix = bogus + 2
    with pytest.raises(abi.ToError) as e:
        plan.apply(fl)
    assert e.value.status == abi.TO_ERR_ALIGNMENT


def test_u_norm2_is_checked_before_any_launch():
    """The deferred normalisation (to_sem3d_fields.u_norm2) is for assembled
    plans and wants an 8-byte aligned double."""
    H, Hw, w = _ops()
    bogus = 0x1000  # never dereferenced
    fl = abi.Sem3dFields()
    for c in range(3):
        fl.u[c] = bogus
        fl.f[c] = bogus
    for n in abi.POINT_ARRAYS:
        setattr(fl, n, bogus)
    fl.u_norm2 = bogus
    local = abi.Sem3dPlan(np.float64, 8, 4, *_ops(8))
    with pytest.raises(abi.ToError) as e:
        local.apply(fl)
    assert e.value.status == abi.TO_ERR_UNSUPPORTED
    fl.ibool = bogus
    fl.u_norm2 = bogus + 4
    asm = abi.Sem3dPlan(np.float64, 8, 4, *_ops(8), nglob=100, assembled=True)
    with pytest.raises(abi.ToError) as e:
        asm.apply(fl)
    assert e.value.status == abi.TO_ERR_ALIGNMENT


def test_algorithmic_bytes_and_flops_of_the_bench_config():
    H, Hw, w = _ops()
    E = 64 ** 3
    nglob = 257 ** 3
    plan = abi.Sem3dPlan(np.float32, 5, E, H, Hw, w, nglob=nglob, assembled=True)
    assert plan.algorithmic_bytes() == E * 125 * (12 * 4 + 4) + nglob * 3 * 4 * 2
    assert abs(plan.algorithmic_bytes() / 2.111e9 - 1) < 1e-3
    assert plan.flops() == E * 125 * 339
    loc = abi.Sem3dPlan(np.float32, 5, E, H, Hw, w)
    assert loc.algorithmic_bytes() == E * 125 * 72


def test_structured_ibool_numbering():
    nex, ney, nez, n = 3, 2, 4, 5
    ib = abi.structured_ibool(nex, ney, nez, n)
    n1 = n - 1
    nx, ny = nex * n1 + 1, ney * n1 + 1
    for e in range(nex * ney * nez):
        ex, ey, ez = e % nex, (e // nex) % ney, e // (nex * ney)
        k, j, i = np.meshgrid(np.arange(n), np.arange(n), np.arange(n), indexing="ij")
        expect = ((ez * n1 + k) * ny + ey * n1 + j) * nx + ex * n1 + i
        np.testing.assert_array_equal(ib[e], expect)
    nglob = nx * ny * (nez * n1 + 1)
    assert ib.min() == 0 and ib.max() == nglob - 1
    assert len(np.unique(ib)) == nglob  # every node touched
    with pytest.raises(abi.ToError):
        abi.structured_ibool(0, 1, 1, 5)


def test_synth_fill_is_deterministic_and_sliceable():
    a = abi.synth_fill(100000, np.float64, 42, "uniform", 0.5, 1.5)
    b = abi.synth_fill(100000, np.float64, 42, "uniform", 0.5, 1.5)
    np.testing.assert_array_equal(a, b)
    assert 0.5 <= a.min() and a.max() < 1.5 and abs(a.mean() - 1.0) < 0.01
    c = abi.synth_fill(1000, np.float32, 42, "uniform", 0.5, 1.5)
    np.testing.assert_array_equal(c, a[:1000].astype(np.float32))
    g = abi.synth_fill(200000, np.float64, 9, "normal", 0.0, 1.0)
    assert abs(g.mean()) < 0.01 and abs(g.std() - 1.0) < 0.01
    assert not np.array_equal(abi.synth_fill(10, np.float64, 1, "uniform", 0, 1),
                              abi.synth_fill(10, np.float64, 2, "uniform", 0, 1))
