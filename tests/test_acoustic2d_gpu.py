"""2D acoustic stiffness, assembled (the first configuration) on the GPU.

Against the CPU oracle's restatement of the same operator (the reference has
no acoustic kernel, so parity is unpinned by execution): relative L2 <= 1e-12
(f64, the configuration's 128 x 128 quads) and <= 1e-5 (f32); accumulate
semantics; a constant potential has zero force; the assembled operator is
symmetric (v.Ku == u.Kv) since Hw = H^T w.
"""
import numpy as np
import pytest

from oracle import sem as osem
from tensoroperations_b200 import abi
from tensoroperations_b200.sem2d import acoustic_problem

pytestmark = pytest.mark.gpu


def _dev(u, arrays, ibool, dtype):
    import torch
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    du = torch.from_numpy(np.ascontiguousarray(u, dtype=dtype)).cuda()
    da = {k: torch.from_numpy(np.ascontiguousarray(v, dtype=dtype)).cuda() for k, v in arrays.items()}
    return du, da, torch.from_numpy(ibool).cuda(), tdt


def _apply(prob, dtype, u=None, accumulate=False, f=None):
    import torch
    uh, arrays, ibool, nglob, H, Hw, w = prob
    du, da, dib, tdt = _dev(uh if u is None else u, arrays, ibool, dtype)
    if f is None:
        f = torch.full((nglob,), float("nan") if not accumulate else 0.0, dtype=tdt, device="cuda")
    abi.sem2d_acoustic_apply(5, len(ibool) // 25, nglob, H, Hw, w, du, f, dib, da, dtype,
                             accumulate=accumulate)
    torch.cuda.synchronize()
    return f


@pytest.mark.parametrize("dtype,tol,mesh", [(np.float64, 1e-12, (128, 128)), (np.float32, 1e-5, (17, 9))])
def test_matches_oracle(dtype, tol, mesh):
    prob = acoustic_problem(*mesh, dtype=dtype)
    uh, arrays, ibool, nglob, H, Hw, w = prob
    got = _apply(prob, dtype).cpu().numpy()
    ref = osem.sem2d_acoustic(len(ibool) // 25, 5, nglob, ibool, uh, arrays, H, Hw, w, dtype)
    assert osem.rel_l2([got], [ref]) < tol


def test_accumulate_adds():
    prob = acoustic_problem(8, 8)
    f1 = _apply(prob, np.float64)
    f2 = _apply(prob, np.float64, accumulate=True, f=f1.clone())
    assert np.allclose(f2.cpu().numpy(), 2 * f1.cpu().numpy(), rtol=1e-13, atol=1e-13)


def test_constant_potential_and_symmetry():
    prob = acoustic_problem(16, 12)
    uh, arrays, ibool, nglob, H, Hw, w = prob
    f0 = _apply(prob, np.float64, u=np.full(nglob, 3.0))
    assert float(np.max(np.abs(f0.cpu().numpy()))) < 1e-11
    rng = np.random.default_rng(5)
    v = rng.standard_normal(nglob)
    Ku = _apply(prob, np.float64).cpu().numpy()
    Kv = _apply(prob, np.float64, u=v).cpu().numpy()
    assert abs(v @ Ku - uh @ Kv) <= 1e-10 * abs(v @ Ku)
