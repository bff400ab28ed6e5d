"""2D elastic P-SV stiffness (element-local, NGLL 8, f32) on the GPU.

Against the CPU restatement of the reference's 2D host loop
(oracle.sem.sem2d_local; bench_sem_stiffness.cpp:1335-1385):
relative L2 <= 1e-5, on the reference's own deterministic fill (where the
reference program also requires max |x - ref| / (|ref| + 1e-6) < 1e-4) and on
seeded synthetic fields with the true GLL operators; ragged element counts.
"""
import numpy as np
import pytest

from oracle import sem as osem
from tensoroperations_b200 import abi
from tensoroperations_b200.sem2d import ARRAYS, reference_fill_2d, synthetic_2d

pytestmark = pytest.mark.gpu
N = 8


def _run(u, arrays, H, Hw, w, nelem):
    import torch
    du = [torch.from_numpy(x).cuda() for x in u]
    df = [torch.full_like(x, float("nan")) for x in du]
    da = {k: torch.from_numpy(arrays[k]).cuda() for k in ARRAYS}
    abi.sem2d_elastic_local(N, nelem, H, Hw, w, du, df, da)
    torch.cuda.synchronize()
    return [x.cpu().numpy() for x in df]


@pytest.mark.parametrize("nelem", [1, 3, 4, 37, 4096])
def test_reference_fill(nelem):
    u, arrays, H, Hw, w = reference_fill_2d(nelem)
    got = _run(u, arrays, H, Hw, w, nelem)
    ref = osem.sem2d_local(nelem, N, u, arrays, H.astype(np.float32), Hw.astype(np.float32),
                           w.astype(np.float32), np.float32)
    assert osem.rel_l2(got, ref) < 1e-5
    worst = max(float(np.max(np.abs(g.astype(np.float64) - r) / (np.abs(r) + 1e-6)))
                for g, r in zip(got, ref))
    assert worst < 1e-4  # the reference program's own acceptance test


@pytest.mark.parametrize("nelem", [5, 20001])
def test_synthetic_fields(nelem):
    u, arrays, H, Hw, w = synthetic_2d(nelem)
    got = _run(u, arrays, H, Hw, w, nelem)
    ref = osem.sem2d_local(nelem, N, u, arrays, H.astype(np.float32), Hw.astype(np.float32),
                           w.astype(np.float32), np.float32)
    assert osem.rel_l2(got, ref) < 1e-5
    ref64 = osem.sem2d_local(nelem, N, [x.astype(np.float64) for x in u],
                             {k: v.astype(np.float64) for k, v in arrays.items()}, H, Hw, w,
                             np.float64)
    assert osem.rel_l2(got, ref64) < 1e-5


def test_rigid_motion_is_in_the_kernel():
    """A constant displacement has zero stiffness force (GLL rows of H sum to 0)."""
    nelem = 64
    u, arrays, H, Hw, w = synthetic_2d(nelem)
    u = [np.full_like(u[0], 1.5), np.full_like(u[1], -0.25)]
    got = _run(u, arrays, H, Hw, w, nelem)
    assert max(float(np.max(np.abs(g))) for g in got) < 1e-4
