"""The CUDA kernels against golden vectors made by the reference's own code (GPU).

tests/golden/*.npz hold the reference benchmarks' own inputs and host-reference
outputs (tests/golden/make_golden.py).  The sm_100a element-local 3D kernel
(NGLL 5, f32) and the 2D P-SV kernel (NGLL 8, f32) must match them to the
f32 tolerance (relative L2 <= 1e-5), and to the reference programs' own
acceptance tests (3D: max |x - ref| / max |ref| < 1e-4; 2D: max |x - ref| /
(|ref| + 1e-6) < 1e-2).
"""
import numpy as np
import pytest

from oracle import sem as osem
from tensoroperations_b200 import abi
from tensoroperations_b200.sem2d import ARRAYS as ARRAYS2
from tensoroperations_b200.sem3d import Sem3dProblem, to_device

from test_golden_cpu import NAMES3, load2, load3

pytestmark = pytest.mark.gpu


def test_golden_3d_kernel():
    import torch
    g = load3()
    E, N = int(g["E"]), int(g["ngll"])
    prob = Sem3dProblem(ngll=N, nelem=E, dtype=np.dtype(np.float32), H=g["H"].astype(np.float64),
                        Hw=g["Hw"].astype(np.float64), w=g["w"].astype(np.float64),
                        arrays={n: g[n] for n in NAMES3[3:]}, u=[g["u0"], g["u1"], g["u2"]])
    u, f, arrays, ibool = to_device(prob)
    plan = prob.plan()
    plan.apply(plan.fields(u, f, arrays, ibool), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = [x.cpu().numpy() for x in f]
    ref = [g["f0"], g["f1"], g["f2"]]
    assert osem.rel_l2(got, ref) <= 1e-5
    worst = max(float(np.max(np.abs(a.astype(np.float64) - b))) for a, b in zip(got, ref))
    scale = max(float(np.max(np.abs(b))) for b in ref)
    assert worst / scale < 1e-4


def test_golden_2d_kernel():
    import torch
    g = load2()
    E, N = int(g["E"]), int(g["ngll"])
    du = [torch.from_numpy(g[n]).cuda() for n in ("u0", "u1")]
    df = [torch.full_like(x, float("nan")) for x in du]
    da = {k: torch.from_numpy(g[k]).cuda() for k in ARRAYS2}
    abi.sem2d_elastic_local(N, E, g["H"].astype(np.float64), g["Hw"].astype(np.float64),
                            g["w"].astype(np.float64), du, df, da)
    torch.cuda.synchronize()
    got = [x.cpu().numpy() for x in df]
    ref = [g["f0"], g["f1"]]
    assert osem.rel_l2(got, ref) <= 1e-5
    worst = max(float(np.max(np.abs(a.astype(np.float64) - b) / (np.abs(b) + 1e-6)))
                for a, b in zip(got, ref))
    assert worst < 1e-2
