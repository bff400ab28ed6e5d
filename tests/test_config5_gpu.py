"""The large fp64 configuration's pieces on the GPU (small meshes).

* NGLL 8 operator, f64 (relative L2 <= 1e-12) and f32 (<= 1e-5), assembled
  and element-local, against the same-precision CPU oracle;
* the sum of squares (deterministic: same bits on every call) and the
  device-side rescale;
* u <- K u / ||K u|| through SlabOperator.power_step, against the same
  iteration with the oracle on the whole mesh.
"""
import math

import numpy as np
import pytest

from oracle import sem as osem
from tensoroperations_b200 import abi
from tensoroperations_b200.sem3d import structured_problem, to_device
from tensoroperations_b200.slab import SlabOperator, SlabPartition, slab_problem

pytestmark = pytest.mark.gpu
TOL = {np.float64: 1e-12, np.float32: 1e-5}


def _torch():
    import torch
    return torch


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("assembled", [True, False])
def test_ngll8_operator(dtype, assembled):
    torch = _torch()
    prob = structured_problem(3, 2, 3, ngll=8, dtype=dtype, assembled=assembled, seed=8)
    u, f, arrays, ibool = to_device(prob, "cuda")
    plan = prob.plan()
    plan.apply(plan.fields(u, f, arrays, ibool))
    torch.cuda.synchronize()
    got = [x.cpu().numpy() for x in f]
    if assembled:
        ref = osem.assembled(prob.nelem, 8, prob.nglob, prob.ibool, prob.u, prob.arrays, prob.H,
                             prob.Hw, prob.w, dtype)
    else:
        ref = osem.local(prob.nelem, 8, prob.u, prob.arrays, prob.H, prob.Hw, prob.w, dtype)
    assert osem.rel_l2(got, ref) < TOL[dtype]


@pytest.mark.parametrize("variant", ["10", "12", "2"])
def test_every_ngll8_kernel_matches_oracle(variant):
    """TO_SEM3D_VARIANT forces the NGLL-8 kernel (10: half-column, the fp64
    default; 12: whole-column, the fp32 default; 2: register streaming); each is
    checked in a fresh process for both precisions, assembled and element-local,
    with a partial last batch."""
    import os
    import subprocess
    import sys
    code = (
        "import numpy as np, torch\n"
        "from oracle import sem as osem\n"
        "from tensoroperations_b200 import abi\n"
        "from tensoroperations_b200.sem3d import structured_problem, to_device\n"
        "for dt, tol in ((np.float64, 1e-12), (np.float32, 1e-5)):\n"
        "    for asm, mesh in ((True, (3, 2, 3)), (False, (5, 1, 1))):\n"
        "        p = structured_problem(*mesh, ngll=8, dtype=dt, assembled=asm, seed=5)\n"
        "        u, f, a, ib = to_device(p, 'cuda')\n"
        "        pl = p.plan(); pl.apply(pl.fields(u, f, a, ib)); torch.cuda.synchronize()\n"
        "        got = [x.cpu().numpy() for x in f]\n"
        "        ref = (osem.assembled(p.nelem, 8, p.nglob, p.ibool, p.u, p.arrays, p.H, p.Hw, p.w, dt)\n"
        "               if asm else osem.local(p.nelem, 8, p.u, p.arrays, p.H, p.Hw, p.w, dt))\n"
        "        err = osem.rel_l2(got, ref)\n"
        "        assert err <= tol, (dt, asm, err)\n"
        "abi.check(abi.lib.to_device_status(0), 'status')\n"
        "print('ok')\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, TO_SEM3D_VARIANT=variant, PYTHONPATH=root)
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("n,first", [(1, 0), (1000, 7), (200_003, 11), (131072, 0)])
def test_sumsq3(dtype, n, first):
    torch = _torch()
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    x = [torch.randn(first + n + 5, dtype=tdt, device="cuda") for _ in range(3)]
    res = torch.zeros(1, dtype=torch.float64, device="cuda")
    ws = torch.empty(abi.sumsq3_workspace_bytes(n), dtype=torch.uint8, device="cuda")
    abi.sumsq3(dtype, x, first, n, res, ws)
    r1 = float(res.item())
    abi.sumsq3(dtype, x, first, n, res, ws)
    assert float(res.item()) == r1  # deterministic
    ref = math.fsum(float(v) ** 2 for c in range(3) for v in x[c][first:first + n].double().cpu().numpy())
    assert abs(r1 - ref) <= 1e-13 * ref
    with pytest.raises(abi.ToError):
        abi.sumsq3(dtype, x, first, n, res, ws[:max(0, ws.numel() - 8)] if ws.numel() > 8 else ws[:0])


def test_scale3():
    torch = _torch()
    x = [torch.randn(5000, dtype=torch.float64, device="cuda") for _ in range(3)]
    y = [torch.empty_like(v) for v in x]
    ss = torch.tensor([4.0], dtype=torch.float64, device="cuda")
    abi.scale3(np.float64, y, x, 5000, ss)
    torch.cuda.synchronize()
    for a, b in zip(x, y):
        assert torch.equal(b, a / 2.0)


def _oracle_power(prob, steps):
    u = prob.u
    for _ in range(steps):
        f = osem.assembled(prob.nelem, prob.ngll, prob.nglob, prob.ibool, u, prob.arrays, prob.H,
                           prob.Hw, prob.w, prob.dtype)
        nrm = math.sqrt(sum(float(np.dot(v.astype(np.float64), v.astype(np.float64))) for v in f))
        u = [(v / nrm).astype(prob.dtype) for v in f]
    return u


@pytest.mark.parametrize("ngll", [5, 8])
def test_power_iteration_single_gpu(ngll):
    torch = _torch()
    part = SlabPartition(3, 2, 3, ngll, 1, 0)
    prob = slab_problem(part, np.float64, 55)
    u, f, arrays, ibool = to_device(prob, "cuda")
    plan = prob.plan()
    op = SlabOperator(part, plan, plan.fields(u, f, arrays, ibool), f, "cuda", u=u)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(4):
            op.power_step(stream)
        op.power_u(stream)
    torch.cuda.synchronize()
    ref = _oracle_power(structured_problem(3, 2, 3, ngll=ngll, dtype=np.float64, assembled=True,
                                           seed=55), 4)
    assert osem.rel_l2([x.cpu().numpy() for x in u], ref) < 1e-12


@pytest.mark.parametrize("ngll,dtype", [(8, np.float64), (5, np.float64), (5, np.float32)])
def test_deferred_normalisation_is_bitwise_the_rescale(ngll, dtype):
    """power_step folds 1/||f|| into the next application's gather: the
    iterate after 3 steps equals apply + sum of squares + to_scale3 every step
    (the same products, rounded once) up to the order of the scatter-adds,
    which the GPU does not fix: relative L2 1e-14 (f64) / 1e-6 (f32)."""
    torch = _torch()
    part = SlabPartition(3, 2, 3, ngll, 1, 0)
    prob = slab_problem(part, dtype, 57)
    stream = torch.cuda.Stream()
    u1, f1, arrays, ibool = to_device(prob, "cuda")
    plan = prob.plan()
    lazy = SlabOperator(part, plan, plan.fields(u1, f1, arrays, ibool), f1, "cuda", u=u1)
    u2, f2, _, _ = to_device(prob, "cuda")
    eager = SlabOperator(part, plan, plan.fields(u2, f2, arrays, ibool), f2, "cuda", u=u2)
    s = stream.cuda_stream
    with torch.cuda.stream(stream):
        for _ in range(3):
            lazy.power_step(stream)
        lazy.power_u(stream)
        for _ in range(3):
            eager.apply(stream)
            abi.sumsq3(plan.dtype, f2, 0, part.nglob, eager.sumsq, eager.sumsq_ws, s)
            abi.scale3(plan.dtype, u2, f2, part.nglob, eager.sumsq, s)
    torch.cuda.synchronize()
    tol = 1e-14 if dtype == np.float64 else 1e-6
    assert osem.rel_l2([x.cpu().numpy() for x in u1], [x.cpu().numpy() for x in u2]) < tol


@pytest.mark.parametrize("dtype,ngll,world,rank", [(np.float64, 8, 3, 1), (np.float32, 5, 2, 0)])
def test_device_generated_slab_matches_host(dtype, ngll, world, rank):
    """slab_problem_device == slab_problem: uniform arrays and ibool bit for bit,
    u (normal: device log / cos) to 1e-14."""
    torch = _torch()
    from tensoroperations_b200.slab import slab_problem_device
    part = SlabPartition(3, 2, 4, ngll, world, rank)
    host = slab_problem(part, dtype, 91)
    prob, u, f, arrays, ibool = slab_problem_device(part, dtype, "cuda", 91)
    torch.cuda.synchronize()
    for name, a in host.arrays.items():
        assert np.array_equal(arrays[name].cpu().numpy(), a), name
    assert np.array_equal(ibool.cpu().numpy(), host.ibool)
    for c in range(3):
        got = u[c].cpu().numpy()
        assert np.max(np.abs(got - host.u[c])) <= 1e-6 * (np.max(np.abs(host.u[c])) if dtype == np.float32 else 1e-8)
    assert prob.nglob == host.nglob and prob.nelem == host.nelem
