"""Z-slab path on the GPU: element-range apply, interface-plane kernels, and
the whole multi-rank operator against the CPU oracle on the whole mesh.

Tolerance: relative L2 <= 1e-5 (f32) against the f32 oracle.
"""
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import sem as osem
from tensoroperations_b200 import abi
from tensoroperations_b200.sem3d import structured_problem, to_device
from tensoroperations_b200.slab import SlabPartition, slab_problem

pytestmark = pytest.mark.gpu
N = 5
TOL = 1e-5
ROOT = Path(__file__).resolve().parent.parent


def _torch():
    import torch
    return torch


@pytest.mark.parametrize("assembled", [True, False])
def test_element_ranges_sum_to_the_whole_apply(assembled):
    torch = _torch()
    prob = structured_problem(5, 4, 3, ngll=N, dtype=np.float32, assembled=assembled, seed=31)
    u, f, arrays, ibool = to_device(prob, "cuda")
    plan = prob.plan()
    plan.apply(plan.fields(u, f, arrays, ibool))
    whole = [x.clone() for x in f]
    for x in f:
        x.zero_()
    fl = plan.fields(u, f, arrays, ibool)
    # ragged ranges, starts not a multiple of 4 elements (16-byte fallback path too)
    for first, count in ((0, 3), (3, 17), (20, 1), (21, prob.nelem - 21)):
        plan.apply_elements(fl, first, count)
    torch.cuda.synchronize()
    got = [x.cpu().numpy() for x in f]
    assert osem.rel_l2(got, [x.cpu().numpy() for x in whole]) < TOL
    with pytest.raises(abi.ToError):
        plan.apply_elements(fl, prob.nelem - 1, 2)


def test_halo_pack_and_accumulate():
    torch = _torch()
    n, off, nglob = 1000, 777, 3000
    f = [torch.randn(nglob, device="cuda", dtype=torch.float64) for _ in range(3)]
    buf = torch.empty(3 * n, device="cuda", dtype=torch.float64)
    abi.halo_pack(np.float64, f, off, n, buf)
    torch.cuda.synchronize()
    want = torch.cat([x[off:off + n] for x in f])
    assert torch.equal(buf, want)
    before = [x.clone() for x in f]
    add = torch.randn(3 * n, device="cuda", dtype=torch.float64)
    abi.halo_accumulate(np.float64, f, off, n, add)
    torch.cuda.synchronize()
    for c in range(3):
        exp = before[c].clone()
        exp[off:off + n] += add[c * n:(c + 1) * n]
        assert torch.equal(f[c], exp)


@pytest.mark.parametrize("world", [2, 3])
def test_emulated_ranks_on_one_gpu(world):
    """Every rank's slab on one GPU, the exchange done by device copies."""
    torch = _torch()
    nex, ney, nez = 4, 3, 5
    ranks = []
    for r in range(world):
        part = SlabPartition(nex, ney, nez, N, world, r)
        prob = slab_problem(part, np.float32, 77)
        u, f, arrays, ibool = to_device(prob, "cuda")
        plan = prob.plan()
        fl = plan.fields(u, f, arrays, ibool)
        bnd, interior = part.element_ranges()
        for first, count in bnd + ([interior] if interior[1] else []):
            plan.apply_elements(fl, first, count)
        sends = {}
        for peer, off in part.interfaces():
            buf = torch.empty(3 * part.plane, device="cuda")
            abi.halo_pack(np.float32, f, off, part.plane, buf)
            sends[peer] = buf
        ranks.append((part, f, sends))
    for part, f, _ in ranks:
        for peer, off in part.interfaces():
            abi.halo_accumulate(np.float32, f, off, part.plane, ranks[peer][2][part.rank])
    torch.cuda.synchronize()
    whole = structured_problem(nex, ney, nez, ngll=N, dtype=np.float32, assembled=True, seed=77)
    ref = osem.assembled(whole.nelem, N, whole.nglob, whole.ibool, whole.u, whole.arrays, whole.H,
                         whole.Hw, whole.w, np.float32)
    for part, f, _ in ranks:
        got = [x.cpu().numpy() for x in f]
        want = [x[part.node_first:part.node_first + part.nglob] for x in ref]
        assert osem.rel_l2(got, want) < TOL


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("layer", [(6, 5), (4, 3)])
def test_nccl_ranks_reproduce_the_whole_mesh(tmp_path, layer):
    """30-element layers take the per-range fallback; 12-element layers the
    bulk-copy kernel with ticketed batches (one full, one partial batch)."""
    torch = _torch()
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    (nex, ney), nez, seed = layer, 4 * world, 99
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(ROOT / "tests" / "slab_mgpu_check.py"),
           str(tmp_path), str(nex), str(ney), str(nez), str(seed)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    whole = structured_problem(nex, ney, nez, ngll=N, dtype=np.float32, assembled=True, seed=seed)
    ref = osem.assembled(whole.nelem, N, whole.nglob, whole.ibool, whole.u, whole.arrays, whole.H,
                         whole.Hw, whole.w, np.float32)
    for rk in range(world):
        p = SlabPartition(nex, ney, nez, N, world, rk)
        got = list(np.load(tmp_path / f"f{rk}.npy"))
        want = [x[p.node_first:p.node_first + p.nglob] for x in ref]
        assert osem.rel_l2(got, want) < TOL, rk


def test_nccl_power_iteration_ngll8_f64(tmp_path):
    torch = _torch()
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    nex, ney, nez, seed, steps = 3, 2, 2 * world, 17, 3
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(ROOT / "tests" / "slab_mgpu_check.py"),
           str(tmp_path), str(nex), str(ney), str(nez), str(seed), "power", "8"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    whole = structured_problem(nex, ney, nez, ngll=8, dtype=np.float64, assembled=True, seed=seed)
    u = whole.u
    for _ in range(steps):
        f = osem.assembled(whole.nelem, 8, whole.nglob, whole.ibool, u, whole.arrays, whole.H,
                           whole.Hw, whole.w, np.float64)
        nrm = np.sqrt(sum(float(np.dot(x, x)) for x in f))
        u = [x / nrm for x in f]
    for rk in range(world):
        p = SlabPartition(nex, ney, nez, 8, world, rk)
        got = list(np.load(tmp_path / f"u{rk}.npy"))
        want = [x[p.node_first:p.node_first + p.nglob] for x in u]
        assert osem.rel_l2(got, want) < 1e-12, rk
