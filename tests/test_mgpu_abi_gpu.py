"""The z-slab operator's C ABI (to_sem3d_elastic_mgpu) on one GPU.

* A slab with no neighbours (a single rank, no communicator): the interior is
  the whole mesh, scattered by one launch of the line-owner kernel with
  ticketed batches; f must equal the CPU oracle's assembled result.
* A slab that is its own neighbour on both sides, through a one-rank NCCL
  communicator: the two boundary layers run as one launch, the shared planes
  go through the real NCCL group (send to self, receive into `recv`) and are
  added back, so f must equal the oracle with its first and last node planes
  doubled.  Meshes whose layers are a multiple of 4 elements take the bulk-copy
  kernel (12 elements per layer: one full and one partial batch); 30 elements
  per layer take the per-range fallback; one layer touching both planes is
  scattered once.
* Two applications in a row give the same f (tickets and f are reset).
* The interleaved node layout (u, f as [nglob][4]) through the same call:
  the planes travel as one contiguous range each; f, de-interleaved, equals
  the planar result.
"""
import numpy as np
import pytest

from oracle import sem as osem
from tensoroperations_b200 import abi
from tensoroperations_b200.sem3d import structured_problem, to_device

pytestmark = pytest.mark.gpu
N = 5
TOL = 1e-5


def _oracle(prob):
    return osem.assembled(prob.nelem, N, prob.nglob, prob.ibool, prob.u, prob.arrays, prob.H,
                          prob.Hw, prob.w, np.float32)


def _slab(torch, nex, ney, prev, nxt, f_is_zero=0):
    plane = (nex * (N - 1) + 1) * (ney * (N - 1) + 1)
    recv = [torch.empty(3 * plane, device="cuda") for _ in range(2)]
    sync = torch.zeros(abi.slab_sync_bytes(), dtype=torch.uint8, device="cuda")
    sl = abi.Slab()
    sl.prev, sl.next = prev, nxt
    sl.layer_elems = nex * ney
    sl.plane_nodes = plane
    sl.recv[0], sl.recv[1] = recv[0].data_ptr(), recv[1].data_ptr()
    sl.sync = sync.data_ptr()
    sl.f_is_zero = f_is_zero
    return sl, (recv, sync), plane


@pytest.mark.parametrize("mesh", [(4, 3, 5), (6, 5, 3), (8, 2, 2)])
def test_single_rank_without_neighbours(mesh):
    import torch
    prob = structured_problem(*mesh, ngll=N, dtype=np.float32, assembled=True, seed=31)
    u, f, arrays, ibool = to_device(prob, "cuda")
    plan = prob.plan()
    sl, keep, _ = _slab(torch, mesh[0], mesh[1], -1, -1)
    cs = torch.cuda.Stream()
    xs = torch.cuda.Stream(priority=-100)
    fl = plan.fields(u, f, arrays, ibool)
    abi.sem3d_elastic_mgpu(plan, fl, sl, None, cs.cuda_stream, xs.cuda_stream)
    torch.cuda.synchronize()
    first = [x.cpu().numpy().copy() for x in f]
    abi.sem3d_elastic_mgpu(plan, fl, sl, None, cs.cuda_stream, xs.cuda_stream)
    torch.cuda.synchronize()
    got = [x.cpu().numpy() for x in f]
    ref = _oracle(prob)
    assert osem.rel_l2(got, ref) < TOL
    assert osem.rel_l2(first, got) < 1e-6  # atomics may reorder the sums: not bitwise


@pytest.mark.parametrize("mesh", [(4, 3, 5), (6, 5, 3), (4, 4, 1)])
def test_self_exchange_through_nccl(mesh):
    import torch
    nex, ney, nez = mesh
    prob = structured_problem(nex, ney, nez, ngll=N, dtype=np.float32, assembled=True, seed=32)
    u, f, arrays, ibool = to_device(prob, "cuda")
    plan = prob.plan()
    sl, keep, plane = _slab(torch, nex, ney, 0, 0)
    cs = torch.cuda.Stream()
    xs = torch.cuda.Stream(priority=-100)
    comm = abi.nccl_comm_init(1, 0, abi.nccl_unique_id())
    try:
        fl = plan.fields(u, f, arrays, ibool)
        for _ in range(2):
            abi.sem3d_elastic_mgpu(plan, fl, sl, comm, cs.cuda_stream, xs.cuda_stream)
        torch.cuda.synchronize()
    finally:
        abi.nccl_comm_destroy(comm)
    got = [x.cpu().numpy() for x in f]
    want = [x.copy() for x in _oracle(prob)]
    for x in want:
        x[:plane] *= 2
        x[-plane:] *= 2
    assert osem.rel_l2(got, want) < TOL


def test_rejects_partial_layers_and_missing_communicator():
    import torch
    prob = structured_problem(4, 3, 2, ngll=N, dtype=np.float32, assembled=True, seed=33)
    u, f, arrays, ibool = to_device(prob, "cuda")
    plan = prob.plan()
    fl = plan.fields(u, f, arrays, ibool)
    sl, keep, _ = _slab(torch, 5, 3, -1, -1)  # 15-element layers do not divide 24 elements
    with pytest.raises(abi.ToError) as e:
        abi.sem3d_elastic_mgpu(plan, fl, sl, None, 0, 0)
    assert e.value.status == abi.TO_ERR_INVALID_ARGUMENT
    sl, keep, _ = _slab(torch, 4, 3, 0, -1)  # a neighbour but no communicator
    with pytest.raises(abi.ToError) as e:
        abi.sem3d_elastic_mgpu(plan, fl, sl, None, 0, 0)
    assert e.value.status == abi.TO_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("mesh", [(4, 3, 5), (4, 4, 1)])
@pytest.mark.parametrize("self_exchange", [False, True])
def test_interleaved_nodes(mesh, self_exchange):
    import torch
    nex, ney, nez = mesh
    prob = structured_problem(nex, ney, nez, ngll=N, dtype=np.float32, assembled=True, seed=34)
    u, f, arrays, ibool = to_device(prob, "cuda")
    u4 = torch.empty((prob.nglob, 4), dtype=torch.float32, device="cuda")
    f4 = torch.full((prob.nglob, 4), 7.0, dtype=torch.float32, device="cuda")  # zeroed by the call
    abi.nodes_interleave(u, u4, prob.nglob)
    plan = abi.Sem3dPlan(np.float32, N, prob.nelem, prob.H, prob.Hw, prob.w, nglob=prob.nglob,
                         assembled=True, interleaved=True)
    nb = -1 if not self_exchange else 0
    sl, keep, plane = _slab(torch, nex, ney, nb, nb)
    recv4 = [torch.empty(4 * plane, device="cuda") for _ in range(2)]
    sl.recv[0], sl.recv[1] = recv4[0].data_ptr(), recv4[1].data_ptr()
    cs = torch.cuda.Stream()
    xs = torch.cuda.Stream(priority=-100)
    comm = abi.nccl_comm_init(1, 0, abi.nccl_unique_id()) if self_exchange else None
    try:
        fl = plan.fields([u4, None, None], [f4, None, None], arrays, ibool)
        for _ in range(2):
            abi.sem3d_elastic_mgpu(plan, fl, sl, comm, cs.cuda_stream, xs.cuda_stream)
        torch.cuda.synchronize()
    finally:
        if comm:
            abi.nccl_comm_destroy(comm)
    back = [torch.empty(prob.nglob, device="cuda") for _ in range(3)]
    abi.nodes_deinterleave(f4, back, prob.nglob)
    torch.cuda.synchronize()
    assert float(f4[:, 3].abs().max()) == 0.0  # the unused lane stays zero
    got = [x.cpu().numpy() for x in back]
    want = [x.copy() for x in _oracle(prob)]
    if self_exchange:
        for x in want:
            x[:plane] *= 2
            x[-plane:] *= 2
    assert osem.rel_l2(got, want) < TOL


def test_node_layout_round_trip():
    import torch
    n = 1001
    x = [torch.randn(n, device="cuda") for _ in range(3)]
    x4 = torch.empty((n, 4), device="cuda")
    abi.nodes_interleave(x, x4, n)
    y = [torch.empty(n, device="cuda") for _ in range(3)]
    abi.nodes_deinterleave(x4, y, n)
    torch.cuda.synchronize()
    for a, b in zip(x, y):
        assert torch.equal(a, b)
    assert torch.equal(x4[:, 1], x[1]) and float(x4[:, 3].abs().max()) == 0.0


_AGG_CHECK = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from oracle import sem as osem
from tensoroperations_b200 import abi
from tensoroperations_b200.sem3d import structured_problem, to_device
nex, ney, nez, il = map(int, sys.argv[2:6])
prob = structured_problem(nex, ney, nez, ngll=5, dtype=np.float32, assembled=True, seed=35)
u, f, arrays, ibool = to_device(prob, "cuda")
plan = abi.Sem3dPlan(np.float32, 5, prob.nelem, prob.H, prob.Hw, prob.w, nglob=prob.nglob,
                     assembled=True, interleaved=bool(il))
if il:
    u4 = torch.empty((prob.nglob, 4), device="cuda"); abi.nodes_interleave(u, u4, prob.nglob)
    f4 = torch.empty((prob.nglob, 4), device="cuda")
    fl = plan.fields([u4, None, None], [f4, None, None], arrays, ibool)
else:
    fl = plan.fields(u, f, arrays, ibool)
sl = abi.Slab(); sl.prev = sl.next = -1; sl.layer_elems = nex * ney
sl.plane_nodes = (nex * 4 + 1) * (ney * 4 + 1)
sync = torch.zeros(abi.slab_sync_bytes(), dtype=torch.uint8, device="cuda"); sl.sync = sync.data_ptr()
abi.sem3d_elastic_mgpu(plan, fl, sl, None, 0, 0)
if il:
    abi.nodes_deinterleave(f4, f, prob.nglob)
torch.cuda.synchronize()
got = [x.cpu().numpy() for x in f]
ref = osem.assembled(prob.nelem, 5, prob.nglob, prob.ibool, prob.u, prob.arrays, prob.H, prob.Hw,
                     prob.w, np.float32)
err = osem.rel_l2(got, ref)
print("rel", err)
sys.exit(0 if err < 1e-5 else 1)
"""


@pytest.mark.parametrize("mesh", [(8, 3, 2), (5, 4, 3), (12, 2, 2)])
@pytest.mark.parametrize("il", [0, 1])
def test_warp_aggregated_scatter(mesh, il):
    """TO_SEM3D_WARP_AGG=1: x-face partners summed by a shuffle before the atomic;
    rows of 5 elements (an x-row boundary inside a batch) check that only
    equal nodes are combined."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    env = dict(os.environ, TO_SEM3D_WARP_AGG="1")
    r = subprocess.run([sys.executable, "-c", _AGG_CHECK, str(root), *map(str, mesh), str(il)],
                       capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


@pytest.mark.parametrize("il", [False, True])
def test_host_buffer_entry(il):
    """to_sem3d_elastic_mgpu_host: host u in, host f out (one array per
    component), with the device layout conversion inside the call."""
    import torch
    nex, ney, nez = 4, 3, 5
    prob = structured_problem(nex, ney, nez, ngll=N, dtype=np.float32, assembled=True, seed=36)
    _, f, arrays, ibool = to_device(prob, "cuda")
    plan = abi.Sem3dPlan(np.float32, N, prob.nelem, prob.H, prob.Hw, prob.w, nglob=prob.nglob,
                         assembled=True, interleaved=il)
    u_host = [torch.from_numpy(x).pin_memory() for x in prob.u]
    f_host = [torch.full((prob.nglob,), 5.0).pin_memory() for _ in range(3)]
    if il:
        du = [torch.empty((prob.nglob, 4), device="cuda"), None, None]
        df = [torch.empty((prob.nglob, 4), device="cuda"), None, None]
        stage = [torch.empty(prob.nglob, device="cuda") for _ in range(3)]
    else:
        du = [torch.empty(prob.nglob, device="cuda") for _ in range(3)]
        df = f
        stage = [None] * 3
    sl, keep, _ = _slab(torch, nex, ney, -1, -1)
    h = abi.HostNodes()
    for c in range(3):
        h.u[c], h.f[c] = u_host[c].data_ptr(), f_host[c].data_ptr()
        h.stage[c] = stage[c].data_ptr() if stage[c] is not None else None
    s = torch.cuda.Stream()
    abi.sem3d_elastic_mgpu_host(plan, plan.fields(du, df, arrays, ibool), sl, None, h,
                                s.cuda_stream, s.cuda_stream)
    s.synchronize()
    got = [x.numpy() for x in f_host]
    assert osem.rel_l2(got, _oracle(prob)) < TOL
