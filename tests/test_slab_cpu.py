"""Z-slab partition and interface exchange on the host (no GPU).

* The ranks' element ranges tile the global mesh; node ranges overlap only in
  the shared planes; each rank's problem is exactly its slice of the whole
  problem (same seeds).
* With world_size 2 and 3 gloo ranks (processes on this host) the slab path's
  host logic runs end to end: each rank computes its elements' contribution
  with the CPU oracle (boundary layers and interior separately, the order the
  GPU operator uses), packs its shared planes, exchanges them with
  `exchange_planes`, adds the neighbour's partial sums, and the result must
  equal that rank's slice of the oracle on the whole mesh.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import sem as osem
from tensoroperations_b200.sem3d import structured_problem
from tensoroperations_b200.slab import SlabPartition, exchange_planes, slab_problem

MESH = (3, 2, 5)  # nex, ney, nez (global)
N = 5
SEED = 4242


@pytest.mark.parametrize("world", [1, 2, 3, 4, 5])
def test_partition_tiles_the_mesh(world):
    nex, ney, nez = MESH
    parts = [SlabPartition(nex, ney, nez, N, world, r) for r in range(world)]
    assert parts[0].z0 == 0 and parts[-1].z1 == nez
    for a, b in zip(parts, parts[1:]):
        assert a.z1 == b.z0
        # the last plane of a is the first plane of b
        assert a.node_first + a.nglob - a.plane == b.node_first
    assert sum(p.nelem for p in parts) == nex * ney * nez
    for p in parts:
        bnd, (f0, c0) = p.element_ranges()
        covered = sorted([(f, c) for f, c in bnd] + ([(f0, c0)] if c0 else []))
        pos = 0
        for f, c in covered:
            assert f == pos
            pos += c
        assert pos == p.nelem
        assert len(p.interfaces()) == (p.rank > 0) + (p.rank < world - 1)


def test_rejects_more_ranks_than_layers():
    with pytest.raises(ValueError):
        SlabPartition(2, 2, 3, N, 4, 0)


@pytest.mark.parametrize("world", [2, 3])
def test_slab_problem_is_a_slice_of_the_whole(world):
    nex, ney, nez = MESH
    whole = structured_problem(nex, ney, nez, ngll=N, dtype=np.float32, assembled=True, seed=SEED)
    P = N ** 3
    for r in range(world):
        p = SlabPartition(nex, ney, nez, N, world, r)
        s = slab_problem(p, np.float32, SEED)
        e0 = p.elem_first * P
        for name, a in s.arrays.items():
            np.testing.assert_array_equal(a, whole.arrays[name][e0:e0 + p.nelem * P])
        for c in range(3):
            np.testing.assert_array_equal(s.u[c], whole.u[c][p.node_first:p.node_first + p.nglob])
        # local numbering + node offset = global numbering
        np.testing.assert_array_equal(s.ibool.astype(np.int64) + p.node_first,
                                      whole.ibool[e0:e0 + p.nelem * P])


def _local_contribution(prob, first, count):
    P = N ** 3
    sl = slice(first * P, (first + count) * P)
    arrays = {k: np.ascontiguousarray(v[sl]) for k, v in prob.arrays.items()}
    return osem.assembled(count, N, prob.nglob, np.ascontiguousarray(prob.ibool[sl]), prob.u,
                          arrays, prob.H, prob.Hw, prob.w, prob.dtype)


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nex, ney, nez = MESH
        part = SlabPartition(nex, ney, nez, N, world, rank)
        prob = slab_problem(part, np.float64, SEED)
        f = [np.zeros(part.nglob) for _ in range(3)]
        bnd, interior = part.element_ranges()
        for first, count in bnd + ([interior] if interior[1] else []):
            g = _local_contribution(prob, first, count)
            for c in range(3):
                f[c] += g[c]
        faces = part.interfaces()
        sends = [torch.from_numpy(np.concatenate([f[c][off:off + part.plane] for c in range(3)]))
                 for _, off in faces]
        recvs = [torch.empty(3 * part.plane, dtype=torch.float64) for _ in faces]
        exchange_planes(part, sends, recvs)
        for (_, off), r in zip(faces, recvs):
            rv = r.numpy()
            for c in range(3):
                f[c][off:off + part.plane] += rv[c * part.plane:(c + 1) * part.plane]
        np.save(os.path.join(out_dir, f"f{rank}.npy"), np.stack(f))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ranks_reproduce_the_whole_mesh(world, tmp_path):
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    nex, ney, nez = MESH
    whole = structured_problem(nex, ney, nez, ngll=N, dtype=np.float64, assembled=True, seed=SEED)
    ref = osem.assembled(whole.nelem, N, whole.nglob, whole.ibool, whole.u, whole.arrays, whole.H,
                         whole.Hw, whole.w, np.float64)
    for r in range(world):
        p = SlabPartition(nex, ney, nez, N, world, r)
        got = np.load(tmp_path / f"f{r}.npy")
        want = np.stack([x[p.node_first:p.node_first + p.nglob] for x in ref])
        assert osem.rel_l2(list(got), list(want)) < 1e-12, r


def _power_worker(rank, world, port, out_dir, steps):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nex, ney, nez = MESH
        part = SlabPartition(nex, ney, nez, N, world, rank)
        prob = slab_problem(part, np.float64, SEED)
        u = [x.copy() for x in prob.u]
        faces = part.interfaces()
        for _ in range(steps):
            prob.u = u
            f = _local_contribution(prob, 0, part.nelem)
            sends = [torch.from_numpy(np.concatenate([f[c][off:off + part.plane] for c in range(3)]))
                     for _, off in faces]
            recvs = [torch.empty(3 * part.plane, dtype=torch.float64) for _ in faces]
            exchange_planes(part, sends, recvs)
            for (_, off), r in zip(faces, recvs):
                rv = r.numpy()
                for c in range(3):
                    f[c][off:off + part.plane] += rv[c * part.plane:(c + 1) * part.plane]
            o = part.owned_first
            ss = torch.tensor([sum(float(np.dot(x[o:], x[o:])) for x in f)], dtype=torch.float64)
            dist.all_reduce(ss)
            u = [x / np.sqrt(float(ss[0])) for x in f]
        np.save(os.path.join(out_dir, f"u{rank}.npy"), np.stack(u))
    finally:
        dist.destroy_process_group()


def whole_mesh_power(steps, seed=SEED, dtype=np.float64):
    nex, ney, nez = MESH
    whole = structured_problem(nex, ney, nez, ngll=N, dtype=dtype, assembled=True, seed=seed)
    u = whole.u
    for _ in range(steps):
        f = osem.assembled(whole.nelem, N, whole.nglob, whole.ibool, u, whole.arrays, whole.H,
                           whole.Hw, whole.w, dtype)
        nrm = np.sqrt(sum(float(np.dot(x, x)) for x in f))
        u = [x / nrm for x in f]
    return u


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_power_iteration_counts_shared_planes_once(world, tmp_path):
    steps = 3
    mp.start_processes(_power_worker, args=(world, _free_port(), str(tmp_path), steps),
                       nprocs=world, join=True, start_method="spawn")
    ref = whole_mesh_power(steps)
    nex, ney, nez = MESH
    for r in range(world):
        p = SlabPartition(nex, ney, nez, N, world, r)
        got = np.load(tmp_path / f"u{r}.npy")
        want = [x[p.node_first:p.node_first + p.nglob] for x in ref]
        assert osem.rel_l2(list(got), want) < 1e-12, r
