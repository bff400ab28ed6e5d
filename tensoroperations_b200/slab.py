"""Z-slab partition of the structured SEM 3D operator over ranks (one per GPU).

Element e = (ez*ney + ey)*nex + ex, so a range of element layers [z0, z1) is a
contiguous range of elements, and with the structured numbering the node
planes it touches, [z0*(N-1), z1*(N-1)], are a contiguous range of global
nodes.  Rank r owns layers [z0, z1) and all of their node planes; the first
and last planes are duplicated on the neighbours (r-1 and r+1).

One application on a rank (`SlabOperator.apply`, one call of the C ABI's
to_sem3d_elastic_mgpu on CUDA tensors):
  1. zero f; scatter the element layers next to a neighbour (compute stream,
     both layers in one launch);
  2. on a second, high-priority stream: exchange the shared planes with the
     neighbours (one NCCL group of send/recv, sent in place from f) and add
     the neighbour's partial sums in;
  3. meanwhile scatter the interior layers on the compute stream (batches
     handed out by a ticket counter) -- they touch no shared plane, so 2 and
     3 overlap;
  4. the compute stream waits for 2.
Afterwards every copy of a shared node holds the full sum: f on each rank
equals the slice of the single-mesh result for its nodes.

Each rank generates exactly its slice of the global synthetic problem
(`slab_problem`), so a multi-rank result can be checked against one
whole-mesh computation.  The reference is single-GPU; this partition is this
build's own.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import abi
from .sem3d import DEFAULT_SEED, Sem3dProblem, point_arrays


@dataclass(frozen=True)
class SlabPartition:
    nex: int
    ney: int
    nez: int  # layers of the GLOBAL mesh
    ngll: int
    world: int
    rank: int

    def __post_init__(self):
        if not (0 <= self.rank < self.world):
            raise ValueError(f"rank {self.rank} outside world {self.world}")
        if self.nez < self.world:
            raise ValueError(f"{self.nez} element layers cannot give {self.world} ranks one each")

    # ---- element layers ------------------------------------------------------
    @property
    def z0(self) -> int:
        base, extra = divmod(self.nez, self.world)
        return self.rank * base + min(self.rank, extra)

    @property
    def z1(self) -> int:
        base, extra = divmod(self.nez, self.world)
        return self.z0 + base + (1 if self.rank < extra else 0)

    @property
    def nez_local(self) -> int:
        return self.z1 - self.z0

    @property
    def layer(self) -> int:
        return self.nex * self.ney

    @property
    def nelem(self) -> int:
        return self.nez_local * self.layer

    @property
    def elem_first(self) -> int:
        return self.z0 * self.layer

    # ---- nodes -------------------------------------------------------------------
    @property
    def plane(self) -> int:
        n1 = self.ngll - 1
        return (self.nex * n1 + 1) * (self.ney * n1 + 1)

    @property
    def nglob(self) -> int:
        return self.plane * (self.nez_local * (self.ngll - 1) + 1)

    @property
    def node_first(self) -> int:
        return self.z0 * (self.ngll - 1) * self.plane

    @property
    def nglob_global(self) -> int:
        return self.plane * (self.nez * (self.ngll - 1) + 1)

    # ---- neighbours ------------------------------------------------------------
    def interfaces(self):
        """[(neighbour rank, offset of the shared plane in this rank's nodes)]"""
        out = []
        if self.rank > 0:
            out.append((self.rank - 1, 0))
        if self.rank < self.world - 1:
            out.append((self.rank + 1, self.nglob - self.plane))
        return out

    @property
    def owned_first(self) -> int:
        """First node this rank owns: a shared plane belongs to the lower rank."""
        return self.plane if self.rank > 0 else 0

    def element_ranges(self):
        """(boundary ranges, interior range) as (first, count) in local elements.

        Boundary = the layers that touch a shared plane; interior = the rest
        (one contiguous range, possibly empty)."""
        lo = self.rank > 0
        hi = self.rank < self.world - 1
        bnd = []
        if lo:
            bnd.append((0, self.layer))
        if hi and not (lo and self.nez_local == 1):
            bnd.append((self.nelem - self.layer, self.layer))
        b0 = self.layer if lo else 0
        e0 = self.nelem - self.layer if hi else self.nelem
        interior = (b0, max(0, e0 - b0))
        return bnd, interior


def layer_problem(nex: int, ney: int, za: int, zb: int, ngll: int, dtype=np.float32,
                  seed: int = DEFAULT_SEED) -> Sem3dProblem:
    """Element layers [za, zb) of structured_problem(nex, ney, nez, ...) for any
    nez >= zb (same seeds): its elements, the nodes they touch, numbered from
    the first of those nodes."""
    dt = np.dtype(dtype)
    N = ngll
    P = N ** 3
    _, w, H, Hw = abi.gll_operators(N)
    layer = nex * ney
    plane = (nex * (N - 1) + 1) * (ney * (N - 1) + 1)
    nel = (zb - za) * layer
    nglob = plane * ((zb - za) * (N - 1) + 1)
    arrays = point_arrays(nel * P, dt, seed, first=za * layer * P)
    ibool = abi.structured_ibool(nex, ney, zb - za, N).reshape(-1)
    u = [abi.synth_fill(nglob, dt, seed + c, "normal", 0.0, 1.0, first=za * (N - 1) * plane)
         for c in range(3)]
    return Sem3dProblem(N, nel, dt, H, Hw, w, arrays, u, ibool, nglob, (nex, ney, zb - za))


def slab_problem(part: SlabPartition, dtype=np.float32, seed: int = DEFAULT_SEED) -> Sem3dProblem:
    """This rank's slice of structured_problem(nex, ney, nez, ...) (same seeds)."""
    return layer_problem(part.nex, part.ney, part.z0, part.z1, part.ngll, dtype, seed)


def slab_problem_device(part: SlabPartition, dtype, device, seed: int = DEFAULT_SEED,
                        stream: int = 0):
    """slab_problem generated directly in device memory (no host arrays).

    Returns (problem, u, f, arrays, ibool): the problem carries the operators
    and sizes only (its host arrays are empty); the tensors are on `device`.
    Uniform inputs equal slab_problem's bit for bit; u (normal) may differ in
    the last bits (device log / cos)."""
    import torch
    dt = np.dtype(dtype)
    code = abi.TO_F32 if dt == np.float32 else abi.TO_F64
    tdt = torch.float32 if dt == np.float32 else torch.float64
    N = part.ngll
    P = N ** 3
    npts = part.nelem * P
    first = part.elem_first * P
    _, w, H, Hw = abi.gll_operators(N)

    def fill(t, seed_, dist, a, b, add=0.0, first_=first):
        abi.check(abi.lib.to_synth_fill_device(t.data_ptr(), code, first_, t.numel(), seed_, dist,
                                                a, b, add, stream), "to_synth_fill_device")

    arrays = {}
    for r, name in enumerate(abi.POINT_ARRAYS[:9]):
        t = torch.empty(npts, dtype=tdt, device=device)
        fill(t, seed + 3 + r, 0, 0.5, 1.5, 1.0 if name in ("xix", "etay", "gamz") else 0.0)
        arrays[name] = t
    arrays["jac"] = torch.empty(npts, dtype=tdt, device=device)
    fill(arrays["jac"], seed + 12, 0, 0.5, 2.0)
    arrays["l2m"] = torch.empty(npts, dtype=tdt, device=device)
    fill(arrays["l2m"], seed + 13, 0, 1.0, 3.0)  # lambda, then + 2 mu in place
    arrays["mu"] = torch.empty(npts, dtype=tdt, device=device)
    fill(arrays["mu"], seed + 14, 0, 0.5, 2.0)
    abi.check(abi.lib.to_axpy2_device(arrays["l2m"].data_ptr(), arrays["mu"].data_ptr(), code, npts,
                                      stream), "to_axpy2_device")
    ibool = torch.empty(npts, dtype=torch.int32, device=device)
    abi.check(abi.lib.to_mesh_structured_ibool_device(part.nex, part.ney, part.nez_local, N,
                                                      ibool.data_ptr(), stream),
              "to_mesh_structured_ibool_device")
    u = []
    for c in range(3):
        t = torch.empty(part.nglob, dtype=tdt, device=device)
        fill(t, seed + c, 1, 0.0, 1.0, first_=part.node_first)
        u.append(t)
    f = [torch.zeros(part.nglob, dtype=tdt, device=device) for _ in range(3)]
    prob = Sem3dProblem(N, part.nelem, dt, H, Hw, w, {}, [], np.empty(0, np.int32), part.nglob,
                        (part.nex, part.ney, part.nez_local))
    return prob, u, f, arrays, ibool


def exchange_planes(part: SlabPartition, sends, recvs, group=None):
    """Send sends[i] to and receive recvs[i] from neighbour i of part.interfaces().

    One batched group of point-to-point operations (NCCL: one group, so the
    chain of neighbours cannot deadlock); tensors live where the process
    group's backend expects them (CUDA for NCCL, CPU for gloo).  Returns after
    the operations are enqueued and waited on (NCCL: the current stream waits;
    gloo: the host waits)."""
    import torch.distributed as dist
    ops = []
    for (peer, _), s, r in zip(part.interfaces(), sends, recvs):
        ops.append(dist.P2POp(dist.isend, s, peer, group))
        ops.append(dist.P2POp(dist.irecv, r, peer, group))
    if not ops:
        return
    for w in dist.batch_isend_irecv(ops):
        w.wait()


class SlabOperator:
    """f = K u on this rank's slab, interface planes summed with the neighbours.

    `plan` is a Sem3dPlan over the rank's elements (assembled); `u`, `f`, the
    per-point arrays and ibool are this rank's device tensors.

    On CUDA tensors (the product path) apply() is ONE call of the C ABI,
    to_sem3d_elastic_mgpu: the boundary layers, then the interior with the
    shared planes exchanged over NCCL on a high-priority second stream.  The
    NCCL communicator is this library's own, created here from a unique id
    that rank 0 broadcasts through `group` (torch.distributed); a single rank
    needs none.  `native=False` keeps the step-by-step host orchestration
    (torch.distributed send/recv of packed planes), which the gloo tests run
    on the CPU.  Exchange buffers are allocated once here; apply() allocates
    nothing.

    power_step(): one step of u <- K u / ||K u|| (the steady-state loop of the
    large configuration): apply, sum of squares over the nodes this rank owns
    (shared planes counted once, by the lower rank), all-reduce of that one
    double across ranks -- no host round trip.  The division by the norm is
    folded into the NEXT application (to_sem3d_fields.u_norm2: the operator
    reads u * 1/sqrt(||f||^2) as it gathers), so a step makes no separate pass
    over u and f; u and f swap roles every step.  power_u() writes the current
    iterate, normalised, into the u tensors (the products of a step-by-step
    rescale, rounded once the same way)."""

    def __init__(self, part: SlabPartition, plan, fields, f, device, group=None, u=None,
                 native=None, comm=None):
        import torch
        self.part = part
        self.plan = plan
        self.fields = fields
        self.f = f
        self.group = group
        self.dtype = np.dtype(plan.dtype)
        device = torch.device(device)
        tdt = torch.float32 if self.dtype == np.float32 else torch.float64
        n = 3 * part.plane
        self.native = (device.type == "cuda") if native is None else bool(native)
        self.boundary, self.interior = part.element_ranges()
        self.u = u
        self.sumsq = torch.zeros(1, dtype=torch.float64, device=device)
        nown = part.nglob - part.owned_first
        self.sumsq_ws = torch.empty(max(1, abi.sumsq3_workspace_bytes(nown)), dtype=torch.uint8,
                                    device=device)
        self._pw_parity = 0     # the latest unnormalised iterate: 0 in u (or none yet), 1 in f
        self._pw_pending = False  # an iterate awaits the division by sqrt(sumsq)
        self._pw_fields = None
        self.comm = None  # this library's NCCL communicator (native, world > 1)
        self._own_comm = False
        if self.native:
            self.xstream = torch.cuda.Stream(device=device, priority=-100)  # highest priority
            nrecv = 4 * part.plane if getattr(plan, "interleaved", False) else n
            self.recv = [torch.empty(nrecv, dtype=tdt, device=device) if side else None
                         for side in (part.rank > 0, part.rank < part.world - 1)]
            self.sync = torch.zeros(abi.slab_sync_bytes(), dtype=torch.uint8, device=device)
            sl = abi.Slab()
            sl.prev = part.rank - 1 if part.rank > 0 else -1
            sl.next = part.rank + 1 if part.rank < part.world - 1 else -1
            sl.layer_elems = part.layer
            sl.plane_nodes = part.plane
            sl.recv[0] = self.recv[0].data_ptr() if self.recv[0] is not None else None
            sl.recv[1] = self.recv[1].data_ptr() if self.recv[1] is not None else None
            sl.sync = self.sync.data_ptr()
            self.slab = sl
            if part.world > 1:
                if comm:  # share another operator's communicator (same ranks)
                    self.comm = comm
                else:
                    self.comm = self._make_comm(device)
                    self._own_comm = True
        else:
            k = len(part.interfaces())
            self.send = [torch.empty(n, dtype=tdt, device=device) for _ in range(k)]
            self.recv = [torch.empty(n, dtype=tdt, device=device) for _ in range(k)]
            self.xstream = torch.cuda.Stream(device=device) if device.type == "cuda" else None
            self.ev_bnd = torch.cuda.Event() if device.type == "cuda" else None
            self.ev_done = torch.cuda.Event() if device.type == "cuda" else None

    def _make_comm(self, device) -> int:
        """NCCL communicator over the slab's ranks: id from rank 0, broadcast via `group`."""
        import torch
        import torch.distributed as dist
        uid = abi.nccl_unique_id() if self.part.rank == 0 else bytes(abi.NCCL_UNIQUE_ID_BYTES)
        backend = dist.get_backend(self.group)
        where = device if backend == "nccl" else "cpu"
        t = torch.tensor(list(uid), dtype=torch.uint8, device=where)
        dist.broadcast(t, src=dist.get_global_rank(self.group, 0) if self.group else 0,
                       group=self.group)
        with torch.cuda.device(device):
            return abi.nccl_comm_init(self.part.world, self.part.rank, bytes(t.cpu().tolist()))

    def close(self):
        """Release the NCCL communicator this operator created (every rank calls
        it, after the operators sharing it are done; idempotent)."""
        if self.comm and self._own_comm:
            abi.nccl_comm_destroy(self.comm)
        self.comm = None

    def kernel_launches(self) -> int:
        """Launches of this library's kernels per apply (fills excluded)."""
        k = len(self.part.interfaces())
        if self.native:
            return (1 if self.boundary else 0) + (1 if self.interior[1] else 0) + k
        return len(self.boundary) + (1 if self.interior[1] else 0) + 2 * k

    def apply(self, stream, events=None, fields=None, f=None):
        """One application on `stream`; `events` = (start, end) CUDA events are
        recorded on it around this rank's operator (f's zeroing excluded).
        `fields` / `f` replace the operator's own (the power iteration's
        swapped buffers)."""
        fields = self.fields if fields is None else fields
        f_out = self.f if f is None else f
        if self.native:
            import torch
            with torch.cuda.stream(stream):
                for x in f_out:
                    x.zero_()
            self.slab.f_is_zero = 1
            if events is not None:
                events[0].record(stream)
            abi.sem3d_elastic_mgpu(self.plan, fields, self.slab, self.comm,
                                   stream.cuda_stream, self.xstream.cuda_stream)
            if events is not None:
                events[1].record(stream)
            return
        import torch
        s = stream.cuda_stream
        for x in f_out:
            x.zero_()
        if events is not None:
            events[0].record(stream)
        for first, count in self.boundary:
            self.plan.apply_elements(fields, first, count, s)
        faces = self.part.interfaces()
        if faces:
            self.ev_bnd.record(stream)
            self.xstream.wait_event(self.ev_bnd)
            cs = self.xstream.cuda_stream
            with torch.cuda.stream(self.xstream):
                for (_, off), buf in zip(faces, self.send):
                    abi.halo_pack(self.dtype, f_out, off, self.part.plane, buf, cs)
                exchange_planes(self.part, self.send, self.recv, self.group)
                for (_, off), buf in zip(faces, self.recv):
                    abi.halo_accumulate(self.dtype, f_out, off, self.part.plane, buf, cs)
            self.ev_done.record(self.xstream)
        first, count = self.interior
        if count:
            self.plan.apply_elements(fields, first, count, s)
        if faces:
            stream.wait_event(self.ev_done)
        if events is not None:
            events[1].record(stream)

    def power_step(self, stream, events=None):
        """f = K u, then ||f||^2 over the ranks into self.sumsq; the next step
        reads f as its u divided by sqrt(||f||^2) (the buffers swap)."""
        import torch
        import torch.distributed as dist
        if self.u is None:
            raise ValueError("power_step needs the operator's u tensors (SlabOperator(..., u=u))")
        if getattr(self.plan, "interleaved", False):
            raise ValueError("power_step: one array per component (node_layout 0)")
        if self._pw_fields is None:
            scaled = self.fields.copy()  # u -> f, u read divided by the norm
            scaled.u_norm2 = self.sumsq.data_ptr()
            swapped = scaled.copy()      # f -> u
            for c in range(3):
                swapped.u[c], swapped.f[c] = self.fields.f[c], self.fields.u[c]
            self._pw_fields = (scaled, swapped)
        if self._pw_parity == 0:
            fields = self._pw_fields[0] if self._pw_pending else self.fields
            out = self.f
        else:
            fields, out = self._pw_fields[1], self.u
        self.apply(stream, events, fields, out)
        s = stream.cuda_stream
        first = self.part.owned_first
        abi.sumsq3(self.dtype, out, first, self.part.nglob - first, self.sumsq, self.sumsq_ws, s)
        if self.part.world > 1:
            if self.comm:
                abi.nccl_allreduce_sum_f64(self.sumsq, 1, self.comm, s)
            else:
                with torch.cuda.stream(stream):
                    dist.all_reduce(self.sumsq, group=self.group)
        self._pw_parity ^= 1
        self._pw_pending = True

    def power_u(self, stream):
        """Write the current iterate K u / ||K u|| into the u tensors (one
        to_scale3 on `stream`); later steps start from it."""
        if not self._pw_pending:
            return
        src = self.f if self._pw_parity == 1 else self.u
        abi.scale3(self.dtype, self.u, src, self.part.nglob, self.sumsq, stream.cuda_stream)
        self._pw_parity = 0
        self._pw_pending = False
