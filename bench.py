#!/usr/bin/env python
"""Benchmark of the B200 SEM stiffness operator (the hot path).

Workload (the configuration the headline metric and the
north star are quoted on): 3D SEM isotropic-elastic stiffness, NGLL=5, f32,
structured 64x64x64 hexes per GPU (262,144 elements, 257^3 global nodes on one
GPU), assembled through ibool (gather u, scatter-add f).  One step = one
application f = K u: zero f, then the fused kernel.  On the device u and f are
interleaved per node ([nglob][4] f32: one 16-byte gather and one 16-byte
scatter-add per point; --layout components keeps one array per component);
the end-to-end leg moves one array per component over PCIe and converts on
the device inside its timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

For N > 1 (torchrun, one rank per GPU) the mesh is 64x64x(64N) hexes split in
z-slabs, one per rank (weak scaling); each rank scatters the element layers
next to its neighbours first, then exchanges and sums the shared node planes
over NCCL on a second stream while its interior layers compute
(tensoroperations_b200/slab.py).

Prints ONE JSON line on rank 0.  `value` is whole-job elements/s (Melem/s),
timed with CUDA events on the launching stream over exactly K steps between
barriers, max over ranks.  `roofline.achieved` = algorithmic bytes per launch
(12 per-point f32 arrays + ibool per point, u read and f written once per
global node) / the kernel's average CUDA-event duration.  `e2e` times the same
operator through the C ABI's host-buffer call (to_sem3d_elastic_mgpu_host) with
pinned HOST u and f: H2D of u and D2H of f of every step inside the timed
region, mesh resident; two buffer sets on two streams overlap consecutive
steps' copies.  The CPU baseline is the OpenMP C++
restatement of the reference's host loop (the reference itself needs Kokkos,
which is not installed), timed on this host on a bounded number of full
applications.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("SEM stiffness Melem/s and HBM GB/s (% of ~8 TB/s) at 1/2/4/8 B200 vs host CPU")
MESH_PER_GPU = (64, 64, 64)
NGLL = 5
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) per launch of the kernel at 64^3: variant 5 from one
# ncu capture of a single 64^3 launch (profiles/sem3d_elastic_v5_64cube_mix.md),
# variant 0 from the 32^3 capture scaled by elements
# (profiles/sem3d_elastic_v3_32cube_full.md); None where not captured.
NCU_TRAFFIC_PER_LAUNCH = {"0": 276.76e6 * 8, "5": 2225873664.0 + 214804736.0}
NCU_TRAFFIC_SOURCE = {"0": "ncu dram__bytes_read+write of the 32^3 case x8",
                      "5": "ncu dram__bytes_read+write of one 64^3 launch"}
DEFAULT_VARIANT = "5"
# The z-slab call's kernel (ticketed batches) per node layout, and its DRAM bytes per
# 64^3 launch from one ncu capture (profiles/sem3d_elastic_v5_64cube_mix.md,
# profiles/sem3d_elastic_v5_il_64cube.md).
KERNEL_BY_LAYOUT = {"components": "sem3d_elastic_v5_kernel<8,3,true,false,6>",
                    "interleaved": "sem3d_elastic_v5_kernel<8,3,true,true,6>"}
NCU_TRAFFIC_BY_LAYOUT = {
    "components": (2225873664.0 + 214804736.0,
                   "ncu dram__bytes_read+write of one 64^3 launch (grid-stride build of the "
                   "same kernel, identical data movement)"),
    "interleaved": (2248828672.0 + 242721792.0, "ncu dram__bytes_read+write of one 64^3 launch")}
KERNEL_NAMES = {"0": "sem3d_elastic_v3_kernel<5,8,2,true>",
                "1": "sem3d_elastic_tma_kernel<float,5,8,2,true>",
                "2": "sem3d_elastic_kernel<float,5,32,true>",
                "3": "sem3d_elastic_v3_kernel<5,4,4,true>",
                "4": "sem3d_elastic_v3_kernel<5,16,1,true>",
                "5": "sem3d_elastic_v5_kernel<8,3,true>",
                "6": "sem3d_elastic_v5_kernel<4,5,true>"}


def measured_peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in the background.

    Start it before the warm-up (nvidia-smi needs a moment to start); mark the
    timed region with begin() / end(); summary() keeps the samples taken inside
    it, or -- when the region was shorter than the sampling interval -- the
    samples of the warm-up and the region together, and says which."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []  # (host time, line)
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", self.gpu_id], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def wait_first(self, timeout: float = 3.0):
        """Block until nvidia-smi has produced a sample (or timeout)."""
        t_end = time.time() + timeout
        while self.proc is not None and not self.lines and time.time() < t_end:
            time.sleep(0.02)

    def begin(self):
        self.t0 = time.time()

    def end(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        inside = [ln for t, ln in self.lines
                  if self.t0 is None or (self.t0 <= t <= (self.t1 or t))]
        window = "timed region"
        if not inside:
            inside = [ln for _, ln in self.lines]
            window = "warm-up and timed region (timed region shorter than the 200 ms interval)"
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in inside:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm), "window": window}


def gpu_id_for(dev) -> str:
    import torch
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev)


def cpu_baseline(prob, seconds: float = 12.0, max_reps: int = 50):
    """OpenMP restatement of the reference host loop on all host threads."""
    from oracle import sem as osem
    osem.set_num_threads(osem.host_cores())  # torchrun exports OMP_NUM_THREADS=1
    cpu = osem.AssembledCPU(prob.nelem, prob.ngll, prob.nglob, prob.ibool, prob.arrays,
                            prob.H, prob.Hw, prob.w, prob.dtype)
    f = [np.empty(prob.nglob, dtype=prob.dtype) for _ in range(3)]
    cpu(prob.u, f)  # warm-up
    times = []
    t_end = time.perf_counter() + seconds
    while len(times) < max_reps and (time.perf_counter() < t_end or len(times) < 2):
        t0 = time.perf_counter()
        cpu(prob.u, f)
        times.append(time.perf_counter() - t0)
    best = min(times)
    return {"value": prob.nelem / best / 1e6, "unit": "Melem/s", "cores": osem.num_threads(),
            "kind": "port",
            "sample": (f"{len(times)} full applications of the {prob.mesh[0]}x{prob.mesh[1]}x"
                       f"{prob.mesh[2]} mesh ({prob.nelem} elements), best time "
                       f"{best * 1e3:.1f} ms; OpenMP colour-parallel C++ restatement of "
                       "bench_sem3d_levelgraph.cpp:600-663 (Kokkos absent)")}


def make_problem(rank: int, world: int, strong: bool = False):
    """This rank's z-slab, generated as the exact slice of the whole synthetic
    problem: weak scaling cuts the nex x ney x (world*nez) mesh (nez layers per
    rank), strong scaling the fixed nex x ney x nez mesh."""
    from tensoroperations_b200.slab import SlabPartition, slab_problem
    nex, ney, nez = MESH_PER_GPU
    part = SlabPartition(nex, ney, nez if strong else nez * world, NGLL, world, rank)
    return part, slab_problem(part, np.float32)


def check_against_one_gpu(part, u, f, arrays, dev, stream):
    """Relative L2 error of this rank's assembled f against the same operator
    applied on ONE GPU (to_sem3d_apply, no partition, no exchange) to the
    rank's element layers plus the neighbouring layer on each side -- the
    layers that contribute to the rank's nodes.  The middle of the extended
    inputs is the rank's own device data; the extra layers come from the same
    seeded generator."""
    import torch
    from tensoroperations_b200 import abi
    from tensoroperations_b200.slab import layer_problem
    N, P, L, plane = part.ngll, part.ngll ** 3, part.layer, part.plane
    lo = 1 if part.rank > 0 else 0
    hi = 1 if part.rank < part.world - 1 else 0
    za, zb = part.z0 - lo, part.z1 + hi
    nel = (zb - za) * L
    nglob = plane * ((zb - za) * (N - 1) + 1)
    below = layer_problem(part.nex, part.ney, za, za + 1, N, np.float32) if lo else None
    above = layer_problem(part.nex, part.ney, zb - 1, zb, N, np.float32) if hi else None
    ext = {}
    for name in abi.POINT_ARRAYS:
        t = torch.empty(nel * P, dtype=torch.float32, device=dev)
        t[lo * L * P:lo * L * P + part.nelem * P].copy_(arrays[name])
        if lo:
            t[:L * P].copy_(torch.from_numpy(below.arrays[name]))
        if hi:
            t[-L * P:].copy_(torch.from_numpy(above.arrays[name]))
        ext[name] = t
    off = lo * (N - 1) * plane  # the rank's first node inside the extended numbering
    ue = []
    for c in range(3):
        t = torch.empty(nglob, dtype=torch.float32, device=dev)
        t[off:off + part.nglob].copy_(u[c])
        if lo:
            t[:off].copy_(torch.from_numpy(below.u[c][:off]))
        if hi:
            t[off + part.nglob:].copy_(torch.from_numpy(above.u[c][plane:]))
        ue.append(t)
    ib = torch.from_numpy(abi.structured_ibool(part.nex, part.ney, zb - za, N).reshape(-1)).to(dev)
    fe = [torch.empty(nglob, dtype=torch.float32, device=dev) for _ in range(3)]
    _, w, H, Hw = abi.gll_operators(N)
    plan = abi.Sem3dPlan(np.float32, N, nel, H, Hw, w, nglob=nglob, assembled=True)
    plan.apply(plan.fields(ue, fe, ext, ib), stream=stream.cuda_stream)
    torch.cuda.synchronize()
    num = sum(float(torch.sum((f[c].double() - fe[c][off:off + part.nglob].double()) ** 2))
              for c in range(3))
    den = sum(float(torch.sum(fe[c][off:off + part.nglob].double() ** 2)) for c in range(3))
    return (num / max(den, 1e-300)) ** 0.5


def run_reference(args):
    """The reference arm: the CPU port of the reference's host loop on all host threads.

    Each step is one application on a z-slab sample of the configured mesh, sized so
    the whole K + W run stays within about 90 s of CPU time (Melem/s is per element,
    so a thinner slab of the same mesh measures the same rate)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import sem as osem
    from tensoroperations_b200.sem3d import structured_problem
    osem.set_num_threads(osem.host_cores())  # torchrun exports OMP_NUM_THREADS=1
    nex, ney, nez = MESH_PER_GPU
    probe = structured_problem(nex, ney, max(1, nez // 16), ngll=NGLL, dtype=np.float32,
                               assembled=True)
    cpu = osem.AssembledCPU(probe.nelem, probe.ngll, probe.nglob, probe.ibool, probe.arrays,
                            probe.H, probe.Hw, probe.w, probe.dtype)
    f = [np.empty(probe.nglob, dtype=np.float32) for _ in range(3)]
    cpu(probe.u, f)
    t0 = time.perf_counter()
    cpu(probe.u, f)
    t_elem = (time.perf_counter() - t0) / probe.nelem
    budget = 90.0
    nsteps = max(args.steps, 1) + max(args.warmup, 0)
    nez_s = int(max(1, min(nez, budget / (nsteps * t_elem * nex * ney))))
    prob = structured_problem(nex, ney, nez_s, ngll=NGLL, dtype=np.float32, assembled=True)
    cpu = osem.AssembledCPU(prob.nelem, prob.ngll, prob.nglob, prob.ibool, prob.arrays,
                            prob.H, prob.Hw, prob.w, prob.dtype)
    f = [np.empty(prob.nglob, dtype=prob.dtype) for _ in range(3)]
    for _ in range(args.warmup):
        cpu(prob.u, f)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu(prob.u, f)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    v = prob.nelem / dt / 1e6
    cfg = {"workload": ("3D SEM isotropic elastic stiffness, NGLL=5, f32, structured "
                        f"{nex}x{ney}x{nez * args.gpus} hexes, assembled through ibool"),
           "nelem_per_gpu": nex * ney * nez, "ngll": NGLL, "mode": "assembled",
           "parallelism": "host CPU (rank 0 only)"}
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "Melem/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": v, "unit": "Melem/s", "cores": osem.num_threads(),
                         "kind": "port",
                         "sample": (f"each step one application on a {nex}x{ney}x{nez_s}-hex "
                                    f"z-slab sample ({prob.nelem} elements) of the configured "
                                    "mesh; the reference's own Kokkos OpenMP build is "
                                    "unavailable (Kokkos, GoogleTest and KokkosKernels are "
                                    "fetched at configure time and absent), so this is the "
                                    "OpenMP C++ restatement of its host loop "
                                    "(bench_sem3d_levelgraph.cpp:600-663)")},
        "e2e": {"value": v, "unit": "Melem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_gemm(args):
    """The general contraction's tensor-core GEMM (to_gemm_tf32x3), printed with
    --workload gemm.  A step = one call, C = A B^T with K-major fp32 operands
    already split into TF32 hi/lo (the frontend's pack step is not timed here);
    M = N = K = --gemm-size.  Useful flops 2 M N K; the tensor cores run three
    TF32 products."""
    import torch
    from tensoroperations_b200 import abi
    n = args.gemm_size
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(5)
    A = torch.randn((n, n), generator=g, device=dev)
    B = torch.randn((n, n), generator=g, device=dev)

    def split(x):
        b = x.view(torch.int32)
        hb = (b + 0x1000) & ~0x1FFF
        hi = hb.view(torch.float32)
        return hi.contiguous(), (x - hi).contiguous()
    Ahi, Alo = split(A)
    Bhi, Blo = split(B)
    C = torch.empty((n, n), device=dev)
    stream = torch.cuda.Stream(device=dev)
    s = stream.cuda_stream
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            abi.gemm_tf32x3(n, n, n, Ahi, Alo, Bhi, Blo, C, stream=s)
    torch.cuda.synchronize()
    steps = args.steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    with ClockSampler(gpu_id_for(dev)) as clocks:
        ev[0].record(stream)
        for _ in range(steps):
            abi.gemm_tf32x3(n, n, n, Ahi, Alo, Bhi, Blo, C, stream=s)
        ev[1].record(stream)
        torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / steps
    abi.check(abi.lib.to_device_status(1), "device status")
    useful = 2.0 * n ** 3
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = A.double() @ B.double().T
    rel = float((C.double() - ref).norm() / ref.norm())
    for _ in range(2):
        A @ B.T
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        A @ B.T
    e1.record()
    torch.cuda.synchronize()
    torch_ms = e0.elapsed_time(e1) / 5
    mp_path = ROOT / "MEASURED_PEAKS.json"
    mp = json.loads(mp_path.read_text()) if mp_path.exists() else {}
    peak = float(mp.get("bf16_tflops", 1590.0)) / 2
    achieved = 3 * useful / (ms * 1e-3) / 1e12
    line = {"metric": "general contraction GEMM on tcgen05 (fp32 via 3xTF32), useful TFLOP/s",
            "value": useful / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": 1, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32 (3xTF32 on tcgen05)",
            "data": "synthetic N(0,1), seeded",
            "config": {"workload": f"C = A B^T, M = N = K = {n}, K-major split operands",
                       "l2": f"operands 4 x {4 * n * n / 2**20:.0f} MB"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": None,
                         "peak_source": "measured bf16_tflops / 2 (TF32 rate is half the bf16 rate)"},
            "library_fp32": {"torch_fp32_ms": torch_ms, "speedup": torch_ms / ms},
            "rel_l2_vs_float64": rel, "gpu_launches": steps, "clocks": clocks.summary()}
    print(json.dumps(line))


def run_chain(args):
    """Config 4: the permuted multilevel contraction chain (E = 64) on the tensor cores.

    Not the headline line (that is the SEM operator); printed when asked for
    with --workload chain.  One step = one to_chain_f32 call: the TF32 split /
    regroup pre-pass, the tcgen05 GEMM with the fused second contraction, R
    zeroed first.  Inputs 4 x 64 MB, above L2."""
    import torch
    from tensoroperations_b200 import abi
    E = args.chain_extent
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(4)
    A = torch.randn((E,) * 4, generator=g, device=dev)
    B = torch.randn((E,) * 4, generator=g, device=dev)
    Cm = torch.randn((E, E), generator=g, device=dev)
    R = torch.empty((E, E), device=dev)
    ws = torch.empty(abi.lib.to_chain_workspace_bytes(E), dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    s = stream.cuda_stream
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            abi.chain_f32(E, A, B, Cm, R, ws, stream=s)
    torch.cuda.synchronize()
    steps = args.steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    with ClockSampler(gpu_id_for(dev)) as clocks:
        ev[0].record(stream)
        for _ in range(steps):
            abi.chain_f32(E, A, B, Cm, R, ws, stream=s)
        ev[1].record(stream)
        torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / steps
    useful = abi.lib.to_chain_flops(E)
    tensor_flops = 3 * 2.0 * E ** 6
    # library comparison: torch fp32 (TF32 off) on the same permuted problem
    torch.backends.cuda.matmul.allow_tf32 = False
    def torch_chain():
        Am = A.permute(0, 2, 1, 3).reshape(E * E, E * E)
        Bm = B.permute(2, 0, 1, 3).reshape(E * E, E * E)
        T = (Am @ Bm).reshape(E, E, E, E).permute(0, 2, 1, 3)
        return torch.einsum("abcd,cb->ad", T, Cm)
    for _ in range(2):
        torch_chain()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        Rt = torch_chain()
    e1.record()
    torch.cuda.synchronize()
    torch_ms = e0.elapsed_time(e1) / 5
    rel = float((R - Rt).norm() / Rt.norm())
    # CPU baseline: numpy float32 on the host's BLAS threads, one chain
    An, Bn, Cn = (x.cpu().numpy() for x in (A, B, Cm))
    t0 = time.perf_counter()
    Tn = (An.transpose(0, 2, 1, 3).reshape(E * E, E * E) @
          Bn.transpose(2, 0, 1, 3).reshape(E * E, E * E)).reshape(E, E, E, E)
    np.einsum("acbd,cb->ad", Tn, Cn, optimize=True)
    cpu_s = time.perf_counter() - t0
    mp_path = ROOT / "MEASURED_PEAKS.json"
    mp = json.loads(mp_path.read_text()) if mp_path.exists() else {}
    peak = float(mp.get("bf16_tflops", 1590.0)) / 2
    achieved = tensor_flops / (ms * 1e-3) / 1e12
    line = {"metric": "permuted multilevel contraction chain (config 4), useful TFLOP/s",
            "value": useful / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": 1, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32 (3xTF32 on tcgen05)",
            "data": "synthetic N(0,1), seeded",
            "config": {"workload": f"T=sum_ef A[a,e,c,f]B[f,b,e,d]; R=sum_bc T C[c,b]; all extents {E}",
                       "extent": E, "l2": "inputs 4 x 64 MB + workspace 256 MB, above L2"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": None,
                         "peak_source": "measured bf16_tflops / 2 (TF32 rate is half the bf16 rate)",
                         "tensor_flops_per_step": tensor_flops},
            "library_fp32": {"torch_fp32_ms": torch_ms, "speedup": torch_ms / ms,
                             "rel_l2_vs_torch_fp32": rel},
            "cpu_baseline": {"value": useful / cpu_s / 1e12, "unit": "TFLOP/s",
                             "cores": os.cpu_count(), "kind": "port",
                             "sample": "one chain in numpy float32 (host BLAS, all threads)"},
            "gpu_launches": steps * 3, "clocks": clocks.summary()}
    print(json.dumps(line), flush=True)
    return 0


def run_batched_gemm(args):
    """Config 2: C[b] = A B[b], A 5x5 shared, B[b] 5x25, batch 65536, f32 and f64.

    Printed with --workload batched-gemm.  HBM-bound (read B, write C once:
    65.5 MB in f32); 100 back-to-back launches are captured in one CUDA graph
    and the graph is replayed, so launch latency does not dominate a 10 us
    kernel."""
    import torch
    from tensoroperations_b200 import abi
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    batch, M, N, reps = 65536, 5, 25, 100
    rng = np.random.default_rng(2)
    A = rng.standard_normal((M, M))
    results = {}
    peak, peak_src = measured_peak_hbm()
    for name, tdt in (("f32", torch.float32), ("f64", torch.float64)):
        g = torch.Generator(device=dev).manual_seed(3)
        # four input / output sets rotate (>= 262 MB, twice L2) so no launch reads
        # what an earlier one left in L2
        nset = 4
        Bs = [torch.randn((batch, M, N), generator=g, dtype=tdt, device=dev) for _ in range(nset)]
        Cs = [torch.empty((batch, M, N), dtype=tdt, device=dev) for _ in range(nset)]
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            for k in range(4):
                abi.batched_small_gemm(A, Bs[k % nset], Cs[k % nset], stream=stream.cuda_stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for k in range(reps):
                abi.batched_small_gemm(A, Bs[k % nset], Cs[k % nset],
                                       stream=torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (args.steps * reps)
        nbytes = 2 * batch * M * N * Bs[0].element_size()
        results[name] = {"us_per_launch": us, "gb_s": nbytes / (us * 1e-6) / 1e9,
                         "frac": nbytes / (us * 1e-6) / 1e9 / peak, "bytes": nbytes}
        del graph
    # host baseline: numpy einsum over the batch, f32
    Bn = rng.standard_normal((batch, M, N)).astype(np.float32)
    t0 = time.perf_counter()
    for _ in range(5):
        np.matmul(A.astype(np.float32)[None], Bn)
    cpu_us = (time.perf_counter() - t0) / 5 * 1e6
    r = results["f32"]
    line = {"metric": "batched small GEMM (config 2) GB/s", "value": r["gb_s"], "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": 3, "ms_per_step": r["us_per_launch"] * 1e-3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic N(0,1), seeded",
            "config": {"workload": "C[b] = A B[b], A 5x5 shared, B[b] 5x25, batch 65536",
                       "graph": f"{reps} launches per CUDA graph, 4 input/output sets rotate (262 MB f32)"},
            "roofline": {"bound": "hbm", "achieved": r["gb_s"], "peak": peak, "unit": "GB/s",
                         "frac": r["frac"], "traffic": None, "peak_source": peak_src},
            "f64": results["f64"],
            "cpu_baseline": {"value": r["bytes"] / (cpu_us * 1e-6) / 1e9, "unit": "GB/s",
                             "cores": os.cpu_count(), "kind": "port",
                             "sample": "numpy matmul over the batch, f32, 5 runs"},
            "gpu_launches": args.steps * reps}
    print(json.dumps(line), flush=True)
    return 0


def run_large(args):
    """Config 5: 128^3 hexes, NGLL 8, f64, z-slabs over the ranks (strong
    scaling), 10 power-iteration steps u <- K u / ||K u|| timed.

    Printed with --workload large.  Inputs are generated on the device (142 GB
    on one GPU).  A step = one application (boundary layers, NCCL exchange of
    the shared planes overlapped with the interior; u read divided by the
    previous step's norm), the owner-counted sum of squares, one NCCL
    all-reduce; the normalised iterate is written out once after the last
    step, inside the timed region."""
    import torch
    import torch.distributed as dist
    from tensoroperations_b200.slab import SlabOperator, SlabPartition, slab_problem_device
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    n = args.large_mesh
    part = SlabPartition(n, n, n, 8, world, rank)
    prob, u, f, arrays, ibool = slab_problem_device(part, np.float64, dev)
    plan = prob.plan()
    op = SlabOperator(part, plan, plan.fields(u, f, arrays, ibool), f, dev, u=u)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 1)):
            op.power_step(stream)
    torch.cuda.synchronize()
    steps = args.steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(gpu_id_for(dev)) as clocks:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                op.power_step(stream)
            op.power_u(stream)  # the normalised iterate written out once, inside the timing
            e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    nelem = n ** 3
    alg = plan.algorithmic_bytes()  # this rank's share
    ta = torch.tensor([alg], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ta)
    alg_total = float(ta[0])
    peak, peak_src = measured_peak_hbm()
    if rank == 0:
        line = {"metric": "SEM stiffness Melem/s (config 5: 128^3, NGLL 8, f64, power iteration)",
                "value": nelem / (ms * 1e-3) / 1e6, "unit": "Melem/s", "n_gpus": world,
                "steps": steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
                "data": "synthetic, generated on the device (same seeded streams as the host fill)",
                "config": {"workload": f"{n}^3 hexes, NGLL 8, f64, assembled; 10-step u <- Ku/|Ku|",
                           "parallelism": f"z-slabs x{world}", "nelem": nelem,
                           "nglob": part.plane * (n * 7 + 1)},
                "roofline": {"bound": "hbm", "achieved": alg_total / world / (ms * 1e-3) / 1e9,
                             "peak": peak, "unit": "GB/s",
                             "frac": alg_total / world / (ms * 1e-3) / 1e9 / peak, "traffic": None,
                             "peak_source": peak_src, "algorithmic_bytes_per_step_all_ranks": alg_total},
                "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)
    op.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_sem2d(args):
    """The reference's 2D benchmark operator: elastic P-SV, NGLL 8, f32,
    element-local, E = 2,621,440 elements (7.4 GB moved per application).

    Printed with --workload sem2d.  Inputs generated on the device (seeded
    streams, the 3D configuration's distributions).  Algorithmic bytes per
    element: 9 input arrays + 2 outputs, 64 points each, 4 B."""
    import torch
    from tensoroperations_b200 import abi
    from tensoroperations_b200.sem2d import ARRAYS
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    E = args.sem2d_elements
    npts = E * 64
    _, w, H, Hw = abi.gll_operators(8)

    def gen(seed, dist, a, b, add=0.0):
        t = torch.empty(npts, dtype=torch.float32, device=dev)
        abi.check(abi.lib.to_synth_fill_device(t.data_ptr(), abi.TO_F32, 0, npts, seed, dist, a, b,
                                                add, 0), "to_synth_fill_device")
        return t
    seed = 0x2D5EED
    arrays = {"xix": gen(seed + 3, 0, 0.5, 1.5, 1.0), "xiz": gen(seed + 4, 0, 0.5, 1.5),
              "gamx": gen(seed + 5, 0, 0.5, 1.5), "gamz": gen(seed + 6, 0, 0.5, 1.5, 1.0),
              "jac": gen(seed + 12, 0, 0.5, 2.0), "l2m": gen(seed + 13, 0, 1.0, 3.0),
              "mu": gen(seed + 14, 0, 0.5, 2.0)}
    abi.check(abi.lib.to_axpy2_device(arrays["l2m"].data_ptr(), arrays["mu"].data_ptr(), abi.TO_F32,
                                      npts, 0), "to_axpy2_device")
    u = [gen(seed + c, 1, 0.0, 1.0) for c in range(2)]
    f = [torch.empty(npts, dtype=torch.float32, device=dev) for _ in range(2)]
    stream = torch.cuda.Stream(device=dev)
    s = stream.cuda_stream
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            abi.sem2d_elastic_local(8, E, H, Hw, w, u, f, arrays, stream=s)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id_for(dev)) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            abi.sem2d_elastic_local(8, E, H, Hw, w, u, f, arrays, stream=s)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    alg = E * 64 * 4 * 11.0
    peak, peak_src = measured_peak_hbm()
    # CPU: the restated host loop (one thread) on a bounded sample
    from oracle import sem as osem
    from tensoroperations_b200.sem2d import synthetic_2d
    ns = 20000
    us, arr, Hh, Hwh, wh = synthetic_2d(ns)
    t0 = time.perf_counter()
    osem.sem2d_local(ns, 8, us, arr, Hh.astype(np.float32), Hwh.astype(np.float32),
                     wh.astype(np.float32), np.float32)
    cpu_s = time.perf_counter() - t0
    line = {"metric": "SEM 2D elastic P-SV stiffness Melem/s (NGLL 8, f32, element-local)",
            "value": E / (ms * 1e-3) / 1e6, "unit": "Melem/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic, generated on the device",
            "config": {"workload": f"2D elastic P-SV, NGLL 8, {E} elements, element-local",
                       "l2": f"{alg / 1e9:.1f} GB per application, no flush needed"},
            "roofline": {"bound": "hbm", "achieved": alg / (ms * 1e-3) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": alg / (ms * 1e-3) / 1e9 / peak, "traffic": None,
                         "peak_source": peak_src, "algorithmic_bytes_per_launch": alg},
            "cpu_baseline": {"value": ns / cpu_s / 1e6, "unit": "Melem/s", "cores": 1,
                             "kind": "port",
                             "sample": f"{ns} elements through the restated host loop "
                                       "(bench_sem_stiffness.cpp:1335-1385), one thread"},
            "gpu_launches": args.steps, "clocks": clocks.summary()}
    print(json.dumps(line), flush=True)
    return 0


def run_acoustic2d(args):
    """Config 1: 2D acoustic stiffness, fp64, NGLL 5, 128 x 128 quads, assembled.

    Printed with --workload acoustic2d.  The problem (29 MB) is launch-bound on
    a B200; the reference runs it on the host, so the CPU baseline (the oracle
    restatement, one thread) is the comparison that matters here."""
    import torch
    from oracle import sem as osem
    from tensoroperations_b200 import abi
    from tensoroperations_b200.sem2d import acoustic_problem
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    uh, arrays, ibool, nglob, H, Hw, w = acoustic_problem()
    E = len(ibool) // 25
    du = torch.from_numpy(uh).to(dev)
    da = {k: torch.from_numpy(v).to(dev) for k, v in arrays.items()}
    dib = torch.from_numpy(ibool).to(dev)
    f = torch.empty(nglob, dtype=torch.float64, device=dev)
    stream = torch.cuda.Stream(device=dev)
    s = stream.cuda_stream
    for _ in range(max(args.warmup, 3)):
        abi.sem2d_acoustic_apply(5, E, nglob, H, Hw, w, du, f, dib, da, np.float64, stream=s)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        abi.sem2d_acoustic_apply(5, E, nglob, H, Hw, w, du, f, dib, da, np.float64, stream=s)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    alg = E * 25 * (6 * 8 + 4) + nglob * 8 * 2
    t0 = time.perf_counter()
    for _ in range(3):
        osem.sem2d_acoustic(E, 5, nglob, ibool, uh, arrays, H, Hw, w, np.float64)
    cpu_s = (time.perf_counter() - t0) / 3
    peak, peak_src = measured_peak_hbm()
    line = {"metric": "SEM 2D acoustic stiffness Melem/s (config 1: 128x128, NGLL 5, f64)",
            "value": E / (ms * 1e-3) / 1e6, "unit": "Melem/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic, seeded",
            "config": {"workload": "2D acoustic, 128x128 quads, NGLL 5, f64, assembled (513^2 nodes)",
                       "note": "29 MB per application: launch-bound on the GPU"},
            "roofline": {"bound": "hbm", "achieved": alg / (ms * 1e-3) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": alg / (ms * 1e-3) / 1e9 / peak, "traffic": None,
                         "peak_source": peak_src, "algorithmic_bytes_per_launch": alg},
            "cpu_baseline": {"value": E / cpu_s / 1e6, "unit": "Melem/s", "cores": 1, "kind": "port",
                             "sample": "the full 128x128 problem through the oracle restatement, one thread, 3 runs"},
            "gpu_launches": args.steps}
    print(json.dumps(line), flush=True)
    return 0


def run_local(args):
    """Element-local 3D operator at the sizes of the reference's published
    numbers (H100 NVL; bench_sem_stiffness_3d.cpp:35-36): NGLL 5 with
    E = 786,432 and NGLL 8 with E = 196,608, f32, u and f per point.

    Printed with --workload local.  Inputs generated on the device."""
    import torch
    from tensoroperations_b200 import abi
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    published = {5: {"hand_ms": 3.94, "library_ms": 10.49}, 8: {"hand_ms": 13.67, "library_ms": 11.74}}
    results = {}
    peak, peak_src = measured_peak_hbm()
    for N, E in ((5, 786432), (8, 196608)):
        P = N ** 3
        npts = E * P
        _, w, H, Hw = abi.gll_operators(N)

        def gen(seed, dist, a, b, add=0.0):
            t = torch.empty(npts, dtype=torch.float32, device=dev)
            abi.check(abi.lib.to_synth_fill_device(t.data_ptr(), abi.TO_F32, 0, npts, seed, dist,
                                                    a, b, add, 0), "to_synth_fill_device")
            return t
        arrays = {}
        for r, name in enumerate(abi.POINT_ARRAYS[:9]):
            arrays[name] = gen(11 + r, 0, 0.5, 1.5, 1.0 if name in ("xix", "etay", "gamz") else 0.0)
        arrays["jac"] = gen(30, 0, 0.5, 2.0)
        arrays["l2m"] = gen(31, 0, 1.0, 3.0)
        arrays["mu"] = gen(32, 0, 0.5, 2.0)
        abi.check(abi.lib.to_axpy2_device(arrays["l2m"].data_ptr(), arrays["mu"].data_ptr(),
                                          abi.TO_F32, npts, 0), "to_axpy2_device")
        u = [gen(40 + c, 1, 0.0, 1.0) for c in range(3)]
        f = [torch.empty(npts, dtype=torch.float32, device=dev) for _ in range(3)]
        plan = abi.Sem3dPlan(np.float32, N, E, H, Hw, w)
        fl = plan.fields(u, f, arrays)
        stream = torch.cuda.Stream(device=dev)
        s = stream.cuda_stream
        for _ in range(max(args.warmup, 3)):
            plan.apply(fl, stream=s)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        steps = max(20, args.steps // 10)
        e0.record(stream)
        for _ in range(steps):
            plan.apply(fl, stream=s)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        alg = plan.algorithmic_bytes()
        results[N] = {"nelem": E, "ms": ms, "melem_s": E / (ms * 1e-3) / 1e6,
                      "gb_s": alg / (ms * 1e-3) / 1e9, "frac": alg / (ms * 1e-3) / 1e9 / peak,
                      "reference_h100_hand_ms": published[N]["hand_ms"],
                      "reference_h100_library_ms": published[N]["library_ms"],
                      "speedup_vs_reference_library": published[N]["library_ms"] / ms}
        del arrays, u, f
        torch.cuda.empty_cache()
    r5 = results[5]
    line = {"metric": "SEM 3D stiffness Melem/s, element-local f32 (the reference's published sizes)",
            "value": r5["melem_s"], "unit": "Melem/s", "n_gpus": 1, "steps": max(20, args.steps // 10),
            "warmup": args.warmup, "ms_per_step": r5["ms"], "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": r5["melem_s"] / (786432 / 3.94e-3 / 1e6),
            "dtype": "f32", "data": "synthetic, generated on the device",
            "config": {"workload": "3D elastic, element-local, NGLL 5 E=786432 and NGLL 8 E=196608",
                       "vs_baseline": "value / the reference's hand kernel on H100 NVL (199.6 Melem/s)"},
            "roofline": {"bound": "hbm", "achieved": r5["gb_s"], "peak": peak, "unit": "GB/s",
                         "frac": r5["frac"], "traffic": None, "peak_source": peak_src},
            "ngll5": results[5], "ngll8": results[8]}
    print(json.dumps(line), flush=True)
    return 0


def config_dict(prob, world, part):
    return {"workload": ("3D SEM isotropic elastic stiffness, NGLL=5, f32, structured "
                         f"{part.nex}x{part.ney}x{part.nez} hexes, assembled through ibool"),
            "nelem_per_gpu": prob.nelem, "nglob_per_gpu": prob.nglob, "ngll": prob.ngll,
            "mode": "assembled", "parallelism": f"z-slabs x{world}" if world > 1 else "single GPU",
            "l2": (f"inputs larger than L2 ({prob.plan().algorithmic_bytes() / 1e9:.2f} GB "
                   "streamed per step per GPU vs 126 MB of L2), no flush")}


def main():
    global MESH_PER_GPU
    # Native libraries write to file descriptor 1 directly (NCCL prints its
    # version line there at communicator set-up): point it at stderr and keep
    # Python's stdout on a duplicate of the original, so stdout carries only
    # the result line
    sys.stdout.flush()
    result_fd = os.dup(1)
    os.dup2(2, 1)
    sys.stdout = os.fdopen(result_fd, "w", buffering=1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--variant", type=int, default=None,
                    help="f32 kernel variant (TO_SEM3D_VARIANT): 0 point-pair 8x2, 1 TMA 8x2, "
                         "2 streaming, 3 point-pair 4x4, 4 point-pair 16x1, 5 line-owner 8x3, 6 line-owner 4x5")
    ap.add_argument("--workload", default="sem3d",
                    choices=["sem3d", "chain", "batched-gemm", "large", "sem2d", "acoustic2d",
                             "local", "gemm"],
                    help="sem3d: the headline SEM operator (default); gemm: the general "
                         "contraction's tensor-core GEMM; chain: config 4 "
                         "contraction; batched-gemm: config 2; large: config 5; sem2d: the "
                         "reference's 2D elastic operator; acoustic2d: config 1; local: "
                         "element-local at the reference's published sizes")
    ap.add_argument("--sem2d-elements", type=int, default=2621440)
    ap.add_argument("--large-mesh", type=int, default=128, help="hexes per side for --workload large")
    ap.add_argument("--gemm-size", type=int, default=4096, help="M = N = K for --workload gemm")
    ap.add_argument("--chain-extent", type=int, default=64)
    ap.add_argument("--layout", default="interleaved", choices=["components", "interleaved"],
                    help="assembled u / f on the device: interleaved per node as (x, y, z, "
                         "unused) (default; the host data stays one array per component), or "
                         "one array per component")
    ap.add_argument("--mesh", type=int, nargs=3, default=[64, 64, 64],
                    metavar=("NEX", "NEY", "NEZ"), help="hexes per GPU (profiling runs)")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="weak: --mesh per GPU (nex x ney x N*nez hexes in all); strong: the "
                         "--mesh hexes in all, split over the N GPUs")
    ap.add_argument("--no-check", action="store_true",
                    help="skip the post-run comparison of f with the one-GPU operator")
    args = ap.parse_args()
    MESH_PER_GPU = tuple(args.mesh)
    if args.variant is not None:
        os.environ["TO_SEM3D_VARIANT"] = str(args.variant)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "chain":
        return run_chain(args)
    if args.workload == "batched-gemm":
        return run_batched_gemm(args)
    if args.workload == "large":
        return run_large(args)
    if args.workload == "gemm":
        return run_gemm(args)
    if args.workload == "sem2d":
        return run_sem2d(args)
    if args.workload == "acoustic2d":
        return run_acoustic2d(args)
    if args.workload == "local":
        return run_local(args)

    import torch
    import torch.distributed as dist
    from tensoroperations_b200 import abi
    from tensoroperations_b200.sem3d import to_device

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from tensoroperations_b200.slab import SlabOperator
    strong = args.scaling == "strong"
    part, prob = make_problem(rank, world, strong)
    u, f, arrays, ibool = to_device(prob, dev)
    stream = torch.cuda.Stream(device=dev)
    il = args.layout == "interleaved"
    if il:
        # the device copy of u and f: one 16-byte node each ([nglob][4] f32)
        u4 = torch.empty((prob.nglob, 4), dtype=torch.float32, device=dev)
        abi.nodes_interleave(u, u4, prob.nglob, stream.cuda_stream)
        f4 = torch.zeros((prob.nglob, 4), dtype=torch.float32, device=dev)
        dev_u, dev_f = [u4, None, None], [f4, None, None]
        f = None  # the planar f of to_device is not used
    else:
        dev_u, dev_f = u, f
    plan = abi.Sem3dPlan(np.float32, prob.ngll, prob.nelem, prob.H, prob.Hw, prob.w,
                         nglob=prob.nglob, assembled=True, interleaved=il)
    fields = plan.fields(dev_u, dev_f, arrays, ibool)
    op = SlabOperator(part, plan, fields, [x for x in dev_f if x is not None], dev)

    clocks = ClockSampler(gpu_id_for(dev))
    clocks.__enter__()
    clocks.wait_first()
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            op.apply(stream)
    torch.cuda.synchronize()

    # ---- timed region: K steps, CUDA events on the launching stream ----
    kstarts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.begin()
    with torch.cuda.stream(stream):
        e_start.record(stream)
        for it in range(args.steps):
            op.apply(stream, (kstarts[it], kends[it]))
        e_end.record(stream)
    torch.cuda.synchronize()
    clocks.end()
    clocks.__exit__(None, None, None)
    if world > 1:
        dist.barrier()
    total_ms = e_start.elapsed_time(e_end)
    kern_ms = sum(a.elapsed_time(b) for a, b in zip(kstarts, kends)) / args.steps
    t = torch.tensor([total_ms, kern_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, kern_ms = float(t[0]), float(t[1])
    ms_per_step = total_ms / args.steps
    nelem_total = part.nex * part.ney * part.nez
    value = nelem_total / (ms_per_step * 1e-3) / 1e6

    # ---- correctness of the timed path: f of the last step against the one-GPU
    # operator on the rank's layers plus their neighbours (max over ranks) ----
    check = None
    if not args.no_check:
        if il:
            f_planar = [torch.empty(prob.nglob, dtype=torch.float32, device=dev) for _ in range(3)]
            abi.nodes_deinterleave(dev_f[0], f_planar, prob.nglob, stream.cuda_stream)
            torch.cuda.synchronize()
        else:
            f_planar = dev_f
        rel = check_against_one_gpu(part, u, f_planar, arrays, dev, stream)
        del f_planar
        t = torch.tensor([rel], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        check = {"rel_l2_max": float(t[0]), "tol": 1e-5,
                 "reference": "the same operator on one GPU (to_sem3d_apply) over each rank's "
                              "element layers plus one neighbouring layer per side; f of the "
                              "last timed step, relative L2 over the rank's nodes, max over ranks"}

    # ---- end to end through the C ABI with pinned host buffers ----
    # Every step copies its u host -> device, applies the operator and copies
    # its f device -> host.  Two device buffer sets and three streams let step
    # i's device -> host copy run during step i+1's host -> device copy (PCIe
    # is full duplex); a set is reused only after its previous step's copies
    # and kernels are done.
    # 24 steps (about 0.1 s) whatever --steps is, so the one pipeline fill and
    # drain inside the timed region weigh about 4 % of it
    e2e_steps = 0 if args.no_e2e else 24
    if e2e_steps:
        # Every step is ONE call of the C ABI's host-buffer entry
        # (to_sem3d_elastic_mgpu_host): copy u in from pinned host memory (one
        # array per component), convert it to the device layout, apply with the
        # neighbour exchange, convert f back and copy it out -- all inside the
        # timed region.  Two device buffer sets on two streams overlap one
        # step's copy-out with the next step's copy-in (PCIe is full duplex).
        u_host = [torch.from_numpy(x).pin_memory() for x in prob.u]
        f_host = [[torch.empty(prob.nglob, dtype=torch.float32).pin_memory() for _ in range(3)]
                  for _ in range(2)]
        ops, hosts, keep = [], [], []
        for k in range(2):
            if il:
                u4k = torch.empty((prob.nglob, 4), dtype=torch.float32, device=dev)
                f4k = dev_f[0] if k == 0 else torch.empty((prob.nglob, 4), dtype=torch.float32,
                                                          device=dev)
                stage = [torch.empty(prob.nglob, dtype=torch.float32, device=dev)
                         for _ in range(3)]
                flk = plan.fields([u4k, None, None], [f4k, None, None], arrays, ibool)
                keep += [u4k, f4k] + stage
                fo = [f4k]
            else:
                uk = [torch.empty(prob.nglob, dtype=torch.float32, device=dev) for _ in range(3)]
                fk = [torch.empty(prob.nglob, dtype=torch.float32, device=dev) for _ in range(3)]
                stage = [None, None, None]
                flk = plan.fields(uk, fk, arrays, ibool)
                keep += uk + fk
                fo = fk
            o = SlabOperator(part, plan, flk, fo, dev, comm=op.comm)
            o.slab.f_is_zero = 0  # the call zeroes f itself
            ops.append(o)
            h = abi.HostNodes()
            for c in range(3):
                h.u[c] = u_host[c].data_ptr()
                h.f[c] = f_host[k][c].data_ptr()
                h.stage[c] = stage[c].data_ptr() if stage[c] is not None else None
            hosts.append(h)
        e2e_streams = [torch.cuda.Stream(device=dev) for _ in range(2)]
        xs = ops[0].xstream  # one exchange stream: NCCL calls on one communicator in order

    def e2e_step(i):
        k = i % 2
        abi.sem3d_elastic_mgpu_host(plan, ops[k].fields, ops[k].slab, ops[k].comm, hosts[k],
                                    e2e_streams[k].cuda_stream, xs.cuda_stream)

    e2e_ms = 0.0
    if e2e_steps:
        for i in range(2):
            e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if e2e_steps:
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event()
        a0.record(e2e_streams[0])
        e2e_streams[1].wait_event(a0)
        for i in range(e2e_steps):
            e2e_step(i)
        ev1.record(e2e_streams[1])
        e2e_streams[0].wait_event(ev1)
        a1.record(e2e_streams[0])
        torch.cuda.synchronize()
        e2e_ms = a0.elapsed_time(a1) / e2e_steps
    t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t[0])
    bytes_uf = 3 * prob.nglob * 4

    alg = plan.algorithmic_bytes()
    peak, peak_src = measured_peak_hbm()
    achieved = alg / (kern_ms * 1e-3) / 1e9
    variant = os.environ.get("TO_SEM3D_VARIANT", DEFAULT_VARIANT)
    if il or variant == DEFAULT_VARIANT:  # the ticketed line-owner launches of the slab call
        kernel_name = KERNEL_BY_LAYOUT[args.layout]
        traffic = NCU_TRAFFIC_BY_LAYOUT[args.layout]
    else:
        kernel_name = KERNEL_NAMES.get(variant)
        traffic = (NCU_TRAFFIC_PER_LAUNCH.get(variant), NCU_TRAFFIC_SOURCE.get(variant))
    if rank == 0:
        cpu = None if args.no_cpu_baseline else cpu_baseline(prob)
        line = {
            "metric": METRIC, "value": value, "unit": "Melem/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded splitmix64 fields on a structured mesh, GLL operators)",
            "config": dict(config_dict(prob, world, part),
                           node_layout=("interleaved [nglob][4] f32 on the device (host data one "
                                        "array per component)" if il else
                                        "one [nglob] array per component")),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": (traffic[0] if tuple(MESH_PER_GPU) == (64, 64, 64) else None),
                         "traffic_source": traffic[1],
                         "peak_source": peak_src,
                         "algorithmic_bytes_per_launch": alg, "kernel_ms": kern_ms,
                         "kernel": kernel_name},
            "cpu_baseline": cpu,
            "e2e": None if not e2e_steps else
                   {"value": nelem_total / (e2e_ms * 1e-3) / 1e6, "unit": "Melem/s",
                    "h2d_bytes_per_step": bytes_uf, "d2h_bytes_per_step": bytes_uf,
                    "steps": e2e_steps,
                    "call": "to_sem3d_elastic_mgpu_host (pinned host u / f, one array per "
                            "component; copies and layout conversion inside the call)"},
            "check": check,
            "gpu_launches": args.steps * op.kernel_launches(),
            "clocks": clocks.summary(),
            "gflops": plan.flops() / (kern_ms * 1e-3) / 1e9,
        }
        print(json.dumps(line), flush=True)
    if e2e_steps:
        for o in ops:
            o.close()
    op.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if check is not None and not check["rel_l2_max"] <= check["tol"]:
        print(f"bench: f differs from the one-GPU operator: rel L2 {check['rel_l2_max']:.3e}",
              file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
