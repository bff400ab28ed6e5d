"""Build recipe for artefacts compiled from the REFERENCE's own sources.

Test infrastructure only.  Run here, where the reference tree is mounted; the
outputs (in oracle/_ref/, git-ignored, shipped with the repository snapshot)
are what the tests use on the GPU box, which has no reference tree.

  libref_sem3d.so         benchmarks/sem_stiffness_3d/bench_sem3d_levelgraph.cpp
                          compiled host-only (g++, -ffp-contract=off) through
                          oracle/ref_pin.cpp: the reference's fill() and
                          reference() behind a C ABI, to pin the CPU oracle.
  bench_sem3d_levelgraph  the same reference program, unmodified, compiled for
                          sm_100a against this repository's frontend headers
                          and Kokkos subset: the drop-in check (its own
                          PASS/FAIL against its own host reference).
  bench_sem_stiffness_3d  benchmarks/sem_stiffness_3d/bench_sem_stiffness_3d.cpp
                          (the flat-DAG route: make_dag / add / multi-output
                          combines, its hand-written team kernel and its
                          MDRange kernel), unmodified, the same way.
  bench_sem_stiffness_2d  benchmarks/sem_stiffness/bench_sem_stiffness.cpp (the
                          2D P-SV program: the tree route make_graph().ops /
                          nested bundles, the DAG and multi-output DAG routes,
                          its hand-written and CONTROL kernels), the same way.
  bench_permuted_contraction, bench_multilevel_contraction,
  bench_permuted_combine, bench_team_contraction
                          the contraction benchmarks (tree route, nested and
                          flat tile bundles, hooks, LayoutLeft views), the
                          same way.
  test_<name>             the reference's unit tests that use only the public
                          API (tests/test_dag_graph.cpp, test_device_tuple.cpp,
                          test_contraction_node.cpp, test_concept.cpp),
                          unmodified, compiled for sm_100a against the frontend
                          and tests/cpp/gtest_shim (a stand-in for the GoogleTest
                          calls they make; GoogleTest is not installed).
  libref_sem2d.so         that 2D source compiled host-only through
                          oracle/ref_pin2d.cpp: its fill_field(),
                          fill_operators() and host_reference() behind a C
                          ABI, to pin the 2D oracle.

The reference's own build (CMake fetching Kokkos/GoogleTest/KokkosKernels) is
not used; Kokkos is replaced by tensoroperations_b200/include/Kokkos_Core.hpp.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
OUT = HERE / "_ref"
# The reference tree: TO_REFERENCE_ROOT, else a `reference` directory beside
# this repository's checkout.  Nothing here runs where neither exists.
REF = Path(os.environ.get("TO_REFERENCE_ROOT", str(ROOT.parent / "reference")))
SEM3D = REF / "benchmarks" / "sem_stiffness_3d" / "bench_sem3d_levelgraph.cpp"
SEM3D_DAG = REF / "benchmarks" / "sem_stiffness_3d" / "bench_sem_stiffness_3d.cpp"
SEM2D = REF / "benchmarks" / "sem_stiffness" / "bench_sem_stiffness.cpp"
CONTRACTION_BENCHES = ("permuted_contraction", "multilevel_contraction", "permuted_combine",
                       "team_contraction")
# reference unit tests that compile against the public API alone, with
# whether the file defines its own main()
UNIT_TESTS = {"test_dag_graph": True, "test_device_tuple": True, "test_contraction_node": True,
              "test_concept": False, "test_level_graph": True, "test_level_liveness": True,
              "test_label_tiles": True, "test_graph": True, "test_nodehandle": True,
              "test_slot_liveness": True, "test_combine_node": True}
GTEST_SHIM = ROOT / "tests" / "cpp" / "gtest_shim"
INC = [f"-I{ROOT / 'include'}", f"-I{ROOT / 'tensoroperations_b200' / 'include'}"]
LIBDIR = ROOT / "tensoroperations_b200"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

PIN = OUT / "libref_sem3d.so"
DROPIN = OUT / "bench_sem3d_levelgraph"
DROPIN_DAG = OUT / "bench_sem_stiffness_3d"
DROPIN_2D = OUT / "bench_sem_stiffness_2d"
PIN2D = OUT / "libref_sem2d.so"


def available() -> bool:
    return SEM3D.exists()


def _run(cmd, timeout=900):
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError("reference build failed: " + " ".join(map(str, cmd)) + "\n" + r.stderr[-4000:])


def _stale(target: Path, deps) -> bool:
    return not target.exists() or any(d.stat().st_mtime > target.stat().st_mtime for d in deps)


def _frontend_headers():
    inc = ROOT / "tensoroperations_b200" / "include"
    return sorted(inc.rglob("*.hpp")) + sorted(inc.rglob("*.cuh")) + [ROOT / "include" / "tensoroperations_b200.h"]


def build(force: bool = False):
    if not available():
        return None
    OUT.mkdir(exist_ok=True)
    deps = [SEM3D, HERE / "ref_pin.cpp"] + _frontend_headers()
    if force or _stale(PIN, deps):
        _run(["g++", "-std=c++20", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
              *INC, f'-DBENCH_SEM3D_SOURCE="{SEM3D}"', str(HERE / "ref_pin.cpp"),
              f"-L{LIBDIR}", "-ltensoroperations_b200", f"-Wl,-rpath,{LIBDIR}",
              "-Wl,-rpath,$ORIGIN/../../tensoroperations_b200", "-o", str(PIN)])
    if SEM2D.exists() and (force or _stale(PIN2D, deps + [SEM2D, HERE / "ref_pin2d.cpp"])):
        _run(["g++", "-std=c++20", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
              *INC, f'-DBENCH_SEM2D_SOURCE="{SEM2D}"', str(HERE / "ref_pin2d.cpp"),
              f"-L{LIBDIR}", "-ltensoroperations_b200", f"-Wl,-rpath,{LIBDIR}",
              "-Wl,-rpath,$ORIGIN/../../tensoroperations_b200", "-o", str(PIN2D)])
    progs = [(SEM3D, DROPIN), (SEM3D_DAG, DROPIN_DAG), (SEM2D, DROPIN_2D)]
    progs += [(REF / "benchmarks" / b / f"bench_{b}.cpp", OUT / f"bench_{b}") for b in CONTRACTION_BENCHES]
    for src, out in progs:
        if src.exists() and (force or _stale(out, deps + [src, LIBDIR / "libtensoroperations_b200.so"])):
            _nvcc_program(src, out)
    shim = [GTEST_SHIM / "gtest" / "gtest.h", GTEST_SHIM / "gtest_main.cpp"]
    for name, has_main in UNIT_TESTS.items():
        src = REF / "tests" / f"{name}.cpp"
        out = OUT / name
        if src.exists() and (force or _stale(out, deps + shim + [src, LIBDIR / "libtensoroperations_b200.so"])):
            extra = [] if has_main else [str(GTEST_SHIM / "gtest_main.cpp")]
            _nvcc_program(src, out, [f"-I{GTEST_SHIM}"], extra)
    return PIN, DROPIN, DROPIN_DAG, DROPIN_2D, PIN2D


def _nvcc_program(src: Path, out: Path, inc=(), extra_sources=()):
    _run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++20",
          "--extended-lambda", "--expt-relaxed-constexpr", "-diag-suppress", "186,20012",
          *INC, *inc, "-x", "cu", str(src), *extra_sources, f"-L{LIBDIR}", "-ltensoroperations_b200",
          "-Xlinker", "-rpath,$ORIGIN/../../tensoroperations_b200", "-o", str(out)])


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
