"""Build recipe of the C++ test programs (test infrastructure).

GPU programs are compiled here with nvcc for sm_100a into tests/_bin/
(git-ignored, shipped with the repository snapshot) so the GPU box only runs
them.  Every compile runs under a time limit.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
BIN = ROOT / "tests" / "_bin"
INC = [f"-I{ROOT / 'include'}", f"-I{ROOT / 'tensoroperations_b200' / 'include'}"]
LIBDIR = ROOT / "tensoroperations_b200"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++20",
              "--extended-lambda", "--expt-relaxed-constexpr", "-diag-suppress", "186,20012"]

GPU_PROGRAMS = {"kokkos_subset_gpu": HERE / "kokkos_subset_gpu.cpp",
                "level_graph_runtime_gpu": HERE / "level_graph_runtime_gpu.cpp",
                "tc_contract_gpu": HERE / "tc_contract_gpu.cpp",
                "sem_fused_gpu": HERE / "sem_fused_gpu.cpp"}


def _headers():
    inc = ROOT / "tensoroperations_b200" / "include"
    return sorted(inc.rglob("*.hpp")) + sorted(inc.rglob("*.cuh")) + \
        [ROOT / "include" / "tensoroperations_b200.h"]


def _stale(target: Path, deps) -> bool:
    return not target.exists() or any(d.stat().st_mtime > target.stat().st_mtime for d in deps)


def nvcc_program(src: Path, out: Path, timeout: int = 600):
    cmd = [NVCC] + NVCC_FLAGS + INC + ["-x", "cu", str(src), f"-L{LIBDIR}", "-ltensoroperations_b200",
                                       "-Xlinker", "-rpath,$ORIGIN/../../tensoroperations_b200",
                                       "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr[-4000:]}")


def build(force: bool = False):
    BIN.mkdir(exist_ok=True)
    hdr = _headers()
    built = {}
    for name, src in GPU_PROGRAMS.items():
        if not src.exists():
            continue
        out = BIN / name
        if force or _stale(out, [src] + hdr + [LIBDIR / "libtensoroperations_b200.so"]):
            nvcc_program(src, out)
        built[name] = out
    return built


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv))
