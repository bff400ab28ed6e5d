"""Build recipe of the CPU oracle (test infrastructure, see sem_oracle.cpp).

Two libraries from one source, into oracle/_build/:
  libsem_oracle.so  -O2 -ffp-contract=off   parity checker (IEEE order kept)
  libsem_cpu.so     -O3 -fopenmp            timed CPU port (cpu_baseline,
                                            bench.py --impl reference)
The CPU port targets x86-64-v3 (AVX2 + FMA) rather than -march=native because
it is built here and executed on the GPU box's host.
"""
from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build"
SRC = HERE / "sem_oracle.cpp"
ORACLE = OUT / "libsem_oracle.so"
CPU = OUT / "libsem_cpu.so"

FLAGS_ORACLE = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-std=c++17", "-fPIC", "-shared"]
FLAGS_CPU = ["-O3", "-march=x86-64-v3", "-fopenmp", "-std=c++17", "-fPIC", "-shared"]


def _stale(target: Path) -> bool:
    return not target.exists() or target.stat().st_mtime < SRC.stat().st_mtime


def build(force: bool = False):
    OUT.mkdir(exist_ok=True)
    for target, flags in ((ORACLE, FLAGS_ORACLE), (CPU, FLAGS_CPU)):
        if force or _stale(target):
            r = subprocess.run(["g++"] + flags + [str(SRC), "-o", str(target)],
                               capture_output=True, text=True, timeout=600)
            if r.returncode != 0:
                raise RuntimeError(f"oracle build failed ({target.name}):\n{r.stderr}")
    return ORACLE, CPU


if __name__ == "__main__":
    print(build(force=True))
