"""Build recipe of the product library (sm_100a CUDA + host C++ -> one .so).

`build_library()` compiles every source under csrc/ with nvcc for sm_100a and
links libtensoroperations_b200.so next to this file (in-tree, so it ships with
the repository snapshot).  The build is incremental: nothing is recompiled when
the .so is newer than every source and header.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libtensoroperations_b200.so"
OBJ_DIR = PKG / "_build"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fopenmp",
                     f"-I{INCLUDE}", "--expt-relaxed-constexpr"]


def _sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _deps():
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + \
        sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    if r.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(map(str, cmd)) + "\n" + r.stdout + r.stderr)
    return r


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/ for sm_100a and link the in-tree shared library."""
    deps = _deps()
    if not force and not _stale(LIB, deps):
        return LIB
    OBJ_DIR.mkdir(exist_ok=True)
    objs = []
    headers = [d for d in deps if d.suffix in (".cuh", ".hpp", ".h")]
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    for src in _sources():
        obj = OBJ_DIR / (src.name + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header):
            cmd = [NVCC] + NVCC_FLAGS + ["-c", str(src), "-o", str(obj)]
            if src.suffix == ".cpp":
                cmd = [NVCC, "-x", "cu"] + NVCC_FLAGS + ["-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            r = _run(cmd)
            if verbose:
                print(r.stderr)
        objs.append(obj)
    tmp = LIB.with_suffix(".so.tmp")
    _run([NVCC] + ARCH + ["-shared", "-Xcompiler", "-fopenmp", "-o", str(tmp)] +
         [str(o) for o in objs] + ["-lcudart", "-ldl"])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv))
