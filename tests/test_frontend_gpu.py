"""The LevelGraph runtime and the Kokkos subset on the device.

Both programs are compiled for sm_100a by tests/cpp/build.py (here, or by
conftest when stale) and only run on the GPU box:
* kokkos_subset_gpu: Views, mirrors, deep_copy, RangePolicy/TeamPolicy
  launches, team scratch and the nested range loops, step by step.
* level_graph_runtime_gpu: graphs of every member kind (stage, contraction
  with permuted/relabelled operands, combine with coordinates, several roots,
  ragged last tile) executed at two team sizes against host loops.
"""
import subprocess
from pathlib import Path

import pytest

BIN = Path(__file__).resolve().parent / "_bin"


@pytest.mark.gpu
@pytest.mark.parametrize("program", ["kokkos_subset_gpu", "level_graph_runtime_gpu"])
def test_program(program):
    exe = BIN / program
    assert exe.exists(), f"{exe} not built (tests/cpp/build.py)"
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    print(r.stdout[-4000:])
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
