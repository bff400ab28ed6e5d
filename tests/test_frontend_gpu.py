"""The LevelGraph runtime and the Kokkos subset on the device.

Both programs are compiled for sm_100a by tests/cpp/build.py (here, or by
conftest when stale) and only run on the GPU box:
* kokkos_subset_gpu: Views, mirrors, deep_copy, RangePolicy/TeamPolicy
  launches, team scratch and the nested range loops, step by step.
* level_graph_runtime_gpu: graphs of every member kind (stage, contraction
  with permuted/relabelled operands, combine with coordinates, several roots,
  ragged last tile) executed at two team sizes against host loops.
* tc_contract_gpu: one large fp32 contraction of two inputs (permuted
  operands and output, hooks, ragged sizes) through the tree and DAG routes,
  which the frontend runs as a tensor-core GEMM -- and, with
  TO_FRONTEND_TENSOR_CORES=0, on the level evaluator -- against float64 host
  loops (relative L2 <= 1e-5); the league execute() returns shows which path
  ran (the GEMM's 128 x 256 tile count on the tensor cores).  The same
  program runs contraction chains whose intermediate is contracted over
  several tiles: the tree then runs in steps (intermediate into a buffer,
  then the root), the root of the largest on the tensor cores; and the
  permuted rank-4 chain (config 4) through the same API.
"""
import os
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


# league per case: the GEMM tile count (tensor cores) / the level grid
TC_LEAGUES = {"tree_large": 6, "dag_large": 6, "tree_square": 8, "chain_large": 6,
              "chain_large_one_tile": 128}


@pytest.mark.gpu
@pytest.mark.parametrize("tensor_cores", [True, False])
def test_tensor_core_contraction(tensor_cores):
    exe = BIN / "tc_contract_gpu"
    assert exe.exists(), f"{exe} not built (tests/cpp/build.py)"
    env = dict(os.environ)
    if not tensor_cores:
        env["TO_FRONTEND_TENSOR_CORES"] = "0"
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, env=env)
    print(r.stdout[-4000:])
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    leagues = {ln.split()[1]: int(ln.split()[-1]) for ln in r.stdout.splitlines()
               if ln.startswith("case ")}
    assert set(leagues) == {"tree_large", "dag_large", "tree_square", "dag_small",
                            "chain_one_tile", "chain_three_tiles", "chain_large",
                            "chain_large_one_tile", "config4_n32"}
    for name, tiles in TC_LEAGUES.items():
        assert (leagues[name] == tiles) == tensor_cores, (name, leagues[name])
