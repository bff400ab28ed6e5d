"""The reference's contraction benchmarks, unmodified, on B200 (GPU).

oracle/_ref/bench_<name> are benchmarks/<name>/bench_<name>.cpp compiled for
sm_100a against this repository's frontend and Kokkos subset by
oracle/build_ref.py:
  permuted_contraction  C = sum_{j,k} A B through the tree route for five index
                        orders of A, B and C, the contracted labels (16 each)
                        spanning two tiles of 8 -- the self-staging contraction
                        path; the program checks every variant against the
                        canonical one;
  team_contraction      the same contraction against its own naive and
                        hand-tiled Kokkos team kernels, LayoutRight and
                        LayoutLeft inputs;
  permuted_combine      a contraction with a hook feeding a combine, the operand
                        in four staging paths; every path must give one result;
  multilevel_contraction E = (A B) D against its naive and hand-tiled chains,
                        the intermediate's contracted label in one tile (one
                        fused launch) and in four (run in steps: intermediate
                        into a buffer, then the root).
Each program prints PASS per row when its result matches (max relative
difference < 1e-2); these tests require every row to pass (they do not hold
the programs' timing ratios).
"""
import subprocess
from pathlib import Path

import pytest

REF = Path(__file__).resolve().parent.parent / "oracle" / "_ref"

pytestmark = pytest.mark.gpu


def _run(name, args=()):
    exe = REF / f"bench_{name}"
    if not exe.exists():
        pytest.skip("oracle/_ref not built")
    r = subprocess.run([str(exe), *map(str, args)], capture_output=True, text=True, timeout=900)
    return r


def _result_rows(stdout):
    return [ln for ln in stdout.splitlines() if "PASS(" in ln or "FAIL(" in ln]


@pytest.mark.parametrize("name", ["permuted_contraction", "team_contraction", "permuted_combine",
                                  "multilevel_contraction"])
def test_contraction_benchmark_results_match(name):
    r = _run(name)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    rows = _result_rows(r.stdout)
    assert rows, r.stdout[-2000:]
    bad = [ln for ln in rows if "FAIL(" in ln]
    assert not bad, bad
