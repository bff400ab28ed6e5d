"""The reference's 2D SEM program, unmodified, on B200 (GPU).

oracle/_ref/bench_sem_stiffness_2d is benchmarks/sem_stiffness/
bench_sem_stiffness.cpp (2D elastic P-SV, NGLL 8, f32) compiled for sm_100a
against this repository's frontend and Kokkos subset by oracle/build_ref.py.
It runs the operator through the tree route (make_graph().ops(node) with a
nested Tile / CombineTile bundle, one launch per force component), the flat
DAG route (both components, one launch) and the multi-output DAG route, next
to its own hand-written baseline and CONTROL kernels, and checks each against
its own host reference (max relative difference < 1e-2 on a prefix of up to
65,536 elements); it returns non-zero if the baseline or any library route
fails.
"""
import subprocess
from pathlib import Path

import pytest

BIN = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "bench_sem_stiffness_2d"

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not BIN.exists(), reason="oracle/_ref not built")]

ROWS = ("library (fused, 2 kernels)", "library DAG (1 kernel)", "library DAG-MO (2-out F)")


def test_2d_program_passes_its_own_check():
    r = subprocess.run([str(BIN), "65536", "1", "1"], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    for row in ROWS:
        lines = [ln for ln in r.stdout.splitlines() if ln.startswith(row)]
        assert lines and lines[0].rstrip().endswith("PASS"), (row, lines, r.stdout[-2000:])
