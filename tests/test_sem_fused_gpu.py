"""LevelGraphs with the spectral-element stiffness shape (tests/cpp/sem_fused_gpu.cpp).

The program builds the reference's SEM level graph through the public API
(and a shuffled spelling of the same operator), runs it on the GPU and checks
every output against a double-precision host loop.  It runs twice: with the
fused line-owner kernel the launch selects for this shape, and with
TO_LEVELGRAPH_FUSED=0, which keeps the generic level evaluator.
"""
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
BIN = ROOT / "tests" / "_bin" / "sem_fused_gpu"

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fused", ["1", "0"])
def test_sem_shaped_graphs_match_the_host_loop(fused):
    if not BIN.exists():
        pytest.skip("tests/_bin not built")
    env = dict(os.environ, TO_LEVELGRAPH_FUSED=fused)
    r = subprocess.run([str(BIN)], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "ALL PASS" in r.stdout
    assert r.stdout.count("PASS") >= 5
