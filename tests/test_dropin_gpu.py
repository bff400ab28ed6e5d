"""The reference's own SEM3D level-graph program, unmodified, on B200 (GPU).

oracle/_ref/bench_sem3d_levelgraph is benchmarks/sem_stiffness_3d/
bench_sem3d_levelgraph.cpp compiled for sm_100a against this repository's
frontend (make_level_graph / add / make_*_node / outputs / execute) and Kokkos
subset (built by oracle/build_ref.py where the reference tree is mounted).  It
builds the SEM graph through the public API, static_asserts the plan (6 levels,
35 slots, 19 pools), sweeps TE x team size, runs both the level graph and its
hand-written Kokkos team kernel, and checks both against its own host
reference (max error / max |ref| < 1e-4), returning 0 only if both pass.
"""
import subprocess
from pathlib import Path

import pytest

BIN = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "bench_sem3d_levelgraph"

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not BIN.exists(), reason="oracle/_ref not built")]


def _run(args, timeout=900):
    r = subprocess.run([str(BIN)] + [str(a) for a in args], capture_output=True, text=True,
                       timeout=timeout)
    return r


def test_reference_program_sweep_passes_its_own_check():
    r = _run([8192, 2, 1])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "levelgraph" in r.stdout and "PASS" in r.stdout


def test_reference_program_profile_mode_tiles():
    # 5 arguments: one launch of each implementation at a given TE and team
    for te, team in ((1, 128), (2, 256), (4, 512)):
        r = _run([4096, 1, 1, te, team])
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        assert f"profile TE={te}" in r.stdout
        line = [ln for ln in r.stdout.splitlines() if ln.startswith("profile")][0]
        errs = [float(x.rstrip(",")) for x in line.replace(",", " ").split() if "e-" in x or "e+" in x]
        assert errs and max(errs) < 1e-4, line
