"""The reference's flat-DAG SEM 3D program, unmodified, on B200 (GPU).

oracle/_ref/bench_sem_stiffness_3d is benchmarks/sem_stiffness_3d/
bench_sem_stiffness_3d.cpp compiled for sm_100a against this repository's
frontend (make_dag / DagGraph::add / as<> / multi-output combines / outputs /
execute(TeamPolicyTag<>)) and Kokkos subset (TeamPolicy + team scratch for its
hand kernel, MDRangePolicy<Rank<4>> for its naive kernel), built by
oracle/build_ref.py where the reference tree is mounted.  The program sweeps
TE in {2, 4, 8} x team size in {32 .. 512} for the 24-node DAG and its hand
kernel, runs its two-pass naive kernel, checks each against its own host
reference (max error / max |ref| < 1e-4) and returns 0 only if all three pass.
Profile mode (5 arguments) runs one launch of the DAG and the hand kernel at
one TE and team size and prints both errors.
"""
import re
import subprocess
from pathlib import Path

import pytest

BIN = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "bench_sem_stiffness_3d"

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not BIN.exists(), reason="oracle/_ref not built")]


def _run(args, timeout=900):
    r = subprocess.run([str(BIN)] + [str(a) for a in args], capture_output=True, text=True,
                       timeout=timeout)
    return r


def test_dag_program_sweep_passes_its_own_check():
    r = _run([4096, 1, 1])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    # the results table: "impl time TE team GFLOP/s vs-naive PASS(err)"
    rows = {ln.split()[0]: ln for ln in r.stdout.splitlines()
            if ln.split() and ln.split()[0] in ("naive", "hand", "library")
            and ("PASS(" in ln or "FAIL(" in ln)}
    assert set(rows) == {"naive", "hand", "library"}, r.stdout[-3000:]
    for name, ln in rows.items():
        assert "PASS" in ln, (name, ln)


@pytest.mark.parametrize("te,team", [(2, 64), (4, 128), (8, 256)])
def test_dag_program_profile_mode(te, team):
    r = _run([2048, 1, 1, te, team])
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    m = re.search(r"profile: N=5 E=\d+ TE=(\d+) team=(\d+)\s+lib_err=(\S+) hand_err=(\S+)", r.stdout)
    assert m, r.stdout[-2000:]
    assert int(m.group(1)) == te and int(m.group(2)) == team
    assert float(m.group(3)) < 1e-4 and float(m.group(4)) < 1e-4, m.group(0)
