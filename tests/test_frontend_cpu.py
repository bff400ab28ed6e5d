"""The LevelGraph frontend on the host (no GPU).

* frontend_static.cpp: the planner's slot algebra, tile derivation, declared
  order and the SEM3D plan (6 levels, 35 slots, 19 pools) as static_asserts,
  plus host-side scratch sizing -- compiled by g++ and run.
* level_guard_negative.cpp: every planner guard fires on the graph it forbids,
  with its own diagnostic (the wording the reference's negative tests pin,
  tests/negative/level_guard_negative.cpp and labeltiles_guard_negative.cpp);
  the control case compiles.
* level_kernel_host_check.cpp: the device evaluator (LevelKernel.cuh) compiled
  as host code, one thread per CTA, run on a SEM-shaped graph under
  AddressSanitizer/UBSan and compared with a direct loop -- every pooled-slot
  offset, stride and root store stays inside its buffer.
* dag_host_check.cpp: the flat-DAG route (make_dag / add / as<> / three-output
  combines) lowered onto the level plan -- 6 levels, 57 slots, the grid from
  the last node -- and run through the same host-compiled evaluator under
  AddressSanitizer/UBSan against a direct loop, with a partial last tile.
* the reference's own negative-compilation files, unmodified, from where they
  lie (tests/negative/level_guard_negative.cpp cases 0-5 and
  labeltiles_guard_negative.cpp cases 0-2): each failing case must fail with
  the regular expression the reference's CMakeLists.txt:231-295 pins for it,
  and the controls must compile (skipped where the reference tree is absent).
* dag_guard_negative.cpp: each DagGraph diagnostic fires on the graph it
  forbids; the control graph compiles.
* kokkos_subset_host_check.cpp: the Kokkos subset on the host -- scratch
  requests set on a policy by statement, LayoutLeft views, MDRangePolicy.
* tree_host_check.cpp: the tree route (make_graph().ops with nested Tile /
  CombineTile bundles, and a flat pre-order tile list of a contraction chain)
  lowered through the DAG onto the level plan and run the same way.
"""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CPP = ROOT / "tests" / "cpp"
INC = ["-I", str(ROOT / "include"), "-I", str(ROOT / "tensoroperations_b200" / "include")]
LIBDIR = ROOT / "tensoroperations_b200"
GXX = shutil.which("g++")

pytestmark = pytest.mark.skipif(GXX is None, reason="g++ not found")

GUARDS = {
    1: "a level must be NON-EMPTY and HOMOGENEOUS",
    2: "must share ONE iteration space",
    3: "must share ONE iteration space",
    4: "may not read a slot ITS OWN LEVEL",
    5: "must share ONE iteration space",
    6: "may appear at most once in the map",
    7: "must appear in the graph's tile",
}
ALL_MESSAGES = set(GUARDS.values())


# The reference's own negative files and the message its CMakeLists.txt
# requires of each failing case (PASS_REGULAR_EXPRESSION, :231-238, :285-295).
REF_NEGATIVE = {
    ("level_guard_negative.cpp", "LEVEL_NEG_CASE"): {
        0: None, 1: "a level must be NON-EMPTY and HOMOGENEOUS",
        2: "must share ONE iteration space", 3: "must share ONE iteration space",
        4: "may not read a slot ITS OWN LEVEL", 5: "must share ONE iteration space"},
    ("labeltiles_guard_negative.cpp", "LABELTILES_NEG_CASE"): {
        0: None, 1: "may appear at most once in the map", 2: "must appear in the graph's tile"},
}


def _reference_root():
    import os
    root = Path(os.environ.get("TO_REFERENCE_ROOT", str(ROOT.parent / "reference")))
    return root if (root / "tests" / "negative").is_dir() else None


def _compile(args, timeout=300):
    return subprocess.run([GXX, "-std=c++20", *INC, *args], capture_output=True, text=True,
                          timeout=timeout)


def test_static_plan_checks(tmp_path):
    exe = tmp_path / "frontend_static"
    r = _compile([str(CPP / "frontend_static.cpp"), f"-L{LIBDIR}", "-ltensoroperations_b200",
                  f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)])
    assert r.returncode == 0, r.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "pools 19" in run.stdout


@pytest.mark.parametrize("case", [0, *GUARDS])
def test_level_guard(case):
    r = _compile(["-fsyntax-only", f"-DNEG_CASE={case}", str(CPP / "level_guard_negative.cpp")])
    if case == 0:
        assert r.returncode == 0, r.stderr[-3000:]
        return
    assert r.returncode != 0
    fired = {m for m in ALL_MESSAGES if m in r.stderr}
    assert fired == {GUARDS[case]}, (case, fired, r.stderr[-2000:])


@pytest.mark.parametrize("elements", [5, 6])
def test_evaluator_host_emulation_under_sanitizers(tmp_path, elements):
    exe = tmp_path / "lk_host"
    r = _compile(["-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
                  str(CPP / "level_kernel_host_check.cpp"), "-o", str(exe)], timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    run = subprocess.run([str(exe), str(elements)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "max abs error" in run.stdout


DAG_GUARDS = {
    1: "a contraction node's tile must be Tile<TileA, TileB, TileC>",
    2: "names a slot that no earlier node of this graph produced",
    3: "the node's output tile differs from the tile its operands' tiles give it",
    4: "a handle operand's tile in this node's tile spec differs from the tile its producer",
}


@pytest.mark.parametrize("case", [0, *DAG_GUARDS])
def test_dag_guard(case):
    r = _compile(["-fsyntax-only", f"-DNEG_CASE={case}", str(CPP / "dag_guard_negative.cpp")])
    if case == 0:
        assert r.returncode == 0, r.stderr[-3000:]
        return
    assert r.returncode != 0
    fired = {m for m in DAG_GUARDS.values() if m in r.stderr}
    assert fired == {DAG_GUARDS[case]}, (case, fired, r.stderr[-2000:])


@pytest.fixture(scope="module")
def dag_host_exe(tmp_path_factory):
    exe = tmp_path_factory.mktemp("dag") / "dag_host"
    r = _compile(["-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
                  str(CPP / "dag_host_check.cpp"), "-o", str(exe)], timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return exe


@pytest.mark.parametrize("form", [0, 1])
@pytest.mark.parametrize("elements", [1, 5, 6])
def test_dag_lowering_host_emulation_under_sanitizers(dag_host_exe, elements, form):
    """form 0: operands staged by stage levels; 1: self-staging contractions."""
    run = subprocess.run([str(dag_host_exe), str(elements), str(form)], capture_output=True,
                         text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "max abs error" in run.stdout and "pools" in run.stdout


@pytest.fixture(scope="module")
def tree_host_exe(tmp_path_factory):
    exe = tmp_path_factory.mktemp("tree") / "tree_host"
    r = _compile(["-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
                  str(CPP / "tree_host_check.cpp"), "-o", str(exe)], timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return exe


@pytest.mark.parametrize("elements", [1, 5, 6])
def test_tree_lowering_host_emulation_under_sanitizers(tree_host_exe, elements):
    run = subprocess.run([str(tree_host_exe), str(elements)], capture_output=True, text=True,
                         timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "tree max abs error" in run.stdout and "chain max abs error" in run.stdout
    assert "ktiles max abs error" in run.stdout


def test_kokkos_subset_on_the_host(tmp_path):
    exe = tmp_path / "kk_host"
    r = _compile(["-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
                  str(CPP / "kokkos_subset_host_check.cpp"), "-o", str(exe)], timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and "kokkos subset host ok" in run.stdout, run.stdout + run.stderr


@pytest.mark.parametrize("fname,macro,case", [(f, m, c) for (f, m), cases in REF_NEGATIVE.items()
                                              for c in cases])
def test_reference_negative_file_unmodified(fname, macro, case):
    ref = _reference_root()
    if ref is None:
        pytest.skip("reference tree not mounted")
    want = REF_NEGATIVE[(fname, macro)][case]
    r = _compile(["-fsyntax-only", f"-D{macro}={case}", str(ref / "tests" / "negative" / fname)])
    if want is None:
        assert r.returncode == 0, r.stderr[-3000:]
    else:
        assert r.returncode != 0
        assert want in r.stderr, r.stderr[-3000:]
