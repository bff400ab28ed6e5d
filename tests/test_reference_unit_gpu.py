"""The reference's own unit tests, unmodified, on B200 (GPU).

oracle/_ref/test_<name> are the reference's tests/test_<name>.cpp compiled for
sm_100a against this repository's frontend and Kokkos subset, with
tests/cpp/gtest_shim standing in for the GoogleTest calls they make
(oracle/build_ref.py):
  test_dag_graph         a tree re-expressed as a DAG gives bit-identical
                         results and the same un-pooled scratch; a diamond DAG
                         (one node, two consumers) gives the tree's numbers at
                         less scratch; multi-tiled grid labels gathered by label;
  test_contraction_node  node construction, shapes, stored hooks;
  test_device_tuple      DeviceTuple on host and in a kernel;
  test_concept           TensorLike and the handle's element access;
  test_level_graph       the LevelGraph slot algebra, tile derivation and level
                         guards (static), and graphs executed against host
                         references: one contraction, a three-direction
                         gradient level, combine over contraction, multi-output
                         combine, declared-order roots, combines and
                         contractions over declared slots, the combine's
                         global coordinate;
  test_level_liveness    level liveness and left-edge pooling (static), and the
                         pooled chain ((A B) E) F against a host reference;
  test_label_tiles       every SEM3D tile from the label map (static);
  test_graph             the tree route: einsum permutation plans (static), one
                         and several tiles per label, non-square and
                         non-symmetric tiles, permuted inputs / outputs /
                         contracted order, input and contraction hooks at
                         global indices across tiles, fused two-level chains,
                         permuted fused operands -- each against a host loop;
  test_nodehandle        node tags, input nodes over a user TensorLike type;
  test_slot_liveness     DAG slot liveness and pooling;
  test_combine_node      combines: label gathers, multi-output combines,
                         combines over permuted and hooked contractions and
                         over other combines, coordinates -- against host
                         loops.
The level-graph tests also name the reference's internal plan names, which
b200/ImplNames.hpp spells over this build's plan code.  Their static asserts
are checked when oracle/build_ref.py compiles them.  Each program prints one
line per test and exits non-zero if any failed.
"""
import subprocess
from pathlib import Path

import pytest

REF = Path(__file__).resolve().parent.parent / "oracle" / "_ref"

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["test_dag_graph", "test_contraction_node", "test_device_tuple",
                                  "test_concept", "test_level_graph", "test_level_liveness",
                                  "test_label_tiles", "test_graph", "test_nodehandle",
                                  "test_slot_liveness", "test_combine_node"])
def test_reference_unit_test_passes(name):
    exe = REF / name
    if not exe.exists():
        pytest.skip("oracle/_ref not built")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "[  FAILED  ]" not in r.stdout
    assert "[       OK ]" in r.stdout
