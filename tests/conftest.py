"""pytest configuration: the `gpu` marker, repo on sys.path, in-tree builds.

CPU runs (`-m "not gpu"`) need the product library and the oracle built; the
GPU test programs under tests/_bin are compiled for sm_100a here too.  Every
build is incremental, so it runs only when a source is newer than its output.  GPU tests
skip cleanly when no device is visible.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    import importlib.util
    spec = importlib.util.spec_from_file_location("tensoroperations_b200_build",
                                                  ROOT / "tensoroperations_b200" / "_build.py")
    build_mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build_mod)
    build_mod.build_library()  # loaded by path: importing the package needs the library
    from oracle import build as oracle_build
    oracle_build.build()
    from oracle import build_ref
    build_ref.build()  # no-op without the reference tree (e.g. on the GPU box)
    _cpp_test_build().build()  # sm_100a test programs under tests/_bin (incremental)


def _cpp_test_build():
    import importlib.util
    spec = importlib.util.spec_from_file_location("tests_cpp_build", ROOT / "tests" / "cpp" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _cuda_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
