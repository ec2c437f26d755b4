"""The bounds-checked debug engine (lib/libcuvs_b200_debug.so).

GPU: tests/debug_bounds_worker.py runs the shapes that stress the kernels'
index arithmetic through the debug library, in its own process; any bounds
check that trips fails the search (KNN_ECUDA).  CPU: the debug library is
built next to the release one and exports the same C ABI.
"""
import ctypes
import os
import subprocess
import sys

import pytest

from conftest import ROOT

DEBUG_LIB = os.path.join(ROOT, "cuvs-silicon_b200", "lib", "libcuvs_b200_debug.so")


def test_debug_library_exports_the_c_abi(engine):
    assert os.path.exists(DEBUG_LIB), "build the engine first (make -C cuvs-silicon_b200)"
    lib = ctypes.CDLL(DEBUG_LIB)
    missing = [n for n in engine.header_functions() if not hasattr(lib, n)]
    assert not missing, missing


@pytest.mark.gpu
def test_debug_bounds_build_stays_in_bounds(engine):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "debug_bounds_worker.py")],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    assert "ok re-rank" in r.stdout
