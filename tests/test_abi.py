"""C-ABI checks that need no GPU: the library loads, exports exactly what
include/skmetal_cuda.h declares, and the Python bridge binds every symbol."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "skmetal_cuda.h"


def _declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(skmetal_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_with_all_symbols_resolved():
    from skmetal_b200 import _bridge

    assert _bridge.CUDA_AVAILABLE, _bridge._load_error
    # RTLD_NOW: every undefined symbol must resolve at load time
    ctypes.CDLL(str(_bridge.LIB_PATH), mode=ctypes.RTLD_LOCAL | 2)


def test_header_symbols_are_exported():
    from skmetal_b200 import _bridge

    lib = ctypes.CDLL(str(_bridge.LIB_PATH))
    missing = [s for s in _declared() if not hasattr(lib, s)]
    assert not missing, missing


def test_bridge_binds_every_declared_symbol():
    from skmetal_b200 import _bridge

    declared = set(_declared())
    assert set(_bridge.EXPORTED_SYMBOLS) == declared
    _bridge._load()
    assert set(_bridge._funcs) == declared


def test_package_import_maps_no_native_code():
    """Importing the package (e.g. for its workload generators, as the bench's
    reference arm does) must not load libskmetal_cuda.so; first use does."""
    import sys

    code = ("import skmetal_b200, skmetal_b200._synthetic, skmetal_b200.estimators; "
            "from skmetal_b200 import _bridge; "
            "maps = open('/proc/self/maps').read(); "
            "assert 'libskmetal_cuda' not in maps, 'mapped at import'; "
            "assert not _bridge.is_loaded(); "
            "_bridge.CUDA_AVAILABLE; "
            "assert 'libskmetal_cuda' in open('/proc/self/maps').read(), 'not mapped on first use'")
    r = subprocess.run([sys.executable, "-c", code], cwd=str(ROOT), capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]


def test_dynamic_symbol_table_has_only_the_c_abi():
    from skmetal_b200 import _bridge

    out = subprocess.run(["nm", "-D", "--defined-only", str(_bridge.LIB_PATH)], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("nm unavailable")
    exported = {ln.split()[-1] for ln in out.stdout.splitlines() if " T " in ln}
    skm = {s for s in exported if s.startswith("skmetal_")}
    assert skm == set(_declared())


def test_library_has_no_unresolved_project_symbols():
    from skmetal_b200 import _bridge

    out = subprocess.run(["nm", "-D", "--undefined-only", str(_bridge.LIB_PATH)], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("nm unavailable")
    bad = [ln for ln in out.stdout.splitlines() if "skm" in ln]
    assert not bad, bad


def test_wrappers_raise_without_gpu():
    from skmetal_b200 import _bridge
    import numpy as np

    if _bridge.GPU_AVAILABLE:
        pytest.skip("GPU present")
    X = np.ones((4, 2), dtype=np.float32)
    with pytest.raises(RuntimeError, match="no CPU fallback|CUDA"):
        _bridge.kmeans_fit(X, X[:2].copy(), 5, 0.0)
