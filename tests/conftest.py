"""Shared pytest setup: the ``gpu`` marker, repo paths and package loading."""
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def load_backend():
    """Import the ``tensor-lang_b200`` directory as package ``tensor_lang_b200``."""
    if "tensor_lang_b200" in sys.modules:
        return sys.modules["tensor_lang_b200"]
    pkg_dir = REPO / "tensor-lang_b200"
    spec = importlib.util.spec_from_file_location(
        "tensor_lang_b200", pkg_dir / "__init__.py", submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["tensor_lang_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def golden(name):
    return json.loads((GOLDEN / name).read_text())


def arr(j):
    return np.asarray(j["data"], dtype=np.float64).reshape(j["shape"])


def assert_close(got, ref, rtol, name="", atol=None):
    """|got - ref| <= rtol*|ref| + atol elementwise, atol = rtol * max|ref| unless given.

    Near-zero entries of long sums and products cannot meet a pure relative
    bound, so the absolute part is scaled to the tensor's magnitude.
    """
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (name, got.shape, ref.shape)
    if ref.size == 0:
        return
    scale = float(np.abs(ref).max())
    if atol is None:
        atol = rtol * scale
    err = np.abs(got - ref)
    bad = err > rtol * np.abs(ref) + atol
    if bad.any():
        i = int(np.argmax(err - (rtol * np.abs(ref) + atol)))
        raise AssertionError(
            f"{name}: {int(bad.sum())}/{ref.size} outside rtol={rtol} atol={atol:.3g}; "
            f"worst at {np.unravel_index(i, ref.shape)}: got {got.flat[i]!r} ref {ref.flat[i]!r}")


def gpu_available():
    try:
        tl = load_backend()
        from tensor_lang_b200 import runtime as rt
        import ctypes
        n = ctypes.c_int(0)
        rt.load_library().tl_device_count(ctypes.byref(n))
        return n.value > 0
    except Exception:
        return False
