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
