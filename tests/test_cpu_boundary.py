"""CPU-side checks of the drop-in boundary (no GPU needed).

* the C library loads and exports every entry point ``include/tlb200.h``
  declares, with the ctypes signatures the host binds;
* ``KernelGenerator`` returns the reference generator's ``kernel_info``
  tuples for the same calls (``tests/golden/kinfo_cases.json``);
* every reference test program lowers, fuses and generates region kernels.
"""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from conftest import REPO, arr, golden, load_backend

tl = load_backend()
from tensor_lang_b200 import runtime as rt  # noqa: E402
from tensor_lang_b200.engine import Program  # noqa: E402
from tensor_lang_b200.steps import RegionStep  # noqa: E402


def header_symbols():
    text = (REPO / "include" / "tlb200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tl_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_header():
    lib = rt.load_library()
    syms = header_symbols()
    assert len(syms) >= 50
    for s in syms:
        assert hasattr(lib, s), s
    # the host binding covers exactly the header
    assert sorted(rt.EXPORTED) == syms


def test_library_without_gpu_reports_no_device():
    lib = rt.load_library()
    n = ctypes.c_int(-1)
    lib.tl_device_count(ctypes.byref(n))
    assert n.value >= 0
    assert lib.tl_error_string(1001).decode().startswith("invalid argument")


def _tup(x):
    if isinstance(x, list):
        return tuple(_tup(v) for v in x)
    return x


@pytest.mark.parametrize("case", golden("kinfo_cases.json"),
                         ids=lambda c: f"{c['method']}-{c['args'][1]}-{len(c['args'])}")
def test_kernel_info_matches_reference(case):
    gen = tl.KernelGenerator(False)
    args = []
    for a in case["args"]:
        if isinstance(a, list) and a and not isinstance(a[0], (dict, str)):
            args.append(tuple(a))
        else:
            args.append(a)
    if case["kinfo"] is None:
        with pytest.raises(NotImplementedError):
            getattr(gen, case["method"])(*args)
        return
    src, kinfo = getattr(gen, case["method"])(*args)
    assert isinstance(src, str)
    assert _tup(list(kinfo)) == _tup(case["kinfo"])


def test_generator_validates_like_reference():
    gen = tl.KernelGenerator(False)
    with pytest.raises(ValueError):
        gen.elementwise("pow", "c", "a", "b", 4)
    with pytest.raises(NotImplementedError):
        gen.sum("sum", "s", "x", 2, (2, 3, 4))


PROGS = golden("ref_programs.json")


@pytest.mark.parametrize("name", sorted(PROGS))
def test_reference_program_lowers(name):
    rec = PROGS[name]
    lf = {k: arr(v) for k, v in rec["load_files"].items()}
    P = Program(rec["ast"], rec["env"], load_files=lf)
    P._fuse_all()
    for s in P._all_steps():
        if isinstance(s, RegionStep):
            src, kname = s.region.codegen(148)
            assert kname in src and "__global__" in src
