"""``TensorCompiler(cache_layers=True).compile_and_execute(path)`` -- the
drop-in for tensorlang/compiler.py:858 -- on the GPU, for the reference's 106
test programs.

The facade parses with the reference frontend (``tensorlang.lark``,
``ast_builder``, ``type_checker``), which is the caller's code and is not
present where the GPU runs; its output for every program was recorded with
the reference (``tests/golden/ref_programs.json``), so ``parse_program`` is
replaced by a lookup of that recording.  Everything after parsing is the
facade's own: execution, ``load`` from disk (the ``load_*`` programs read the
``.npy`` files that ``basics.tl`` wrote into the cache in the same working
directory, as the reference's suite does), ``save`` and the cache layout
``cache/<path>/<name>.npy`` / ``<name>.grad.npy``.

Each program's cache is compared with the files the reference's own executor
wrote (recorded beside the AST): the same file names, and values within
rel 1e-5 (rel 1e-4 with a matmul, linear or backward), atol = rtol * max|ref|;
its ``// @EXPECTED`` block with the reference test runner's tolerance.
"""
import numpy as np
import pytest

from conftest import arr, assert_close, golden, load_backend

pytestmark = pytest.mark.gpu

PROGS = golden("ref_programs.json")
BY_FILE = {rec["file"]: rec for rec in PROGS.values()}
# basics.tl writes what the load_* programs read
ORDER = sorted(PROGS, key=lambda n: (0 if n == "basics" else 1, n))


def _heavy(ast):
    def walk(nodes):
        for n in nodes:
            if n["type"] in ("backward", "for"):
                return True
            e = n.get("expr")
            if isinstance(e, dict) and e.get("type") in ("matmul", "linear"):
                return True
        return False
    return walk(ast)


@pytest.fixture(scope="module")
def workdir(tmp_path_factory):
    return tmp_path_factory.mktemp("facade")


@pytest.mark.parametrize("name", ORDER)
def test_compile_and_execute_writes_the_reference_cache(name, workdir, monkeypatch):
    tl = load_backend()
    from tensor_lang_b200 import compiler as facade

    rec = PROGS[name]
    if rec["status"] != "ok":
        pytest.skip(f"the reference itself did not run it: {rec['status']}")
    monkeypatch.chdir(workdir)
    monkeypatch.setattr(facade, "parse_program", lambda path: (BY_FILE[path]["ast"], BY_FILE[path]["env"]))
    tc = tl.TensorCompiler(cache_layers=True)
    results = tc.compile_and_execute(rec["file"])
    cache = workdir / "cache" / rec["file"]
    rtol = 1e-4 if _heavy(rec["ast"]) else 1e-5
    for key, ref_json in rec["outputs"].items():
        f = cache / f"{key}.npy"
        assert f.exists(), f"{name}: {f.name} missing from the cache"
        got = np.load(f)
        ref = arr(ref_json)
        if ref.size == 1 and got.size == 1:
            got, ref = got.reshape(1), ref.reshape(1)
        assert_close(got, ref, rtol, f"{name}/{key}")
    for key, exp in rec["expected"].items():
        got = np.asarray(results[key], np.float64)
        e = np.asarray(exp, np.float64)
        assert np.allclose(got.reshape(e.shape) if got.size == e.size else got, e,
                           rtol=1e-5, atol=1e-8), (name, key)
