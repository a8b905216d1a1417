"""``load`` file formats (tensorlang/compiler.py:68-162) and the names the
``--cache-layers`` facade writes, on the CPU.

The loader is checked on files written here: .npy; .npz with a ``data``
array, without one (first array), with a named array, with ``columns`` and
byte-string ``index`` metadata; .csv with and without an index column; and
the reference's errors (missing file, unknown suffix, missing array,
non-numeric CSV, shape mismatch).  A program whose ``let`` loads a file gets
that file's values as its initial tensor.

The facade writes one ``.npy`` per value into ``cache/<program>/``; every
file the reference's own executor wrote for its 106 test programs (recorded
in ``ref_programs.json``) has a counterpart among the names a program here
keeps.
"""
import numpy as np
import pytest

from conftest import arr, golden, load_backend

tl = load_backend()
from tensor_lang_b200.dataio import check_shape, load_data_file  # noqa: E402


def test_npy(tmp_path):
    a = np.arange(12, dtype=np.float64).reshape(3, 4)
    np.save(tmp_path / "a.npy", a)
    data, meta = load_data_file(str(tmp_path / "a.npy"))
    assert data.dtype == np.float32 and meta["format"] == "npy" and meta["shape"] == (3, 4)
    np.testing.assert_array_equal(data, a.astype(np.float32))


def test_npz_selection_and_metadata(tmp_path):
    x, y = np.ones((2, 3)), np.arange(6.0).reshape(2, 3)
    np.savez(tmp_path / "d.npz", other=x, data=y, columns=np.array(["a", "b", "c"]),
             index=np.array([b"r0", b"r1"]))
    data, meta = load_data_file(str(tmp_path / "d.npz"))
    np.testing.assert_array_equal(data, y)
    assert meta["array_name"] == "data" and meta["columns"] == ["a", "b", "c"]
    assert meta["index"] == ["r0", "r1"]
    data, meta = load_data_file(str(tmp_path / "d.npz"), "other")
    np.testing.assert_array_equal(data, x)
    with pytest.raises(KeyError, match="Available"):
        load_data_file(str(tmp_path / "d.npz"), "missing")
    np.savez(tmp_path / "e.npz", first=x, second=y)
    data, meta = load_data_file(str(tmp_path / "e.npz"))
    assert meta["array_name"] == "first"
    np.testing.assert_array_equal(data, x)


def test_csv(tmp_path):
    (tmp_path / "p.csv").write_text("Date,a,b\n2024-01-01,1.5,2\n2024-01-02,3,4.25\n")
    data, meta = load_data_file(str(tmp_path / "p.csv"))
    np.testing.assert_array_equal(data, np.array([[1.5, 2], [3, 4.25]], np.float32))
    assert meta["index"] == ["2024-01-01", "2024-01-02"] and meta["columns"] == ["a", "b"]
    (tmp_path / "q.csv").write_text("a,b\n1,2\n3,4\n")
    data, meta = load_data_file(str(tmp_path / "q.csv"))
    assert data.shape == (2, 2) and "index" not in meta
    (tmp_path / "r.csv").write_text("a,b\n1,x\n")
    with pytest.raises(ValueError, match="non-numeric"):
        load_data_file(str(tmp_path / "r.csv"))


def test_errors(tmp_path):
    with pytest.raises(FileNotFoundError):
        load_data_file(str(tmp_path / "nope.npy"))
    (tmp_path / "t.txt").write_text("1")
    with pytest.raises(ValueError, match="Unsupported file format"):
        load_data_file(str(tmp_path / "t.txt"))
    with pytest.raises(ValueError, match="Shape mismatch"):
        check_shape("x", "f.npy", np.zeros((2, 3), np.float32), (3, 2))


def test_program_loads_relative_to_cwd(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    v = np.random.default_rng(0).standard_normal((4, 5)).astype(np.float32)
    np.savez("in.npz", data=v)
    ast = [{"type": "let", "name": "x", "ty": {"dtype": "f32", "shape": (4, 5)},
            "expr": {"type": "load", "file_path": "in.npz"}, "requires_grad": False},
           {"type": "let", "name": "y", "ty": None, "requires_grad": False,
            "expr": {"type": "relu", "args": ["x"]}}]
    P = tl.Program(ast, None)
    np.testing.assert_array_equal(P.initial["x"], v)


def test_cache_names_cover_the_reference_cache():
    progs = golden("ref_programs.json")
    for name, rec in sorted(progs.items()):
        if rec["status"] != "ok":
            continue
        lf = {k: arr(v) for k, v in rec["load_files"].items()}
        P = tl.Program(rec["ast"], rec["env"], load_files=lf)
        P._fuse_all()
        needed = set(P.initial)
        for s in P._all_steps():
            needed.update(s.reads)
            needed.update(s.writes)
        lets = P._let_names()
        keep = {n for n in needed if not n.startswith("__") or n in lets}
        keep |= {a for a in P.alias if not a.startswith("__") or a in lets}
        keep |= {f"{g}.grad" for g in P.top_grads}
        missing = set(rec["outputs"]) - keep
        assert not missing, f"{name}: the reference's cache also holds {sorted(missing)}"
