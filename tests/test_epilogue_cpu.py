"""The GEMM epilogue fusion pass (tensor-lang_b200/epilogue.py) on lowered
programs, on the CPU: which rewrites apply, and which are blocked.

The numerics of the rewritten programs are checked on the GPU
(test_gpu_epilogue.py: bit-identical to the unfused program)."""
from conftest import load_backend

load_backend()  # registers the package as tensor_lang_b200


def _mlp3(fetch, **kw):
    tl = load_backend()
    pr = tl.programs
    ast = pr.mlp3_train(B=64, I=32, H=48, C=10, epochs=2)
    return tl.Program(ast, None, feeds=pr.mlp3_inputs(B=64, I=32, H=48, C=10), fetch=fetch, **kw)


def _steps(P):
    from tensor_lang_b200.epilogue import _flat
    return [s for _, s in _flat(P)]


def _opcodes(P):
    return [getattr(s, "opcode", None) for s in _steps(P)]


def test_mlp3_relu_and_mask_fold_into_gemms():
    from tensor_lang_b200.epilogue import fuse_gemm_epilogues
    P = _mlp3(["loss", "W3"])
    assert fuse_gemm_epilogues(P) == 6
    ops = _opcodes(P)
    assert "relu" not in ops and "relu_mask" not in ops
    steps = _steps(P)
    masked = [s for s in steps if getattr(s, "fname", "") == "tl_gemm_masked"]
    assert sorted(s.writes[0] for s in masked) == ["h1_grad", "h2_grad"]
    assert sorted(s.args[14][1] for s in masked) == ["a1", "a2"]   # masks: the relu outputs
    relu_gemms = [s for s in steps if getattr(s, "fname", "") == "tl_gemm" and s.args[13] == ("int", 1)]
    assert sorted(s.writes[0] for s in relu_gemms) == ["a1", "a2"]
    names = {n for s in steps for n in s.reads + s.writes}
    assert "h1" not in names and "h2" not in names      # pre-activations never materialised


def test_nothing_fuses_when_every_tensor_is_fetched():
    from tensor_lang_b200.epilogue import fuse_gemm_epilogues
    P = _mlp3(None)
    assert fuse_gemm_epilogues(P) == 0
    assert _opcodes(P).count("relu") == 2


def test_fetched_pre_activation_keeps_its_relu():
    from tensor_lang_b200.epilogue import fuse_gemm_epilogues
    P = _mlp3(["loss", "h1"])
    fuse_gemm_epilogues(P)
    steps = _steps(P)
    assert any(getattr(s, "opcode", None) == "relu" and s.reads == ["h1"] for s in steps)
    assert any("h1" in s.writes for s in steps)
    # the second layer still folds
    assert not any(getattr(s, "opcode", None) == "relu" and s.reads == ["h2"] for s in steps)


def test_second_reader_blocks_relu_fold():
    tl = load_backend()
    pr = tl.programs
    L, C, F = pr._let, pr._call, pr._fill
    ast = [L("x", F((8, 16)), (8, 16)), L("W", F((16, 32)), (16, 32)), L("b", F((32,)), (32,)),
           L("h", C("linear", "x", "W", "b")), L("a", C("relu", "h")),
           L("s", {"type": "sum", "tensor": "h", "axis": 1})]
    from tensor_lang_b200.epilogue import fuse_gemm_epilogues
    P = tl.Program(ast, None, fetch=["a", "s"])
    assert fuse_gemm_epilogues(P) == 0


def _masked_gemm(s) -> bool:
    """A GEMM carrying the relu-mask epilogue (with or without prepared pairs)."""
    f = getattr(s, "fname", "")
    return f == "tl_gemm_masked" or (f == "tl_gemm_pairs" and s.args[16][0] == "ptr")


def test_engine_runs_the_pass_only_with_fusion_on():
    for fuse_ops, masked in ((False, 0), (True, 2)):
        P = _mlp3(["loss", "W3"], fuse_ops=fuse_ops)
        P._fuse_all()
        assert sum(_masked_gemm(s) for s in _steps(P)) == masked


def test_operand_pairs_planned_once_per_value():
    """pairs.py: each GEMM operand value gets one pair step (both layouts from
    one read) right after its producer; the loop-invariant input's pairs are
    hoisted out of the per-iteration graph; weights rebound in place keep the
    per-call pre-pass."""
    tl = load_backend()
    pr = tl.programs
    kw = dict(B=4096, I=1024, H=4096, C=10)
    P = tl.Program(pr.mlp3_train(epochs=2, **kw), None, fetch=["loss", "W3"])
    P._fuse_all()
    loop = P.loops[0]
    assert [s.label for s in loop.hoisted] == ["pairs:x"]
    assert sorted(loop.hoisted[0].writes) == ["__pair_x_hoist_k0", "__pair_x_hoist_m0"]
    body = loop.body()
    labels = [s.label for s in body]
    prep = {s.label.split("+colsum")[0]: s for s in body
            if getattr(s, "fname", "").startswith("tl_gemm_pair_prepare")}
    labels = [lab.split("+colsum")[0] for lab in labels]
    assert sorted(prep) == ["pairs:a1", "pairs:h1_grad", "pairs:h2_grad"]
    # both layouts from one read where two roles use the value
    pair_writes = {k: [w for w in st.writes if w.startswith("__pair_")] for k, st in prep.items()}
    assert len(pair_writes["pairs:a1"]) == 2 and len(pair_writes["pairs:h2_grad"]) == 2
    # each pair step directly follows the step that writes its tensor
    for lab, st in prep.items():
        x = lab.split(":", 1)[1]
        i = labels.index(lab)
        assert x in body[i - 1].writes, (lab, labels[i - 1])
    users = [s for s in body if getattr(s, "fname", "") == "tl_gemm_pairs"]
    assert len(users) == 5   # both forward GEMMs, dW2, dX1, dW1 (the 10-wide head has none)
    for s in users:
        for name in (s.args[7][1] if s.args[7][0] == "ptr" else None,
                     s.args[10][1] if s.args[10][0] == "ptr" else None):
            assert name is None or name.startswith("__pair_")
    assert not any("W2" in w for s in prep.values() for w in s.writes)


def test_bias_sums_fold_into_pair_steps():
    """pairs.py fuse_bias_colsums: db2 and db1 (the row sums of h2_grad and
    h1_grad) are written by the pair steps of those gradients, one read of
    each instead of two; a1's pair step has no sum to take; with
    fuse_colsum=False the sums keep their own steps."""
    tl = load_backend()
    pr = tl.programs
    kw = dict(B=4096, I=1024, H=4096, C=10)
    P = tl.Program(pr.mlp3_train(epochs=2, **kw), None, fetch=["loss", "W3"])
    P._fuse_all()
    body = P.loops[0].body()
    folded = {s.args[8][1]: s for s in body
              if getattr(s, "fname", "") == "tl_gemm_pair_prepare_colsum"}
    assert sorted(folded) == ["b1_grad", "b2_grad"]
    assert folded["b2_grad"].args[0] == ("ptr", "h2_grad")
    assert folded["b1_grad"].args[0] == ("ptr", "h1_grad")
    for out, st in folded.items():
        # partial sums in a buffer of their own, not the program's scratch
        assert out in st.writes and st.args[9:] == [("ptr", "__colsum_partials"),
                                                    ("bytes", "__colsum_partials")]
    assert P.shapes["__colsum_partials"][0] > 0
    sums = [s for s in body if getattr(s, "fname", "") == "tl_reduce_cols"]
    assert [s.args[2][1] for s in sums] == ["b3_grad"]   # the head's db: no pair step
    # the folded sum is written before every reader of it
    names = [s.label for s in body]
    for out, st in folded.items():
        i = body.index(st)
        assert not any(out in b.reads for b in body[:i])
    Q = tl.Program(pr.mlp3_train(epochs=2, **kw), None, fetch=["loss", "W3"], fuse_colsum=False)
    Q._fuse_all()
    qb = Q.loops[0].body()
    assert not any(getattr(s, "fname", "") == "tl_gemm_pair_prepare_colsum" for s in qb)
    assert sorted(s.args[2][1] for s in qb if getattr(s, "fname", "") == "tl_reduce_cols") == [
        "b1_grad", "b2_grad", "b3_grad"]
    assert names  # labels computed


def test_no_operand_pairs_under_the_three_tf32_scheme():
    """The three-TF32 scheme reads no pair matrices, so nothing is planned."""
    import ctypes
    tl = load_backend()
    L = tl.runtime.lib()
    prev = ctypes.c_int(-1)
    assert L.tl_gemm_set_scheme(0, ctypes.byref(prev)) == 0
    try:
        pr = tl.programs
        kw = dict(B=4096, I=1024, H=4096, C=10)
        P = tl.Program(pr.mlp3_train(epochs=2, **kw), None, fetch=["loss", "W3"])
        P._fuse_all()
        loop = P.loops[0]
        assert not loop.hoisted
        names = [getattr(s, "fname", "") for s in loop.body()]
        assert "tl_gemm_pair_prepare" not in names and "tl_gemm_pairs" not in names
    finally:
        L.tl_gemm_set_scheme(prev.value, None)
    assert prev.value == 2  # BF16X3 is the default


def test_bias_sum_fold_needs_an_untouched_span():
    """fuse_bias_colsums folds a row sum into the pair step of the same tensor
    only when nothing between them writes the tensor or touches the sum, the
    sum is a plain SUM over the tensor's full shape, and cols <= 8192."""
    tl = load_backend()
    from tensor_lang_b200 import pairs
    from tensor_lang_b200.steps import LibCall
    rt = tl.runtime

    class _P:
        alias: dict = {}

        def __init__(self):
            self.shapes = {}

    def pair(rows=512, cols=256):
        return LibCall("pairs:g", "tl_gemm_pair_prepare",
                       [("ptr", "g"), ("int", cols), ("int", rows), ("int", cols),
                        ("ptr", "__pk"), ("int", 0), ("ptr", "__pm"), ("int", 1)],
                       ["g"], ["__pk", "__pm"])

    def rsum(op=rt.RED_SUM, rows=512, cols=256, src="g"):
        return LibCall("db:b", "tl_reduce_cols",
                       [("int", op), ("ptr", src), ("ptr", "b"), ("int", rows), ("int", cols),
                        ("scratch",)], [src], ["b"])

    def other(reads=(), writes=()):
        return LibCall("x", "tl_something", [], list(reads), list(writes))

    cases = [
        ([pair(), other(), rsum()], 1),                         # folds
        ([pair(), other(reads=["b"]), rsum()], 0),              # the sum is read in between
        ([pair(), other(writes=["b"]), rsum()], 0),             # ... or written
        ([pair(), other(writes=["g"]), rsum()], 0),             # the tensor changes in between
        ([pair(), rsum(op=rt.RED_MAX)], 0),                     # not a sum
        ([pair(), rsum(rows=256)], 0),                          # another shape
        ([pair(rows=64, cols=8200), rsum(rows=64, cols=8200)], 0),  # too wide
    ]
    for lst, want in cases:
        P = _P()
        got = pairs._fold_list(P, lst)
        assert got == want, [s.label for s in lst]
        if want:
            assert [s.fname for s in lst] == ["tl_gemm_pair_prepare_colsum", "tl_something"]
            assert "b" in lst[0].writes and P.shapes[pairs.PARTIALS][0] > 0
