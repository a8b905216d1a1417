"""Host-side logic of the data-parallel path, on CPU with 2 processes.

* the TCP rendezvous (broadcast, gather, barrier) between 2 ranks, and its
  failure detection: a rank that never arrives makes the other fail within
  the timeout instead of hanging;
* batch sharding: which tensors carry the batch axis, their per-rank shapes,
  and the global divisors of the loss VJPs;
* the identity the design rests on, with torch.distributed (gloo): each rank
  computes its shard's gradients with the global-batch divisor, the
  all-reduced sum equals the full-batch gradient (float64 oracle).
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from conftest import load_backend


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rdv_worker(rank, world, port, q):
    tl = load_backend()
    from tensor_lang_b200 import dp
    r = dp.Rendezvous(rank, world, "127.0.0.1", port, timeout=20)
    got = r.bcast({"from": 0, "v": [1, 2, 3]} if rank == 0 else None)
    g = r.gather(rank * 10)
    r.barrier()
    q.put((rank, got, g))
    r.close()


def test_rendezvous_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rdv_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (got, g)) for r, got, g in (q.get(timeout=60) for _ in ps))
    for p in ps:
        p.join(timeout=30)
        assert p.exitcode == 0
    assert res[0][0] == res[1][0] == {"from": 0, "v": [1, 2, 3]}
    assert res[0][1] == [0, 10] and res[1][1] is None


def _lonely_root(port, q):
    load_backend()
    from tensor_lang_b200 import dp
    try:
        dp.Rendezvous(0, 2, "127.0.0.1", port, timeout=2)
        q.put("no error")
    except (TimeoutError, socket.timeout, OSError) as e:
        q.put(type(e).__name__)


def test_rendezvous_missing_rank_times_out():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_root, args=(_free_port(), q))
    p.start()
    res = q.get(timeout=60)
    p.join(timeout=30)
    assert res != "no error"


def test_sharding_and_divisors():
    tl = load_backend()
    from tensor_lang_b200 import dp
    from tensor_lang_b200.shapes import complete_env
    ast = tl.programs.mlp3_train(B=1024, I=32, H=64, C=10, epochs=2)
    derived = dp.batch_derived(ast, ["x", "t"])
    assert {"x", "t", "h1", "a1", "h2", "a2", "z", "p"} <= derived
    assert not derived & {"W1", "b1", "W2", "b2", "W3", "b3", "loss", "W1_new", "b3_step"}
    g = complete_env(ast, {})
    local = dp.shard_shapes(g, derived, 4)
    assert local["x"] == (256, 32) and local["h2"] == (256, 64) and local["h2_grad"] == (256, 64)
    assert local["W2"] == (64, 64) and local["W2_grad"] == (64, 64)
    assert dp.loss_divisors(ast, g, derived) == {("ce", "loss"): 1024.0}
    with pytest.raises(ValueError):
        dp.shard_shapes(g, derived, 3)


def _grad_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from oracle import OracleProgram
    tl = load_backend()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    kw = dict(B=64, I=16, H=32, C=10)
    B, b = kw["B"], kw["B"] // world
    ast = tl.programs.mlp2_step(B=b, I=kw["I"], H=kw["H"], C=kw["C"])
    full = tl.programs.mlp2_inputs(B=B, I=kw["I"], H=kw["H"], C=kw["C"], seed=9)
    feeds = dict(full, x=full["x"][rank * b:(rank + 1) * b], t=full["t"][rank * b:(rank + 1) * b])
    env = {k: {"shape": v} for k, v in tl.shapes.complete_env(ast, {}).items()}
    out = OracleProgram(ast, env, dtype=np.float64, feeds=feeds).run()
    names = ["W1_grad", "b1_grad", "W2_grad", "b2_grad"]
    # the shard's CE VJP divided by b; the global divisor is B
    mine = {n: torch.tensor(out[n] * (b / B)) for n in names}
    for n in names:
        dist.all_reduce(mine[n])
    q.put((rank, {n: mine[n].numpy() for n in names}))
    dist.destroy_process_group()


def test_sharded_gradient_sum_equals_full_batch():
    from oracle import OracleProgram
    tl = load_backend()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_grad_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    kw = dict(B=64, I=16, H=32, C=10)
    ast = tl.programs.mlp2_step(**kw)
    feeds = tl.programs.mlp2_inputs(seed=9, **kw)
    env = {k: {"shape": v} for k, v in tl.shapes.complete_env(ast, {}).items()}
    ref = OracleProgram(ast, env, dtype=np.float64, feeds=feeds).run()
    for n, v in res[0].items():
        np.testing.assert_allclose(v, ref[n], rtol=1e-10, atol=1e-12, err_msg=n)
        np.testing.assert_array_equal(v, res[1][n])


def test_bucket_plan_overlaps_backward():
    """Gradient all-reduces are bucketed in the order backward finalises the
    gradients; a bucket is issued right after its last gradient is written,
    the tail is a bucket of its own at the end, and a join closes the list."""
    from conftest import load_backend
    tl = load_backend()
    from tensor_lang_b200 import dp
    from tensor_lang_b200.shapes import numel
    pr = tl.programs
    kw = dict(B=64, I=1024, H=4096, C=10)
    P = tl.Program(pr.mlp3_train(epochs=1, **kw), None, fetch=["loss"])
    bw = P.loops[0].bw
    grads = ["W1_grad", "b1_grad", "W2_grad", "b2_grad", "W3_grad", "b3_grad"]

    class _Comm:  # only identity matters to the planner
        handle = stream = None
    single, _ = dp.plan_buckets(list(bw), grads, P.shapes, _Comm(), None)
    ar = [s for s in single if isinstance(s, dp.AllReduceBucket)]
    assert len(ar) == 1 and sorted(ar[0].names) == sorted(grads)   # default: one, at the end
    assert single.index(ar[0]) == len(single) - 2 and isinstance(single[-1], dp.AllReduceJoin)
    steps, arena = dp.plan_buckets(list(bw), grads, P.shapes, _Comm(), dp.BUCKET_BYTES)
    labels = [s.label for s in steps]
    buckets = [s for s in steps if isinstance(s, dp.AllReduceBucket)]
    assert isinstance(steps[-1], dp.AllReduceJoin)
    assert sorted(arena) == sorted(grads) and len(arena) == len(grads)
    assert [n for b in buckets for n in b.names] == arena
    # W2 (64 MB) closes the first bucket right after its dW step, before dW1
    first = buckets[0]
    assert "W2_grad" in first.names and "W1_grad" not in first.names
    i = labels.index(first.label)
    assert labels[i - 1].startswith("dW:W2_grad")
    assert any(l.startswith("dW:W1_grad") for l in labels[i + 1:])
    # nothing after a bucket touches its gradients before the join
    for b in buckets:
        j = steps.index(b)
        for s in steps[j + 1:-1]:
            if isinstance(s, dp.AllReduceBucket):
                continue
            assert not (set(b.names) & (set(s.reads) | set(s.writes))), (b.label, s.label)
    assert sum(4 * numel(P.shapes[n]) for n in first.names) >= dp.BUCKET_BYTES
    # the last bucket is the tail, issued right before the join
    assert steps.index(buckets[-1]) == len(steps) - 2
    # a 64 MB bucket: W2 closes it, the rest (b2, W1, b1) is the tail
    steps64, _ = dp.plan_buckets(list(bw), grads, P.shapes, _Comm(), 64 << 20)
    b64 = [s for s in steps64 if isinstance(s, dp.AllReduceBucket)]
    assert len(b64) == 2 and "W2_grad" in b64[0].names
    assert sorted(b64[1].names) == ["W1_grad", "b1_grad", "b2_grad"]
    assert steps64.index(b64[1]) == len(steps64) - 2
    assert steps64.index(b64[0]) < len(steps64) - 3


def test_only_parameter_gradients_are_all_reduced():
    """The gradient arena of the training loop holds exactly the six parameter
    gradients, 21,020,682 floats (84 MB): the zero-filled gradients of the
    rebound W_new / b_new values and the loss seed are the same on every rank
    and are neither packed nor all-reduced."""
    tl = load_backend()
    from tensor_lang_b200 import dp
    from tensor_lang_b200.shapes import numel
    pr = tl.programs

    class _Comm:
        world, rank, handle, stream = 2, 0, None, None
    kw = dict(B=512, I=1024, H=4096, C=10)
    ast = pr.mlp3_train(epochs=1, **kw)
    D = dp.DataParallelProgram(ast, None, _Comm(), device=0,
                               feeds=pr.mlp3_inputs(rows=(0, 256), **kw), fetch=["loss", "W3"])
    P = D.program
    assert sorted(D.replicated_grads) == sorted(
        ["W1_grad", "b1_grad", "W2_grad", "b2_grad", "W3_grad", "b3_grad"])
    assert sum(numel(P.shapes[n]) for n in P.arena_names) == 21_020_682
    P._fuse_all()
    ar = [s for s in P._all_steps() if isinstance(s, dp.AllReduceBucket)]
    # default 64 MiB buckets: W3, b3 and W2 (after dW2), then b2, W1 and b1
    assert len(ar) == 2 and sorted(n for b in ar for n in b.names) == sorted(D.replicated_grads)
    assert [n for b in ar for n in b.names] == P.arena_names
