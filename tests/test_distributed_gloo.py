"""Multi-rank host logic of batch-sharded inference, run as 2 gloo ranks on
CPU: row sharding, the one-time weight broadcast, and the output gather.
Per-sample independence (the basis of sharding) is checked with the oracle:
the gathered shard outputs equal the full-batch output."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from pyflame_b200.distributed import shard_range, split_even


def test_shard_range_partitions():
    for n in (0, 1, 7, 8192, 8193):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and b >= a
            assert max(split_even(n, world)) - min(split_even(n, world)) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        import sys
        from pathlib import Path
        sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
        import torch
        import torch.distributed as dist

        import pyflame_b200 as pf
        from oracle import oracle as O
        from pyflame_b200 import distributed as D
        D.init("gloo", timeout_s=60)
        rng = np.random.default_rng(42)
        rows, cols = 37, 64
        x = rng.standard_normal((rows, cols)).astype(np.float32)
        w = (rng.standard_normal((16, cols)) * 0.1).astype(np.float32)
        # weights: only rank 0 holds the real values before the broadcast
        local_w = w if rank == 0 else np.zeros_like(w)
        bw = D.broadcast_weights({7: local_w})
        assert np.array_equal(bw[7].numpy(), w)
        # each rank evaluates its shard of Linear -> LayerNorm-free softmax graph with the oracle
        xs = D.shard_batch(x, rank, world)
        pf.reset_graph()
        lin = pf.nn.Linear(cols, 16)
        lin.set_parameter("weight", bw[7].numpy())
        out = pf.softmax(pf.relu(lin(pf.tensor(xs))), -1)
        ys = O.run(out.graph(), [out.node().id()])[out.node().id()]
        full = D.gather_rows(torch.from_numpy(ys), world)
        if rank == 0:
            pf.reset_graph()
            lin2 = pf.nn.Linear(cols, 16)
            lin2.set_parameter("weight", w)
            ref = pf.softmax(pf.relu(lin2(pf.tensor(x))), -1)
            yr = O.run(ref.graph(), [ref.node().id()])[ref.node().id()]
            assert full.shape == (rows, 16)
            assert np.array_equal(full.numpy(), yr), "sharded result differs from the full batch"
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, traceback.format_exc()))


def test_two_rank_broadcast_shard_gather():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results


def _failing_worker(rank, world, port, fail_at, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        import sys
        from pathlib import Path
        sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
        import pyflame_b200 as pf
        from oracle import oracle as O
        from pyflame_b200 import distributed as D
        rng = np.random.default_rng(7)
        x = rng.standard_normal((10, 12)).astype(np.float32)
        w = rng.standard_normal((5, 12)).astype(np.float32)
        released = []

        def evaluate(weights, shard):
            pf.reset_graph()
            lin = pf.nn.Linear(12, 5)
            lin.set_parameter("weight", weights[3])
            out = pf.relu(lin(pf.tensor(shard)))
            return O.run(out.graph(), [out.node().id()])[out.node().id()]

        r = D.run_sharded(evaluate, x, {3: w if rank == 0 else np.zeros_like(w)}, backend="gloo", timeout_s=4,
                          release=lambda: released.append(True), fail_at=fail_at if rank == 1 else "")
        ok_full = None
        if r.success and rank == 0:
            ok_full = bool(np.array_equal(r.output, evaluate({3: w}, x)))
        q.put((rank, r.success, r.error_message, bool(released), ok_full))
    except Exception:  # noqa: BLE001
        import traceback
        q.put((rank, None, traceback.format_exc(), False, None))


@pytest.mark.parametrize("fail_at", ["", "init", "broadcast", "evaluate"])
def test_sharded_run_reports_a_failed_rank(fail_at):
    """A rank that never joins, fails before the broadcast or fails while
    evaluating makes every rank return success=False (never hang, never
    raise) and release its executor; with no failure the gathered output
    equals the full batch."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, fail_at, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, ok, msg, released, full = q.get(timeout=120)
        res[rank] = (ok, msg, released, full)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    if not fail_at:
        assert res[0][0] and res[1][0], res
        assert res[0][3] is True
        return
    assert res[1][0] is False and "injected" in res[1][1], res
    assert res[0][0] is False and res[0][1], res
    assert res[0][2] and res[1][2], "executor memory released on every failing rank"


def test_serving_cache_and_stats_host_logic():
    """The engine's host-side pieces: LRU eviction order and the statistics
    PyFlame's serving API reports (inference.py:36-138)."""
    from pyflame_b200.serving import InferenceStats, LRUCache
    c = LRUCache(2)
    c.put(1, "a")
    c.put(2, "b")
    assert c.get(1) == "a"  # 1 becomes most recent
    c.put(3, "c")           # evicts 2
    assert c.get(2) is None and c.get(1) == "a" and c.get(3) == "c" and len(c) == 2
    s = InferenceStats(total_inferences=4, total_time_ms=8.0, cache_hits=1, cache_misses=3)
    assert s.average_time_ms == 2.0 and s.throughput == 500.0 and s.cache_hit_rate == 0.25
    assert s.to_dict()["throughput_per_second"] == 500.0
