"""Host-side logic of the document-sharded (N > 1) path, run as 2 gloo ranks on CPU.

Covers what does not need a GPU: shard placement (contiguous, disjoint,
8192-aligned for MVS), that the bench's seeded data is identical under any
sharding, the unique-id broadcast the ranks use to build their communicator,
and that per-rank integer fixed-point histograms sum to the single-rank ones
(the property that makes trees independent of the GPU count).
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n_total, q):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _work(rank, world, n_total, q)
    except BaseException as e:  # surface worker failures instead of a queue timeout
        q.put(repr(e))
        raise
    finally:
        dist.destroy_process_group()


def _work(rank, world, n_total, q):
    if True:
        import bench
        import oracle
        off, n = bench.shard_bounds(n_total, world, rank)
        X, y = bench.make_shard(off, n, 6, 11)
        # the unique-id broadcast, as bench.py does it
        obj = [bytes(range(128)) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        # per-rank exact fixed-point level-0 histogram of this shard
        borders = bench.make_borders(6, 16, 11)
        bins = oracle.quantize(X, borders)
        g = np.sin(np.arange(off, off + n) * 0.37)
        scale = 2.0 ** 30
        qg = np.rint(g * scale).astype(np.int64)
        B = max(len(b) for b in borders) + 1
        hist = np.zeros((6, B), dtype=np.int64)
        for f in range(6):
            np.add.at(hist[f], bins[f], qg)
        gathered = [None] * world
        dist.all_gather_object(gathered, (off, n, X, y, obj[0], hist))
        if rank == 0:
            q.put(gathered)


@pytest.mark.parametrize("n_total", [20000, 8192 * 3 + 5])
def test_two_rank_sharding_and_exact_histogram_sum(n_total):
    import bench
    import oracle
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_total, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=240)
    assert not isinstance(res, str), res
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    offs = [r[0] for r in res]
    ns = [r[1] for r in res]
    assert offs[0] == 0 and offs[1] == ns[0] and sum(ns) == n_total
    assert offs[1] % 8192 == 0
    X = np.concatenate([r[2] for r in res], axis=1)
    y = np.concatenate([r[3] for r in res])
    X1, y1 = bench.make_shard(0, n_total, 6, 11)
    np.testing.assert_array_equal(X, X1)
    np.testing.assert_array_equal(y, y1)
    assert all(r[4] == bytes(range(128)) for r in res)
    # integer sums: rank histograms add up to the single-rank histogram exactly
    borders = bench.make_borders(6, 16, 11)
    bins = oracle.quantize(X1, borders)
    g = np.sin(np.arange(n_total) * 0.37)
    qg = np.rint(g * 2.0 ** 30).astype(np.int64)
    B = max(len(b) for b in borders) + 1
    full = np.zeros((6, B), dtype=np.int64)
    for f in range(6):
        np.add.at(full[f], bins[f], qg)
    np.testing.assert_array_equal(res[0][5] + res[1][5], full)


def test_shard_bounds_cover_rows_aligned():
    import bench
    for n in (1, 8191, 8192, 10_000_000, 50_000_000):
        for w in (1, 2, 4, 8):
            got = [bench.shard_bounds(n, w, r) for r in range(w)]
            assert sum(c for _, c in got) == n
            pos = 0
            for off, c in got:
                assert off == pos or c == 0
                if c:
                    assert off % 8192 == 0
                pos = off + c if c else pos
