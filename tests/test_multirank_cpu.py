"""Host-side logic of the document-sharded (N > 1) path, run as 2 gloo ranks on CPU.

Covers what does not need a GPU: shard placement (contiguous, disjoint,
8192-aligned for MVS), that the bench's seeded data is identical under any
sharding, the unique-id broadcast the ranks use to build their communicator,
and that per-rank integer fixed-point histograms sum to the single-rank ones
(the property that makes trees independent of the GPU count).

The library's own multi-rank decisions run here too, through the C ABI on
the host (the same code the session and its kernels run): each gloo rank
takes its feature slice (cbgpu_rank_feature_slice, also for F not divisible
by the world size and for ranks that own only padding), all-gathers its
slice winner record, and picks the global split and the next level's build
side (cbgpu_rank_select_split); every rank must agree, and the result must be
the single-device first-wins scan (tree.rs:355-366).  The first-tree MVS
lambda sum crosses the ranks in rank order (cbgpu_rank_mvs_partial) and must
be bit-identical to one rank's sum over all rows.
"""
import ctypes as C
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


# ---- the library's multi-rank decisions, on the host --------------------------

NO_KEY = 0x7FFFFFFF


def _scores(F, B, seed):
    """Candidate scores [F][B] with ties across features (so across ranks), a
    -inf and a feature without candidates."""
    rs = np.random.RandomState(seed)
    sc = np.round(rs.standard_normal((F, B)), 1)  # coarse values: many exact ties
    top = sc.max()
    sc[F - 1, 0] = top  # the top score again in the last feature
    sc[F // 2, B // 2] = -np.inf
    counts = np.full(F, B)
    if F > 2:
        counts[1] = 0  # a feature with no borders
    return sc, counts


def _slice_record(sc, counts, f0, fs, level, seed):
    """This rank's slice winner, first max in (feature, border) order, and its
    per-parent (false, true) child weights."""
    best, key = -np.inf, NO_KEY
    for f in range(f0, min(f0 + fs, sc.shape[0])):
        for b in range(counts[f]):
            if sc[f, b] > best:
                best, key = sc[f, b], (f << 8) | b
    rs = np.random.RandomState(seed + key % 977)
    w = rs.randint(0, 1 << 40, size=(1 << level, 2)).astype(np.uint64)
    w[0] = [5, 5]  # equal children: the true child is built
    rec = np.zeros(2 + 2 * (1 << level), dtype=np.uint64)
    rec[0] = np.array([best], dtype=np.float64).view(np.uint64)[0]
    rec[1] = key
    rec[2:] = w.reshape(-1)
    return rec


def _decide_worker(rank, world, port, q, F, B, level, n_total):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch
        import catboost_rs_b200 as cb
        L = cb.load_library()
        f0, fs = C.c_int32(), C.c_int32()
        assert L.cbgpu_rank_feature_slice(F, world, rank, C.byref(f0), C.byref(fs)) == 0
        sc, counts = _scores(F, B, 3)
        rec = _slice_record(sc, counts, f0.value, fs.value, level, 9)
        stride = rec.size
        mine = torch.from_numpy(rec.view(np.int64).copy())
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        all_best = np.concatenate([p.numpy() for p in parts]).view(np.uint64)
        feat, b, score, wr = C.c_int32(), C.c_int32(), C.c_double(), C.c_int32()
        side = np.zeros(1 << level, dtype=np.uint8)
        assert L.cbgpu_rank_select_split(level, world, stride, all_best.ctypes.data, C.byref(feat), C.byref(b),
                                         C.byref(score), C.byref(wr), side.ctypes.data) == 0
        # the first-tree MVS lambda chain in rank order
        rs = np.random.RandomState(21)
        target = rs.standard_normal(n_total)
        approx = rs.standard_normal(n_total) * 0.3
        weight = rs.uniform(0.5, 2.0, n_total)
        per = -(-n_total // world)
        lo, hi = min(n_total, rank * per), min(n_total, (rank + 1) * per)
        acc = torch.zeros(1, dtype=torch.float64)
        if rank > 0:
            dist.recv(acc, src=rank - 1)
        out = C.c_double()
        assert L.cbgpu_rank_mvs_partial(1, hi - lo, approx[lo:].ctypes.data, 0.0, target[lo:].ctypes.data,
                                        weight[lo:].ctypes.data, float(acc.item()), C.byref(out)) == 0
        acc[0] = out.value
        if rank + 1 < world:
            dist.send(acc, dst=rank + 1)
        dist.broadcast(acc, src=world - 1)
        res = [None] * world
        dist.all_gather_object(res, (f0.value, fs.value, feat.value, b.value, score.value, wr.value,
                                     side.tolist(), float(acc.item())))
        if rank == 0:
            q.put(res)
    except BaseException as e:
        q.put(repr(e))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,F,B,level", [(2, 7, 16, 3), (3, 7, 9, 0), (2, 1, 5, 2), (4, 10, 33, 5)])
def test_ranks_agree_on_split_build_side_and_mvs_lambda(world, F, B, level):
    import catboost_rs_b200 as cb
    L = cb.load_library()
    n_total = 12345
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_decide_worker, args=(r, world, port, q, F, B, level, n_total))
             for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=240)
    assert not isinstance(res, str), res
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # slices: contiguous, ceil(F / world) wide, covering every feature
    fs = -(-F // world)
    assert [(r[0], r[1]) for r in res] == [(k * fs, fs) for k in range(world)]
    # every rank took the same decision ...
    assert len({tuple(map(str, r[2:])) for r in res}) == 1
    # ... the single-device first-wins scan over (feature, border)
    sc, counts = _scores(F, B, 3)
    best, bf, bb = -np.inf, -1, -1
    for f in range(F):
        for b in range(counts[f]):
            if sc[f, b] > best:
                best, bf, bb = sc[f, b], f, b
    feat, b, score, wr, side = res[0][2:7]
    assert (feat, b, score) == (bf, bb, best)
    assert wr == bf // fs
    rec = _slice_record(sc, counts, wr * fs, fs, level, 9)
    w = rec[2:].reshape(-1, 2)
    assert side == [1 if w[q_, 1] <= w[q_, 0] else 0 for q_ in range(1 << level)]
    assert side[0] == 1
    # the MVS chain: bit-identical to one rank's sequential sum over all rows
    rs = np.random.RandomState(21)
    target = rs.standard_normal(n_total)
    approx = rs.standard_normal(n_total) * 0.3
    weight = rs.uniform(0.5, 2.0, n_total)
    one = C.c_double()
    assert L.cbgpu_rank_mvs_partial(1, n_total, approx.ctypes.data, 0.0, target.ctypes.data, weight.ctypes.data,
                                    0.0, C.byref(one)) == 0
    assert all(r[7] == one.value for r in res)


def test_select_split_without_candidates():
    import catboost_rs_b200 as cb
    L = cb.load_library()
    recs = np.zeros((2, 6), dtype=np.uint64)
    recs[:, 0] = np.array([-np.inf, -np.inf]).view(np.uint64)
    recs[:, 1] = NO_KEY
    feat, b, score, wr = C.c_int32(), C.c_int32(), C.c_double(), C.c_int32()
    side = np.zeros(2, dtype=np.uint8)
    assert L.cbgpu_rank_select_split(1, 2, 6, recs.ctypes.data, C.byref(feat), C.byref(b), C.byref(score),
                                     C.byref(wr), side.ctypes.data) == 0
    assert (feat.value, b.value, wr.value) == (-1, -1, -1) and score.value == -np.inf
    assert side.tolist() == [1, 1]
