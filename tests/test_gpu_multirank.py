"""Document sharding across GPUs: N ranks (one process per GPU, the library's
own NCCL communicator) must grow the same trees as one GPU.  Histograms, leaf
sums and scales are exact integer reductions, so splits and leaf values are
bit-identical and every rank's approximant equals the matching slice of the
single-GPU one.  Needs >= 2 GPUs; skipped otherwise.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu


def _ngpus():
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


def _rank_fit(rank, world, uid_q, out_q, case):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    try:
        import catboost_rs_b200 as cb
        from synth import make_dataset
        X, y, borders = make_dataset(case["n"], case["F"], seed=case["seed"], nan_frac=0.05,
                                     loss=case["loss"], border_count=32, uniform_half=True)
        n = X.shape[0]
        per = -(-n // world)
        per = -(-per // 8192) * 8192
        off = min(n, rank * per)
        cnt = min(n, off + per) - off
        if rank == 0:
            uid = cb.nccl_unique_id()
            for _ in range(world - 1):
                uid_q.put(uid)
        else:
            uid = uid_q.get(timeout=120)
        fp = cb.FitParams(loss=case["loss"], depth=case["depth"], iterations=case["it"],
                          score_function="Cosine", bootstrap_type=case["boot"], subsample=0.7,
                          random_seed=5, boost_from_average=case["loss"] == "RMSE")
        cols = [np.ascontiguousarray(X[off:off + cnt, f]) for f in range(X.shape[1])]
        bias = cb.starting_approx(fp, y)  # the global bias, as cb-train computes it
        m = cb.fit(cols, borders, y[off:off + cnt], fp, staged=True, device=rank,
                   placement=dict(rank=rank, world_size=world, row_offset=off, n_total=n,
                                  nccl_unique_id=uid), bias=bias)
        out_q.put((rank, off, cnt, m.split_feature, m.split_bin, m.leaf_values, m.staged))
    except BaseException as e:
        out_q.put((rank, repr(e)))
        raise


CASES = [
    dict(n=50000, F=20, depth=6, it=4, loss="Logloss", boot="Bayesian", seed=1),
    dict(n=41000, F=12, depth=5, it=4, loss="RMSE", boot="MVS", seed=2),
    dict(n=30000, F=16, depth=7, it=3, loss="RMSE", boot="Bernoulli", seed=3),
]


@pytest.mark.skipif(_ngpus() < 2, reason="needs >= 2 GPUs")
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c['loss']}-{c['boot']}")
def test_sharded_fit_equals_single_gpu(case):
    import torch.multiprocessing as mp
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import catboost_rs_b200 as cb
    from synth import make_dataset
    X, y, borders = make_dataset(case["n"], case["F"], seed=case["seed"], nan_frac=0.05,
                                 loss=case["loss"], border_count=32, uniform_half=True)
    fp = cb.FitParams(loss=case["loss"], depth=case["depth"], iterations=case["it"],
                      score_function="Cosine", bootstrap_type=case["boot"], subsample=0.7,
                      random_seed=5, boost_from_average=case["loss"] == "RMSE")
    single = cb.fit([np.ascontiguousarray(X[:, f]) for f in range(X.shape[1])], borders, y, fp, staged=True)
    world = 2
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank_fit, args=(r, world, uid_q, out_q, case)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        item = out_q.get(timeout=300)
        assert len(item) != 2, item
        res[item[0]] = item
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        _, off, cnt, sf, sb, lv, st = res[r]
        np.testing.assert_array_equal(sf, single.split_feature)
        np.testing.assert_array_equal(sb, single.split_bin)
        np.testing.assert_array_equal(lv, single.leaf_values)
        np.testing.assert_array_equal(st, single.staged[:, off:off + cnt])
