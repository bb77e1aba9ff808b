"""CPU tests of the oracle (the checker): against a pure-Python restatement on
tiny exact cases, known-answer tests, and the reference's own PQ code."""
import numpy as np
import pytest

import oracle
from tests import refpy

PARAM_SETS = [
    dict(top_m=8, p1_lists=3, limit_k=20, threshold_coeff=1.0, prune_ratio=100.0, rerank_m=200,
         final_k=10, mini_batch=128, epsilon=0.1, beta=2),
    # large threshold: phase-2 lists overflow the reference's 128-slot buffer
    dict(top_m=8, p1_lists=2, limit_k=7, threshold_coeff=50.0, prune_ratio=100.0, rerank_m=300,
         final_k=16, mini_batch=40, epsilon=0.1, beta=3),
    # every list in phase 1, limit_k above most list lengths, shallow rerank
    dict(top_m=6, p1_lists=12, limit_k=500, threshold_coeff=1.0, prune_ratio=100.0, rerank_m=50,
         final_k=5, mini_batch=16, epsilon=0.0, beta=1),
    # pruning by distance ratio, tiny limit_k
    dict(top_m=8, p1_lists=4, limit_k=1, threshold_coeff=2.0, prune_ratio=1.6, rerank_m=1000,
         final_k=20, mini_batch=100, epsilon=0.5, beta=2),
]


def _probes(index, queries, top_m):
    return oracle.coarse(index["centroids"], queries, top_m)


@pytest.mark.parametrize("seed", [0, 1, 2])
@pytest.mark.parametrize("pi", range(len(PARAM_SETS)))
@pytest.mark.parametrize("ref_compat", [True, False])
def test_batch_logic_matches_python_restatement(seed, pi, ref_compat):
    index, base = refpy.toy_index(seed)
    rng = np.random.default_rng(100 + seed)
    q = rng.integers(0, 16, size=(12, index["centroids"].shape[1])).astype(np.float32)
    p = dict(PARAM_SETS[pi], ref_compat=ref_compat)
    pid, pd = _probes(index, q, p["top_m"])
    ti, td, tc, st = oracle.batch_logic(index, q, pid, pd, **p)
    ei, ed, ec, en = refpy.batch_logic(index, q, pid, pd, p)
    np.testing.assert_array_equal(tc, ec)
    np.testing.assert_array_equal(st["count"], en)
    np.testing.assert_array_equal(td, ed)
    np.testing.assert_array_equal(ti, ei)
    oi, od = oracle.rerank(q, ti, tc, base, **p)
    ri, rd = refpy.rerank(q, ei, ec, base, p)
    np.testing.assert_array_equal(od, rd)
    np.testing.assert_array_equal(oi, ri)


def test_overflow_case_is_exercised():
    index, base = refpy.toy_index(0)
    q = np.random.default_rng(5).integers(0, 16, size=(12, 16)).astype(np.float32)
    p = dict(PARAM_SETS[1], ref_compat=True)
    pid, pd = _probes(index, q, p["top_m"])
    _, _, _, st = oracle.batch_logic(index, q, pid, pd, **p)
    assert st["p2_overflow"].sum() > 0


def test_ref_compat_gather_leaves_lanes_past_128_as_zero():
    index, base = refpy.toy_index(1)
    q = np.random.default_rng(3).integers(0, 16, size=(4, 16)).astype(np.float32)
    p = dict(PARAM_SETS[0], rerank_m=300, ref_compat=True)
    pid, pd = _probes(index, q, p["top_m"])
    ti, td, tc, st = oracle.batch_logic(index, q, pid, pd, **p)
    assert (ti[:, 128:] == 0).all() and (td[:, 128:] == 0).all()
    assert (tc == np.minimum(st["count"], 300)).all()


def test_coarse_exact_ranking():
    rng = np.random.default_rng(0)
    cen = rng.integers(0, 50, size=(300, 24)).astype(np.float32)
    q = rng.integers(0, 50, size=(40, 24)).astype(np.float32)
    ids, d = oracle.coarse(cen, q, 17)
    full = ((q[:, None, :].astype(np.int64) - cen[None].astype(np.int64)) ** 2).sum(-1)
    for i in range(q.shape[0]):
        order = np.lexsort((np.arange(cen.shape[0]), full[i]))[:17]
        np.testing.assert_array_equal(ids[i], order)
        np.testing.assert_array_equal(d[i], full[i][order].astype(np.float32))


def test_knn_exact_ties_by_id():
    base = np.zeros((10, 4), np.float32)
    base[3] = 1.0
    q = np.zeros((1, 4), np.float32)
    ids, d = oracle.knn_exact(base, q, 5)
    np.testing.assert_array_equal(ids[0], [0, 1, 2, 4, 5])
    assert (d == 0).all()


def test_mt19937_known_answer():
    # C++ [rand.predef]: the 10000th output of a default-constructed mt19937 (seed 5489)
    assert oracle.mt19937(5489, 9999) == 4123659995


def test_kmeans_update_is_mean_and_empty_keeps_centroid():
    rng = np.random.default_rng(1)
    x = rng.normal(size=(500, 8)).astype(np.float32)
    a = rng.integers(0, 5, size=500).astype(np.int32)
    a[a == 3] = 2  # cluster 3 empty
    c0 = rng.normal(size=(5, 8)).astype(np.float32)
    c, cnt = oracle.kmeans_update(x, a, c0)
    for j in range(5):
        if j == 3:
            np.testing.assert_array_equal(c[j], c0[j])
            assert cnt[j] == 0
        else:
            np.testing.assert_allclose(c[j], x[a == j].astype(np.float64).mean(0), rtol=1e-6, atol=1e-7)


def test_kmeans_objective_decreases():
    from fusiongpu_b200 import datasets as ds
    base, _ = ds.generate(ds.scaled(ds.C1, 4000, 10, n_centres=32))
    prev = None
    for it in (1, 3, 6):
        c = oracle.kmeans(base, 32, it)
        a = oracle.assign(base, c)
        obj = float(((base - c[a]) ** 2).sum())
        if prev is not None:
            assert obj <= prev * (1 + 1e-6)
        prev = obj


@pytest.mark.parametrize("n,seed", [(1, 5), (2, 7), (11, 2), (4096, 1234), (50000, 1234), (50001, 1235),
                                    (65535, 3), (65536, 3), (300000, 12345)])
def test_shuffle_equals_std_shuffle(n, seed):
    """The oracle's std::shuffle restatement against std::shuffle of the C++
    standard library the reference is compiled with (oracle/_ref): both the
    paired-draw path (n*n within the generator's range) and the single-draw
    path."""
    ref = oracle.ref_std_shuffle(n, seed)
    if ref is None:
        pytest.skip("oracle/_ref not built (reference sources absent)")
    np.testing.assert_array_equal(oracle.std_shuffle(n, seed), ref)


@pytest.mark.parametrize("dim,pq_m,sample", [(64, 16, 4000), (128, 32, 50000), (96, 48, 7000), (128, 64, 3000)])
def test_pq_training_equals_reference_pq_utils(dim, pq_m, sample):
    """The oracle's residual PQ trainer reproduces the reference's own
    train_residual_pq_codebooks (pq_utils.h:77-138, compiled from source into
    oracle/_ref) bit for bit: the same shuffled sample, the same seeded
    codewords, the same two-rounding distances and double means."""
    if oracle.ref_lib("pq", dim, pq_m) is None:
        pytest.skip("oracle/_ref not built (reference sources absent)")
    from fusiongpu_b200 import datasets as ds
    spec = ds.dataclasses.replace(ds.scaled(ds.C1, 9000, 10, n_centres=16), dim=dim)
    base, _ = ds.generate(spec)
    cen = oracle.kmeans(base, 24, 3)
    a = oracle.assign(base, cen)
    ours = oracle.pq_train(base, a, cen, pq_m, sample, 5)
    ref = oracle.ref_pq_train(base, a, cen, pq_m, sample, 5)
    np.testing.assert_array_equal(ours, ref)
    if dim == 64:
        # the encoders agree where the reference's unfused arithmetic has no near-ties
        rc = oracle.ref_pq_encode(base, a, cen, ref)
        oc = oracle.pq_encode(base, a, cen, ref)
        assert (rc == oc).mean() > 0.999


def skewed_lists(seed=3, n=12000, k=16):
    """k-means lists with lists 0-4 merged into list 0 (about five times the
    mean; lists 1-4 empty), so that rebalancing has to split."""
    rng = np.random.default_rng(seed)
    x = np.ascontiguousarray(rng.normal(size=(n, 32)), dtype=np.float32)
    cen = oracle.kmeans(x, k, 4)
    a = oracle.assign(x, cen)
    a[a < 5] = 0
    return x, a, cen


def test_rebalance_matches_python_restatement():
    x, a, cen = skewed_lists()
    na, nc = oracle.rebalance(x, a, cen)
    ra, rc = refpy.rebalance(x, a, cen, oracle.kmeans, oracle.assign)
    np.testing.assert_array_equal(na, ra)
    np.testing.assert_array_equal(nc, rc)
    lens = np.bincount(na, minlength=nc.shape[0])
    assert nc.shape[0] > np.unique(a).size and lens.min() > 0
    assert (lens <= int(2 * x.shape[0] / 16)).all()


def test_rebalance_stops_on_identical_points():
    # every point equal: each split would put all points in child 0 again
    x = np.zeros((400, 8), np.float32)
    x[:40] = 1.0
    cen = oracle.kmeans(x, 8, 2)
    a = oracle.assign(x, cen)
    na, nc = oracle.rebalance(x, a, cen)
    ra, rc = refpy.rebalance(x, a, cen, oracle.kmeans, oracle.assign)
    np.testing.assert_array_equal(na, ra)
    np.testing.assert_array_equal(nc, rc)
    assert np.bincount(na).sum() == 400
