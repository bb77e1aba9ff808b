"""Graph index on the CPU: the oracle's restatement of the product's build
and search against plain-Python loops on integer-valued vectors (exact
distances, many ties), including visited-set resets."""
import numpy as np
import pytest

import oracle
from tests import refpy


def _ints(n, dim, seed, lo=-3, hi=4):
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi, size=(n, dim)).astype(np.float32)


@pytest.mark.parametrize("metric", ["ip", "l2"])
def test_graph_build_matches_python(metric):
    x = _ints(260, 12, 5)
    g = oracle.graph_build(x, graph_degree=8, intermediate_degree=16, nlist=6, probe_lists=3, kmeans_iters=3, seed=42,
                           metric=metric)
    r = refpy.graph_build(x, 8, 16, 6, 3, 3, 42, metric, oracle.kmeans, oracle.assign, oracle.coarse)
    np.testing.assert_array_equal(g, r)
    assert (g >= 0).all() and not any(u in g[u] for u in range(len(x)))


@pytest.mark.parametrize("metric,dtype", [("ip", np.float16), ("l2", np.float32)])
def test_graph_search_matches_python(metric, dtype):
    x = _ints(400, 16, 6)
    g = oracle.graph_build(x, 8, 16, 8, 3, 3, 42, metric)
    q = _ints(12, 16, 7)
    oi, od, cnt = oracle.graph_search(x.astype(dtype), g, q.astype(dtype), itopk=32, search_width=2, k=10, seed=3,
                                      metric=metric)
    ri, rd, rc = refpy.graph_search(x, g, q, 32, 2, 0, 10, 3, metric)
    np.testing.assert_array_equal(oi, ri)
    np.testing.assert_array_equal(od, rd)
    assert tuple(int(c) for c in cnt) == rc


def test_graph_search_visited_reset():
    # a long walk on a large ring-like graph: more than 4096 nodes visited
    n, D = 20000, 16
    x = _ints(n, 8, 8)
    rng = np.random.default_rng(9)
    g = rng.integers(0, n, size=(n, D)).astype(np.int32)
    q = _ints(3, 8, 10)
    oi, od, cnt = oracle.graph_search(x, g, q, itopk=256, search_width=8, max_iterations=80, k=10, seed=1, metric="ip")
    ri, rd, rc = refpy.graph_search(x, g, q, 256, 8, 80, 10, 1, "ip")
    assert rc[0] > 3 * 4096  # the visited set was reset on the way
    np.testing.assert_array_equal(oi, ri)
    np.testing.assert_array_equal(od, rd)
    assert tuple(int(c) for c in cnt) == rc


def test_graph_search_padding_and_small_graphs():
    x = _ints(30, 8, 11)
    g = -np.ones((30, 4), np.int32)
    g[:, 0] = (np.arange(30) + 1) % 30
    q = _ints(2, 8, 12)
    oi, od, cnt = oracle.graph_search(x, g, q, itopk=16, search_width=1, k=10, seed=2, metric="l2")
    ri, rd, rc = refpy.graph_search(x, g, q, 16, 1, 0, 10, 2, "l2")
    np.testing.assert_array_equal(oi, ri)
    np.testing.assert_array_equal(od, rd)


def test_graph_search_entry_seeds_match_python():
    x = _ints(500, 16, 13)
    g = oracle.graph_build(x, 8, 16, 8, 3, 3, 42, "ip")
    q = _ints(10, 16, 14)
    ec = _ints(24, 16, 15)  # integer entry centroids: exact distances, ties by id
    en = np.random.default_rng(16).integers(-1, 500, size=24).astype(np.int32)
    oi, od, cnt = oracle.graph_search(x, g, q, itopk=32, search_width=2, k=10, seed=3, metric="ip",
                                      entry_centroids=ec, entry_nodes=en, entry_probes=5)
    ri, rd, rc = refpy.graph_search(x, g, q, 32, 2, 0, 10, 3, "ip", entry_centroids=ec, entry_nodes=en,
                                    entry_probes=5)
    np.testing.assert_array_equal(oi, ri)
    np.testing.assert_array_equal(od, rd)
    assert tuple(int(c) for c in cnt) == rc


def test_graph_entries_are_list_medoids():
    x = _ints(300, 12, 17)
    g, ec, en = oracle.graph_build(x, 8, 16, 6, 3, 3, 42, "l2", entries=True)
    cen = oracle.kmeans(x, 6, 3, 42)
    a = oracle.assign(x, cen)
    np.testing.assert_array_equal(ec, cen)
    for c in range(6):
        members = np.flatnonzero(a == c)
        if members.size == 0:
            assert en[c] == -1
            continue
        d = ((x[members].astype(np.float64) - cen[c]) ** 2).sum(1)
        assert en[c] in members[d <= d.min() + 1e-4]
