"""GPU parity of the graph index (C4 path): fg_graph_build and
fg_graph_search against the CPU oracle's restatement, bit for bit (graph,
ids, distances, device counters), plus recall on a C4-shaped mixture and the
argument checks."""
import numpy as np
import pytest

import oracle
from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def fgg():
    import fusiongpu_b200.graph as g
    return g


def _c4_like(n, nq, dim=128, seed=44):
    import dataclasses
    from fusiongpu_b200 import datasets as ds
    spec = dataclasses.replace(ds.scaled(ds.C4, n, nq, n_centres=40, seed=seed), dim=dim)
    return ds.generate(spec)  # float16, unit norm


_CACHE = {}


def built(kind, fgg):
    if kind in _CACHE:
        return _CACHE[kind]
    if kind == "ip16":
        base, q = _c4_like(6000, 64)
        bp = dict(graph_degree=32, intermediate_degree=64, nlist=24, probe_lists=4, kmeans_iters=4, seed=42,
                  metric="ip")
    else:
        rng = np.random.default_rng(3)
        base = rng.normal(size=(5000, 64)).astype(np.float32)
        q = rng.normal(size=(48, 64)).astype(np.float32)
        bp = dict(graph_degree=16, intermediate_degree=48, nlist=20, probe_lists=3, kmeans_iters=4, seed=5,
                  metric="l2")
    tb = torch.from_numpy(base).cuda()
    gi = fgg.GraphIndex.build(tb, fgg.GraphBuildParams(**bp))
    eg = oracle.graph_build(base.astype(np.float32), **bp, entries=True)
    _CACHE[kind] = (base, q, gi, eg, bp)
    return _CACHE[kind]


@pytest.mark.parametrize("kind", ["ip16", "l2f32"])
def test_graph_build_bit_exact(kind, fgg):
    base, q, gi, (eg, ec, en), bp = built(kind, fgg)
    np.testing.assert_array_equal(gi.graph.cpu().numpy(), eg)
    np.testing.assert_array_equal(gi.entry_centroids.cpu().numpy(), ec)
    np.testing.assert_array_equal(gi.entry_nodes.cpu().numpy(), en)


@pytest.mark.parametrize("kind,itopk,width,k,ep", [("ip16", 64, 2, 10, 0), ("ip16", 128, 4, 10, 0),
                                                   ("ip16", 32, 4, 10, 8), ("ip16", 128, 4, 10, 16),
                                                   ("l2f32", 32, 1, 8, 0), ("l2f32", 96, 3, 16, 5)])
def test_graph_search_bit_exact(kind, itopk, width, k, ep, fgg):
    base, q, gi, (eg, ecen, enodes), bp = built(kind, fgg)
    sp = fgg.GraphSearchParams(itopk=itopk, search_width=width, k=k, seed=11, metric=bp["metric"], entry_probes=ep)
    ids, d, cnt = gi.search(torch.from_numpy(q).cuda(), sp, counters=True)
    ei, ed, ec = oracle.graph_search(base, eg, q, itopk=itopk, search_width=width, k=k, seed=11, metric=bp["metric"],
                                     entry_centroids=ecen, entry_nodes=enodes, entry_probes=ep)
    np.testing.assert_array_equal(ids.cpu().numpy(), ei)
    np.testing.assert_array_equal(d.cpu().numpy(), ed)
    c = cnt.cpu().numpy().astype(np.uint64)
    assert c[2] == 0  # no failed index check
    np.testing.assert_array_equal(c[:2], ec)


def test_graph_search_fixed_iterations_and_reset(fgg):
    # many iterations on a random graph: the visited hash is reset on the way
    rng = np.random.default_rng(9)
    n, D = 30000, 32
    x = rng.normal(size=(n, 64)).astype(np.float16)
    g = rng.integers(0, n, size=(n, D)).astype(np.int32)
    q = rng.normal(size=(20, 64)).astype(np.float16)
    gi = fgg.GraphIndex(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda())
    sp = fgg.GraphSearchParams(itopk=256, search_width=8, max_iterations=60, k=20, seed=4)
    ids, d, cnt = gi.search(torch.from_numpy(q).cuda(), sp, counters=True)
    ei, ed, ec = oracle.graph_search(x, g, q, itopk=256, search_width=8, max_iterations=60, k=20, seed=4)
    assert int(ec[0]) > 20 * 4096
    np.testing.assert_array_equal(ids.cpu().numpy(), ei)
    np.testing.assert_array_equal(d.cpu().numpy(), ed)
    c = cnt.cpu().numpy().astype(np.uint64)
    assert c[2] == 0  # no failed index check
    np.testing.assert_array_equal(c[:2], ec)


def test_graph_recall_c4_shape(fgg):
    base, q, gi, eg, bp = built("ip16", fgg)
    gt, _ = fgg.knn_ip(torch.from_numpy(base).cuda(), torch.from_numpy(q).cuda(), 10)
    ids, _ = gi.search(torch.from_numpy(q).cuda(),
                       fgg.GraphSearchParams(itopk=128, search_width=4, k=10, entry_probes=8))
    got, g = ids.cpu().numpy(), gt.cpu().numpy()
    rec = np.mean([len(set(got[i]) & set(g[i])) / 10 for i in range(len(q))])
    assert rec >= 0.95, rec


def test_knn_ip_matches_numpy(fgg):
    rng = np.random.default_rng(2)
    x = rng.normal(size=(3000, 96)).astype(np.float32)
    q = rng.normal(size=(40, 96)).astype(np.float32)
    ids, d = fgg.knn_ip(torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda(), 10)
    exp = np.argsort(-(q.astype(np.float64) @ x.astype(np.float64).T), axis=1, kind="stable")[:, :10]
    assert np.mean(ids.cpu().numpy() == exp) > 0.99
    np.testing.assert_allclose(-d.cpu().numpy(), np.take_along_axis(q @ x.T, exp, 1), rtol=1e-4, atol=1e-4)


def test_graph_errors(fgg):
    from fusiongpu_b200 import _lib
    x = torch.zeros((100, 12), dtype=torch.float16, device="cuda")  # 12 halves: not 16-byte rows
    g = torch.zeros((100, 8), dtype=torch.int32, device="cuda")
    gi = fgg.GraphIndex(x, g)
    with pytest.raises(_lib.FgError) as e:
        gi.search(x[:2], fgg.GraphSearchParams(k=4, itopk=16))
    assert e.value.status == 1
    gi = fgg.GraphIndex(torch.zeros((100, 16), dtype=torch.float16, device="cuda"), g)
    with pytest.raises(_lib.FgError):
        gi.search(gi.data[:2], fgg.GraphSearchParams(k=32, itopk=16))
    ids, d = gi.search(gi.data[:0], fgg.GraphSearchParams(k=4, itopk=16))
    assert ids.shape == (0, 4)
