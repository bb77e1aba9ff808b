"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle, and
the reference's own kernels (oracle/_ref) against the oracle.

Integer and index outputs must match exactly; distances bit-exactly, since
both sides compute the same float expressions in the same order."""
import ctypes as C

import numpy as np
import pytest

import oracle
from tests import refpy
from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

torch = pytest.importorskip("torch")


def _np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def fg():
    import fusiongpu_b200.index as fgi
    return fgi


SCAN_KERNELS = ["auto", "block", "team_otf/64", "team_otf/128", "team_otf/256", "team_lut/64", "team_lut/128",
                "team_lut/256", "team_otf/64/teamselect", "split", "group"]


@pytest.fixture(params=SCAN_KERNELS)
def scan_kernel(request, monkeypatch):
    """Runs the test once per scan kernel: the per-query CTA kernel, the
    team kernel with table or on-the-fly ADC, teams of 64, 128 or 256 threads
    (FG_SCAN_KERNEL, FG_SCAN_TEAM_NT; 64 yields to 128 under ref_compat), the
    team-wide list selection (FG_SCAN_WARP_SELECT=0), the split path (one
    CTA per probed list, candidates in the workspace) and the group kernel
    (the queries probing one list together; parameters with a phase 2 run
    the team kernel under it)."""
    if request.param != "auto":
        kern, _, rest = request.param.partition("/")
        nt, _, sel = rest.partition("/")
        monkeypatch.setenv("FG_SCAN_KERNEL", kern)
        if nt:
            monkeypatch.setenv("FG_SCAN_TEAM_NT", nt)
        if sel == "teamselect":  # team-wide selection where one warp would do it
            monkeypatch.setenv("FG_SCAN_WARP_SELECT", "0")
    return request.param


def _dataset(kind):
    from fusiongpu_b200 import datasets as ds
    if kind == "int128":
        spec = ds.scaled(ds.C1, 20000, 192, n_centres=64, seed=11)
        base, q = ds.generate(spec)
        index, _ = oracle.build_index(base, 128, 32, kmeans_iters=6, pq_sample=8000, pq_iters=6)
    elif kind == "int128m64":
        spec = ds.scaled(ds.C2, 20000, 192, n_centres=64, seed=12)
        base, q = ds.generate(spec)
        index, _ = oracle.build_index(base, 96, 64, kmeans_iters=6, pq_sample=8000, pq_iters=6)
    elif kind == "unit96":
        spec = ds.scaled(ds.C3, 20000, 192, n_centres=64, seed=13)
        base, q = ds.generate(spec)
        index, _ = oracle.build_index(base, 128, 48, kmeans_iters=6, pq_sample=8000, pq_iters=6)
    else:
        raise ValueError(kind)
    return index, base, q


_CACHE = {}


def dataset(kind):
    if kind not in _CACHE:
        _CACHE[kind] = _dataset(kind)
    return _CACHE[kind]


PARAMS = {
    "c1": dict(top_m=16, p1_lists=6, limit_k=50, threshold_coeff=1.0, prune_ratio=100.0, rerank_m=100,
               final_k=10, mini_batch=128, epsilon=0.1, beta=2),
    "deep": dict(top_m=24, p1_lists=8, limit_k=60, threshold_coeff=1.2, prune_ratio=100.0, rerank_m=700,
                 final_k=100, mini_batch=128, epsilon=0.1, beta=2),
    "overflow": dict(top_m=20, p1_lists=2, limit_k=20, threshold_coeff=4.0, prune_ratio=100.0, rerank_m=400,
                     final_k=20, mini_batch=64, epsilon=0.05, beta=3),
    "prune": dict(top_m=32, p1_lists=40, limit_k=10, threshold_coeff=1.0, prune_ratio=1.05, rerank_m=64,
                  final_k=8, mini_batch=16, epsilon=0.2, beta=1),
    # the C2 operating point's shape: two probes, both in phase 1, deep rerank
    "nprobe2": dict(top_m=2, p1_lists=12, limit_k=50, threshold_coeff=1.0, prune_ratio=100.0, rerank_m=1000,
                    final_k=100, mini_batch=128, epsilon=0.1, beta=2),
}


def _params(fg, name, ref_compat):
    return fg.SearchParams(**PARAMS[name], ref_compat=ref_compat)


@pytest.mark.parametrize("kind", ["int128", "int128m64", "unit96"])
def test_coarse_matches_oracle(fg, kind):
    index, base, q = dataset(kind)
    for top_m in (1, 16, 77):
        ids, d = fg.coarse_search(q, index["centroids"], top_m)
        eids, ed = oracle.coarse(index["centroids"], q, top_m)
        np.testing.assert_array_equal(_np(ids).astype(np.uint32), eids)
        np.testing.assert_array_equal(_np(d), ed)


@pytest.mark.parametrize("kind", ["int128", "unit96"])
@pytest.mark.parametrize("path", ["tc", "simt"])
def test_coarse_paths_match_oracle(fg, kind, path):
    index, base, q = dataset(kind)
    for top_m in (1, 2, 3, 4, 5, 16, 77, 128):
        r = fg.coarse_search(q, index["centroids"], top_m, path=path)
        eids, ed = oracle.coarse(index["centroids"], q, top_m)
        np.testing.assert_array_equal(_np(r[1]), ed)
        np.testing.assert_array_equal(_np(r[0]).astype(np.uint32), eids)
        if path == "tc":
            assert r[2] <= q.shape[0] // 20  # the certificate holds for almost every query


def test_coarse_tc_fallback_on_ties(fg):
    """Every centroid has exactly three ones, so all are at distance 3 from a
    zero query: the tie spans the cut, the certificate cannot hold, and the
    exact fallback must reproduce the oracle's (distance, id) ranking."""
    rng = np.random.default_rng(9)
    cen = np.zeros((700, 32), np.float32)
    for i in range(700):
        cen[i, rng.choice(32, 3, replace=False)] = 1.0
    q = rng.integers(0, 2, size=(64, 32)).astype(np.float32)
    q[::2] = 0.0
    for top_m in (20, 3, 1):  # the multi-pass path and the single-pass top-8 path
        ids, d, nfb = fg.coarse_search(q, cen, top_m, path="tc")
        eids, ed = oracle.coarse(cen, q, top_m)
        np.testing.assert_array_equal(_np(d), ed)
        np.testing.assert_array_equal(_np(ids).astype(np.uint32), eids)
        assert nfb >= 32


def test_coarse_tc_odd_shapes(fg):
    """nlist and nq not multiples of the tiles, dim not a multiple of 64/3."""
    rng = np.random.default_rng(11)
    cen = rng.normal(size=(1001, 40)).astype(np.float32)
    q = rng.normal(size=(333, 40)).astype(np.float32)
    for top_m in (1, 2, 4, 7, 64):
        ids, d, nfb = fg.coarse_search(q, cen, top_m, path="tc")
        eids, ed = oracle.coarse(cen, q, top_m)
        np.testing.assert_array_equal(_np(d), ed)
        np.testing.assert_array_equal(_np(ids).astype(np.uint32), eids)


@pytest.mark.parametrize("nlist", [5, 16, 31])
def test_coarse_tc_fewer_lists_than_a_warp(fg, nlist):
    """nlist below 32: the exactly rescored superset (every list) is shorter
    than a warp, so the finish kernel's rescoring round has idle lanes."""
    rng = np.random.default_rng(nlist)
    cen = rng.normal(size=(nlist, 128)).astype(np.float32)
    q = rng.normal(size=(70, 128)).astype(np.float32)
    for top_m in sorted({1, 2, 4, min(8, nlist), nlist}):
        ids, d, nfb = fg.coarse_search(q, cen, top_m, path="tc")
        eids, ed = oracle.coarse(cen, q, top_m)
        np.testing.assert_array_equal(_np(d), ed)
        np.testing.assert_array_equal(_np(ids).astype(np.uint32), eids)


def test_coarse_tc_ranges_cross_query_tiles(fg):
    """40 query tiles x 8 centroid tiles = 320 (query tile, centroid tile)
    pairs over at most 148 CTAs: ranges of 3 pairs start and end inside query
    tiles, so CTAs reload the query tile and lists come from several segments."""
    rng = np.random.default_rng(21)
    cen = rng.normal(size=(1000, 64)).astype(np.float32)
    q = rng.normal(size=(5000, 64)).astype(np.float32)
    for top_m in (1, 2, 3, 16):
        ids, d, nfb = fg.coarse_search(q, cen, top_m, path="tc")
        eids, ed = oracle.coarse(cen, q, top_m)
        np.testing.assert_array_equal(_np(d), ed)
        np.testing.assert_array_equal(_np(ids).astype(np.uint32), eids)
        assert nfb <= q.shape[0] // 20


def test_coarse_tc_many_lists_two_stage(fg):
    """nlist above one select segment (8192): stage-2 merge in the superset select."""
    rng = np.random.default_rng(10)
    cen = rng.normal(size=(20000, 64)).astype(np.float32)
    q = rng.normal(size=(200, 64)).astype(np.float32)
    for top_m in (64, 4):
        ids, d, nfb = fg.coarse_search(q, cen, top_m, path="tc")
        eids, ed = oracle.coarse(cen, q, top_m)
        np.testing.assert_array_equal(_np(d), ed)
        np.testing.assert_array_equal(_np(ids).astype(np.uint32), eids)


@pytest.mark.parametrize("kind", ["int128", "int128m64", "unit96"])
@pytest.mark.parametrize("pname", list(PARAMS))
@pytest.mark.parametrize("ref_compat", [True, False])
def test_batch_logic_and_rerank_match_oracle(fg, kind, pname, ref_compat, scan_kernel):
    index, base, q = dataset(kind)
    p = _params(fg, pname, ref_compat)
    if ref_compat and p.final_k > 128:
        pytest.skip("ref_compat needs final_k <= 128")
    eids, ed = oracle.coarse(index["centroids"], q, p.top_m)
    idx = fg.IVFPQIndex.from_arrays(index, base)
    ti, td, tc, cc = fg.run_gpu_batch_logic(idx, q, eids.view(np.int32), ed, p)
    pd = dict(PARAMS[pname], ref_compat=ref_compat)
    oi, od, oc, st = oracle.batch_logic(index, q, eids, ed, **pd)
    np.testing.assert_array_equal(_np(cc), st["count"])
    np.testing.assert_array_equal(_np(tc), oc)
    np.testing.assert_array_equal(_np(td), od)
    np.testing.assert_array_equal(_np(ti), oi)
    ri, rd = fg.run_gpu_rerank(q, ti, tc, base, p)
    xi, xd = oracle.rerank(q, oi, oc, base, **pd)
    np.testing.assert_array_equal(_np(rd), xd)
    np.testing.assert_array_equal(_np(ri), xi)


@pytest.mark.parametrize("kind", ["int128", "unit96"])
@pytest.mark.parametrize("ref_compat", [True, False])
def test_full_search_matches_oracle(fg, kind, ref_compat, scan_kernel):
    index, base, q = dataset(kind)
    p = _params(fg, "c1", ref_compat)
    idx = fg.IVFPQIndex.from_arrays(index, base)
    ids, d = idx.search(q, p)
    ei, ed = oracle.search(index, base, q, **PARAMS["c1"], ref_compat=ref_compat)
    np.testing.assert_array_equal(_np(ids), ei)
    np.testing.assert_array_equal(_np(d), ed)


@pytest.mark.parametrize("seed", [0, 1, 2])
@pytest.mark.parametrize("ref_compat", [True, False])
def test_toy_edge_cases(fg, seed, ref_compat, scan_kernel):
    """Empty lists, a 1100-vector list (phase-1 clamp), phase-2 overflow,
    heavy distance ties (integer codebooks)."""
    index, base = refpy.toy_index(seed)
    q = np.random.default_rng(100 + seed).integers(0, 16, size=(12, 16)).astype(np.float32)
    idx = fg.IVFPQIndex.from_arrays(index, base)
    for pd in [dict(top_m=8, p1_lists=3, limit_k=20, threshold_coeff=1.0, prune_ratio=100.0, rerank_m=200,
                    final_k=10, mini_batch=128, epsilon=0.1, beta=2),
               dict(top_m=8, p1_lists=2, limit_k=7, threshold_coeff=50.0, prune_ratio=100.0, rerank_m=300,
                    final_k=16, mini_batch=40, epsilon=0.1, beta=3),
               dict(top_m=6, p1_lists=12, limit_k=500, threshold_coeff=1.0, prune_ratio=100.0, rerank_m=50,
                    final_k=5, mini_batch=16, epsilon=0.0, beta=1)]:
        pd = dict(pd, ref_compat=ref_compat)
        p = fg.SearchParams(**pd)
        eids, ed = oracle.coarse(index["centroids"], q, p.top_m)
        ti, td, tc, cc = fg.run_gpu_batch_logic(idx, q, eids.view(np.int32), ed, p)
        oi, od, oc, st = oracle.batch_logic(index, q, eids, ed, **pd)
        np.testing.assert_array_equal(_np(cc), st["count"])
        np.testing.assert_array_equal(_np(tc), oc)
        np.testing.assert_array_equal(_np(td), od)
        np.testing.assert_array_equal(_np(ti), oi)
        ri, rd = fg.run_gpu_rerank(q, ti, tc, base, p)
        xi, xd = oracle.rerank(q, oi, oc, base, **pd)
        np.testing.assert_array_equal(_np(ri), xi)
        np.testing.assert_array_equal(_np(rd), xd)


def test_knn_matches_oracle(fg):
    index, base, q = dataset("int128")
    ids, d = fg.knn_exact(base, q[:64], 10)
    ei, ed = oracle.knn_exact(base, q[:64], 10)
    np.testing.assert_array_equal(_np(ids), ei)
    np.testing.assert_array_equal(_np(d), ed)


def test_knn_two_stage_selection(fg):
    """More than one 8192-column segment: the stage-2 merge must keep the
    (distance, id) order."""
    rng = np.random.default_rng(4)
    base = rng.integers(0, 4, size=(30000, 8)).astype(np.float32)  # many exact ties
    q = rng.integers(0, 4, size=(16, 8)).astype(np.float32)
    ids, d = fg.knn_exact(base, q, 50)
    ei, ed = oracle.knn_exact(base, q, 50)
    np.testing.assert_array_equal(_np(d), ed)
    np.testing.assert_array_equal(_np(ids), ei)


def test_build_steps_match_oracle(fg):
    from fusiongpu_b200 import datasets as ds
    base, _ = ds.generate(ds.scaled(ds.C1, 12000, 4, n_centres=32, seed=21))
    xb = torch.from_numpy(base).cuda()
    cen = fg.run_kmeans_gpu(xb, 64, 5)
    ecen = oracle.kmeans(base, 64, 5)
    np.testing.assert_array_equal(_np(cen), ecen)
    a = fg.gpu_assign_to_centroids(xb, cen)
    ea = oracle.assign(base, ecen)
    np.testing.assert_array_equal(_np(a), ea)
    order, offs = fg.sort_by_list(a, 64)
    np.testing.assert_array_equal(_np(order), np.argsort(ea, kind="stable"))
    np.testing.assert_array_equal(_np(offs)[1:], np.cumsum(np.bincount(ea, minlength=64)))
    cb = fg.train_residual_pq_codebooks(xb, a, cen, 32, 6000, 4)
    ecb = oracle.pq_train(base, ea, ecen, 32, 6000, 4)
    np.testing.assert_array_equal(_np(cb), ecb)
    codes = fg.encode_residuals_to_pq_gpu(xb, a, cen, cb)
    np.testing.assert_array_equal(_np(codes), oracle.pq_encode(base, ea, ecen, ecb))
    idx = fg.IVFPQIndex.build(xb, 64, 32, kmeans_iters=5, pq_sample=6000, pq_iters=4)
    eidx, _ = oracle.build_index(base, 64, 32, kmeans_iters=5, pq_sample=6000, pq_iters=4)
    got = idx.to_numpy()
    for k in ("centroids", "codebook", "offsets", "ids", "codes"):
        np.testing.assert_array_equal(got[k], eidx[k])


def test_rebalance_bit_exact(fg):
    from tests.test_oracle_cpu import skewed_lists
    x, a, cen = skewed_lists()
    na, nc = fg.rebalance_lists(torch.from_numpy(x).cuda(), torch.from_numpy(a).cuda(), torch.from_numpy(cen).cuda())
    ea, ec = oracle.rebalance(x, a, cen)
    assert ec.shape[0] > np.unique(a).size
    np.testing.assert_array_equal(_np(na), ea)
    np.testing.assert_array_equal(_np(nc), ec)
    # identical points: the split loop must end
    z = np.zeros((400, 8), np.float32)
    z[:40] = 1.0
    zc = oracle.kmeans(z, 8, 2)
    za = oracle.assign(z, zc)
    na, nc = fg.rebalance_lists(torch.from_numpy(z).cuda(), torch.from_numpy(za).cuda(), torch.from_numpy(zc).cuda())
    ea, ec = oracle.rebalance(z, za, zc)
    np.testing.assert_array_equal(_np(na), ea)
    np.testing.assert_array_equal(_np(nc), ec)


def test_rebalanced_build_bit_exact(fg):
    # blobs of unequal spread: two k-means steps leave lists above twice the mean
    rng = np.random.default_rng(7)
    centres = rng.normal(0, 4, size=(3, 64))
    base = np.concatenate([rng.normal(centres[0], 0.5, size=(5000, 64)),
                           rng.normal(centres[1], 1.0, size=(2000, 64)),
                           rng.normal(centres[2], 3.0, size=(1000, 64))]).astype(np.float32)
    base = np.ascontiguousarray(base[rng.permutation(base.shape[0])])
    idx = fg.IVFPQIndex.build(torch.from_numpy(base).cuda(), 32, 16, kmeans_iters=2, pq_sample=4000, pq_iters=3)
    eidx, _ = oracle.build_index(base, 32, 16, kmeans_iters=2, pq_sample=4000, pq_iters=3)
    assert eidx["centroids"].shape[0] > 32
    got = idx.to_numpy()
    for k in ("centroids", "codebook", "offsets", "ids", "codes"):
        np.testing.assert_array_equal(got[k], eidx[k])


def test_errors_are_reported(fg):
    from fusiongpu_b200 import _lib
    index, base, q = dataset("int128")
    idx = fg.IVFPQIndex.from_arrays(index, base)
    with pytest.raises(_lib.FgError) as e:
        idx.search(q[:4], fg.SearchParams(top_m=0))
    assert e.value.status == 1
    with pytest.raises(_lib.FgError) as e:
        idx.search(q[:4], fg.SearchParams(top_m=10, limit_k=2000, ref_compat=True))
    assert e.value.status == 1
    # an empty batch is a no-op
    ids, d = idx.search(q[:0], fg.SearchParams(top_m=10))
    assert ids.shape == (0, 10)


# ---- the reference's own kernels pin the oracle ---------------------------------

def _ref_batch_and_rerank(index, base, q, pid, pdist, p):
    dim = index["centroids"].shape[1]
    pq_m = index["codes"].shape[1]
    L = oracle.ref_lib("gg", dim, pq_m)
    if L is None:
        pytest.skip("oracle/_ref not built")
    dev = "cuda"
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in index.items()}
    tq = torch.from_numpy(q).to(dev)
    tpid = torch.from_numpy(pid.view(np.int32).copy()).to(dev)
    tpd = torch.from_numpy(pdist).to(dev)
    nq, rm, k = q.shape[0], p["rerank_m"], p["final_k"]
    top_i = torch.zeros((nq, rm), dtype=torch.int32, device=dev)  # fresh (zeroed) memory
    top_d = torch.zeros((nq, rm), dtype=torch.float32, device=dev)
    top_c = torch.zeros(nq, dtype=torch.int32, device=dev)
    cnt = torch.zeros(nq, dtype=torch.int32, device=dev)
    P = lambda x: C.c_void_p(x.data_ptr())
    torch.cuda.synchronize()
    rc = L.ref_run_batch_logic(P(t["codebook"]), P(t["offsets"]), P(t["codes"]), P(t["ids"]), P(t["centroids"]),
                               index["centroids"].shape[0], P(tq), P(tpid), P(tpd), nq, p["top_m"], rm, k,
                               C.c_float(p["prune_ratio"]), p["p1_lists"], p["limit_k"],
                               C.c_float(p["threshold_coeff"]), P(top_i), P(top_d), P(top_c), P(cnt))
    assert rc == 0, f"reference batch logic failed: cuda error {rc}"
    tb = torch.from_numpy(base).to(dev)
    fi = torch.zeros((nq, k), dtype=torch.int32, device=dev)
    fd = torch.zeros((nq, k), dtype=torch.float32, device=dev)
    rc = L.ref_run_rerank(P(tq), P(top_i), P(top_c), P(tb), P(fi), P(fd), nq, rm, k, base.shape[0],
                          p["mini_batch"], C.c_float(p["epsilon"]), p["beta"])
    assert rc == 0, f"reference rerank failed: cuda error {rc}"
    return [_np(x) for x in (top_i, top_d, top_c, cnt, fi, fd)]


@pytest.mark.parametrize("kind", ["int128", "int128m64", "unit96"])
@pytest.mark.parametrize("pname", ["c1", "deep", "prune"])
def test_reference_kernels_agree_with_oracle(kind, pname):
    index, base, q = dataset(kind)
    p = dict(PARAMS[pname], ref_compat=True)
    pid, pdist = oracle.coarse(index["centroids"], q, p["top_m"])
    oi, od, oc, st = oracle.batch_logic(index, q, pid, pdist, **p)
    # The reference writes each query's candidates into a region sized by the
    # summed lengths of its probed lists; phase-2 overflow re-emission can
    # write past it.  Run the reference only where the oracle shows it stays
    # inside (the oracle's count is the reference's write count).
    lens = np.diff(index["offsets"])
    best = pdist[:, :1] * np.float32(p["prune_ratio"])
    budget = np.where(pdist > best, 0, lens[pid.astype(np.int64)]).sum(1)
    assert (st["count"] <= budget).all()
    ri, rd, rc, rn, fi, fd = _ref_batch_and_rerank(index, base, q, pid, pdist, p)
    np.testing.assert_array_equal(rn, st["count"])
    np.testing.assert_array_equal(rc, oc)
    clean = st["p2_overflow"] == 0  # overflow re-emission order depends on atomics
    assert clean.mean() > 0.5
    w = min(128, p["rerank_m"])
    np.testing.assert_array_equal(rd[clean, :w], od[clean, :w])
    # ids: equal except where equal distances may be ordered differently
    same = (ri[clean, :w] == oi[clean, :w]) | (rd[clean, :w] == np.roll(rd[clean, :w], 1, axis=1)) | (
        rd[clean, :w] == np.roll(rd[clean, :w], -1, axis=1))
    assert same.all()
    xi, xd = oracle.rerank(q, oi, oc, base, **p)
    np.testing.assert_array_equal(fd[clean], xd[clean])
    assert (fi[clean] == xi[clean]).mean() > 0.999


@pytest.mark.parametrize("n,k,dim", [(50000, 300, 96), (20000, 4096, 128), (8192, 64, 32)])
def test_assign_tensor_cores_bit_exact(fg, n, k, dim):
    rng = np.random.default_rng(n + k)
    x = rng.normal(size=(n, dim)).astype(np.float32)
    c = rng.normal(size=(k, dim)).astype(np.float32)
    c[k // 2] = c[1]  # duplicate centroids: the lower index wins
    x[:50] = c[1]     # points exactly on the duplicated centroid
    got = fg.gpu_assign_to_centroids(torch.from_numpy(x).cuda(), torch.from_numpy(c).cuda())
    np.testing.assert_array_equal(_np(got), oracle.assign(x, c))


def test_uint8_base_search_bit_exact(fg):
    # C1 vectors are integers in [0, 255]: a uint8 copy holds the same values
    index, base, q = dataset("int128")
    assert np.array_equal(base, base.astype(np.uint8).astype(np.float32))
    idx = fg.IVFPQIndex.from_arrays(index, base.astype(np.uint8))
    assert idx.base.dtype == torch.uint8
    for ref_compat in (False, True):
        p = dict(PARAMS["c1"], ref_compat=ref_compat)
        ids, d = idx.search(torch.from_numpy(q).cuda(), fg.SearchParams(**p))
        ei, ed = oracle.search(index, base, q, **p)
        np.testing.assert_array_equal(_np(ids), ei)
        np.testing.assert_array_equal(_np(d), ed)


def test_sampled_kmeans_build_bit_exact(fg):
    index, base, q = dataset("int128")
    idx = fg.IVFPQIndex.build(torch.from_numpy(base).cuda(), 64, 32, kmeans_iters=4, pq_sample=5000, pq_iters=3,
                              kmeans_sample=6000)
    eidx, _ = oracle.build_index(base, 64, 32, kmeans_iters=4, pq_sample=5000, pq_iters=3, kmeans_sample=6000)
    got = idx.to_numpy()
    for k in ("centroids", "codebook", "offsets", "ids", "codes"):
        np.testing.assert_array_equal(got[k], eidx[k])


@pytest.mark.parametrize("zero_copy", [True, False])
@pytest.mark.parametrize("chunks", [1, 2, 3])
def test_search_host_matches_device_search(fg, chunks, zero_copy):
    """The pipelined host-buffer search (pieces on two streams) returns the
    device search's results, whether the rerank writes the pinned result
    tensors in place or the results are copied back; a second call into the
    same buffers overwrites every entry."""
    index, base, q = dataset("int128")
    idx = fg.IVFPQIndex.from_arrays(index, base)
    p = _params(fg, "c1", False)
    ids, d = idx.search(q, p)
    hq = torch.from_numpy(np.ascontiguousarray(q)).pin_memory()
    out = (torch.full((q.shape[0], p.final_k), -7, dtype=torch.int32).pin_memory(),
           torch.full((q.shape[0], p.final_k), -7.0, dtype=torch.float32).pin_memory())
    for _ in range(2):
        hi, hd = idx.search_host(hq, p, out=out, chunks=chunks, zero_copy=zero_copy)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(hi.numpy(), _np(ids))
        np.testing.assert_array_equal(hd.numpy(), _np(d))
        out[0].fill_(-7)
        out[1].fill_(-7.0)


@pytest.mark.parametrize("chunks", [1, 2])
def test_search_host_graph_replays_new_queries(fg, chunks):
    """search_host(graph=True): the first call captures, later calls replay
    the graph on whatever the pinned query tensor holds by then, and each
    replay's results equal the device search of those queries."""
    index, base, q = dataset("int128")
    idx = fg.IVFPQIndex.from_arrays(index, base)
    p = _params(fg, "c1", False)
    n = q.shape[0] // 2
    hq = torch.empty((n, q.shape[1]), dtype=torch.float32).pin_memory()
    out = (torch.empty((n, p.final_k), dtype=torch.int32).pin_memory(),
           torch.empty((n, p.final_k), dtype=torch.float32).pin_memory())
    for rows in (slice(0, n), slice(n, 2 * n), slice(0, n)):
        qs = np.ascontiguousarray(q[rows])
        hq.copy_(torch.from_numpy(qs))
        out[0].fill_(-7)
        hi, hd = idx.search_host(hq, p, out=out, chunks=chunks, graph=True)
        torch.cuda.synchronize()
        ids, d = idx.search(qs, p)
        np.testing.assert_array_equal(hi.numpy(), _np(ids))
        np.testing.assert_array_equal(hd.numpy(), _np(d))


def test_host_memory_mapped_query(fg):
    """Pinned host memory is reported mapped, pageable host memory and device
    memory are not, so the zero-copy result path never hands a kernel memory
    it cannot reach."""
    import ctypes as C
    from fusiongpu_b200 import _lib

    def mapped(ptr):
        m = C.c_int32(-1)
        _lib.call("fg_host_memory_mapped", C.c_void_p(ptr), C.byref(m))
        return m.value

    pinned = torch.zeros(1024, dtype=torch.int32).pin_memory()
    pageable = np.zeros(1024, dtype=np.int32)
    dev = torch.zeros(1024, dtype=torch.int32, device="cuda")
    assert mapped(pinned.data_ptr()) == 1
    assert mapped(pinned.data_ptr() + 64) == 1
    assert mapped(pageable.ctypes.data) == 0
    assert mapped(dev.data_ptr()) == 0
    assert mapped(0) == 0
    with pytest.raises(ValueError):
        index, base, q = dataset("int128")
        idx = fg.IVFPQIndex.from_arrays(index, base)
        p = _params(fg, "c1", False)
        out = (torch.empty((q.shape[0], p.final_k), dtype=torch.int32),
               torch.empty((q.shape[0], p.final_k), dtype=torch.float32))
        idx.search_host(torch.from_numpy(np.ascontiguousarray(q)), p, out=out, zero_copy=True)


def test_search_graph_replay_matches_eager(fg):
    index, base, q = dataset("int128")
    idx = fg.IVFPQIndex.from_arrays(index, base)
    p = fg.SearchParams(**PARAMS["c1"])
    g = idx.capture(64, p)
    for s in (0, 64, 128):
        qb = torch.from_numpy(q[s:s + 64]).cuda()
        ids, d = g.replay(qb)
        ei, ed = idx.search(qb, p)
        np.testing.assert_array_equal(_np(ids), _np(ei))
        np.testing.assert_array_equal(_np(d), _np(ed))


def test_search_host_graphs_of_two_settings_alternate(fg):
    """Two search_host(graph=True) settings (piece count and rerank depth)
    used in turn: each replay keeps the streams, buffers and workspace it was
    captured with, so every replay still equals the device search."""
    index, base, q = dataset("int128")
    idx = fg.IVFPQIndex.from_arrays(index, base)
    pa = _params(fg, "c1", False)
    pb = pa.replace(rerank_m=max(pa.final_k, pa.rerank_m // 2))
    n = q.shape[0] // 2
    hq = torch.empty((n, q.shape[1]), dtype=torch.float32).pin_memory()
    outs = {}
    for rows, p, chunks in ((slice(0, n), pa, 1), (slice(n, 2 * n), pb, 2), (slice(n, 2 * n), pa, 1),
                            (slice(0, n), pb, 2), (slice(0, n), pa, 1)):
        key = (p.rerank_m, chunks)
        if key not in outs:
            outs[key] = (torch.empty((n, p.final_k), dtype=torch.int32).pin_memory(),
                         torch.empty((n, p.final_k), dtype=torch.float32).pin_memory())
        out = outs[key]
        qs = np.ascontiguousarray(q[rows])
        hq.copy_(torch.from_numpy(qs))
        out[0].fill_(-7)
        # an eager host search with yet another piece size replaces the cached eager state
        idx.search_host(torch.from_numpy(qs[:17]).pin_memory(), p, chunks=3)
        hi, hd = idx.search_host(hq, p, out=out, chunks=chunks, graph=True)
        torch.cuda.synchronize()
        ids, d = idx.search(qs, p)
        np.testing.assert_array_equal(hi.numpy(), _np(ids))
        np.testing.assert_array_equal(hd.numpy(), _np(d))


def test_search_graph_survives_a_larger_search(fg):
    """A captured SearchGraph holds its own workspace: a later, larger eager
    search (which grows the index's shared workspace) leaves the replay
    correct."""
    index, base, q = dataset("int128")
    idx = fg.IVFPQIndex.from_arrays(index, base)
    p = fg.SearchParams(**PARAMS["c1"])
    g = idx.capture(32, p)
    big = torch.from_numpy(np.ascontiguousarray(np.concatenate([q] * 4))).cuda()
    idx.search(big, p)
    for s in (0, 32, 64):
        qb = torch.from_numpy(np.ascontiguousarray(q[s:s + 32])).cuda()
        ids, d = g.replay(qb)
        ei, ed = idx.search(qb, p)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(_np(ids), _np(ei))
        np.testing.assert_array_equal(_np(d), _np(ed))


@pytest.mark.parametrize("coeff", [50.0, 1.6])
@pytest.mark.parametrize("ref_compat", [True, False])
def test_split_overflow_falls_back_to_per_query_kernel(fg, monkeypatch, coeff, ref_compat):
    """Queries whose candidates overflow the split path's per-query region
    (4096 keys) are recomputed by the per-query kernel: with every phase-2
    vector passing (coefficient 50) all queries overflow, with 1.6 some do;
    the results still equal the oracle's."""
    monkeypatch.setenv("FG_SCAN_KERNEL", "split")
    index, base, q = dataset("int128")
    pd = dict(top_m=64, p1_lists=2, limit_k=20, threshold_coeff=coeff, prune_ratio=100.0, rerank_m=600,
              final_k=10, mini_batch=64, epsilon=0.1, beta=2, ref_compat=ref_compat)
    p = fg.SearchParams(**pd)
    eids, ed = oracle.coarse(index["centroids"], q, p.top_m)
    idx = fg.IVFPQIndex.from_arrays(index, base)
    ti, td, tc, cc = fg.run_gpu_batch_logic(idx, q, eids.view(np.int32), ed, p)
    oi, od, oc, st = oracle.batch_logic(index, q, eids, ed, **pd)
    if coeff > 10:
        assert (st["count"] > 4096).all()
    np.testing.assert_array_equal(_np(cc), st["count"])
    np.testing.assert_array_equal(_np(tc), oc)
    np.testing.assert_array_equal(_np(td), od)
    np.testing.assert_array_equal(_np(ti), oi)


@pytest.mark.parametrize("dim,pq_m,sample", [(128, 32, 6000), (96, 48, 50000)])
def test_pq_training_equals_reference_codebook(fg, dim, pq_m, sample):
    """fg_pq_train writes the codebook the reference's own
    train_residual_pq_codebooks (pq_utils.h:77-138, oracle/_ref) writes."""
    if oracle.ref_lib("pq", dim, pq_m) is None:
        pytest.skip("oracle/_ref not built")
    from fusiongpu_b200 import datasets as ds
    spec = ds.dataclasses.replace(ds.scaled(ds.C1, 20000, 10, n_centres=16), dim=dim)
    base, _ = ds.generate(spec)
    cen = oracle.kmeans(base, 40, 3)
    a = oracle.assign(base, cen)
    cb = fg.train_residual_pq_codebooks(torch.from_numpy(base).cuda(), torch.from_numpy(a).cuda(),
                                        torch.from_numpy(cen).cuda(), pq_m, sample, 6)
    np.testing.assert_array_equal(_np(cb), oracle.ref_pq_train(base, a, cen, pq_m, sample, 6))
