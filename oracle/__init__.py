"""TEST INFRASTRUCTURE ONLY: ctypes bindings to the CPU oracle (liboracle.so)
and to the reference's own code compiled into ``oracle/_ref`` (when built).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package; the product (``fusiongpu_b200``) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
_lib = None


class Index(C.Structure):
    _fields_ = [("dim", C.c_int), ("pq_m", C.c_int), ("sub_dim", C.c_int), ("nlist", C.c_int),
                ("total", C.c_int), ("codebook", C.c_void_p), ("offsets", C.c_void_p),
                ("ids", C.c_void_p), ("codes", C.c_void_p), ("centroids", C.c_void_p)]


class Params(C.Structure):
    _fields_ = [("top_m", C.c_int), ("p1_lists", C.c_int), ("limit_k", C.c_int),
                ("threshold_coeff", C.c_float), ("prune_ratio", C.c_float),
                ("rerank_m", C.c_int), ("final_k", C.c_int), ("mini_batch", C.c_int),
                ("epsilon", C.c_float), ("beta", C.c_int), ("ref_compat", C.c_int)]


class QStat(C.Structure):
    _fields_ = [("count", C.c_int32), ("p2_overflow", C.c_int32), ("threshold", C.c_float)]


def build(quiet: bool = True) -> str:
    """Compile liboracle.so (gcc) if missing or stale."""
    so = os.path.join(HERE, "liboracle.so")
    src = [os.path.join(HERE, f) for f in ("fg_oracle.c", "fg_oracle.h", "Makefile")]
    if not os.path.exists(so) or any(os.path.getmtime(s) > os.path.getmtime(so) for s in src):
        subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL if quiet else None)
    return so


def lib():
    global _lib
    if _lib is None:
        so = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(so):
            build()
        _lib = C.CDLL(so)
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be C-contiguous"
    return C.c_void_p(a.ctypes.data)


def _check(rc: int, what: str):
    if rc != 0:
        raise RuntimeError(f"oracle {what} failed with status {rc}")


def make_index(index) -> tuple[Index, list]:
    """``index`` is a dict with codebook/offsets/ids/codes/centroids numpy arrays."""
    keep = [np.ascontiguousarray(index[k]) for k in ("codebook", "offsets", "ids", "codes", "centroids")]
    cb, off, ids, codes, cen = keep
    dim = cen.shape[1]
    pq_m = codes.shape[1]
    s = Index(dim, pq_m, dim // pq_m, cen.shape[0], ids.shape[0], *[C.c_void_p(a.ctypes.data) for a in keep])
    return s, keep


def make_params(**kw) -> Params:
    d = default_params()
    d.update(kw)
    return Params(d["top_m"], d["p1_lists"], d["limit_k"], d["threshold_coeff"], d["prune_ratio"],
                  d["rerank_m"], d["final_k"], d["mini_batch"], d["epsilon"], d["beta"],
                  int(d["ref_compat"]))


def default_params() -> dict:
    """Reference defaults (defs.h:17-41, search_pipeline.cu:562-570)."""
    return dict(top_m=20, p1_lists=12, limit_k=50, threshold_coeff=1.0, prune_ratio=100.0,
                rerank_m=10000, final_k=10, mini_batch=128, epsilon=0.1, beta=2, ref_compat=True)


def coarse(centroids, queries, top_m, nthreads=0):
    centroids = np.ascontiguousarray(centroids, np.float32)
    queries = np.ascontiguousarray(queries, np.float32)
    nq = queries.shape[0]
    ids = np.empty((nq, top_m), np.uint32)
    d = np.empty((nq, top_m), np.float32)
    _check(lib().fgo_coarse(_p(centroids), centroids.shape[0], centroids.shape[1], _p(queries), nq,
                            top_m, _p(ids), _p(d), nthreads), "coarse")
    return ids, d


def lut(residual, codebook, pq_m):
    residual = np.ascontiguousarray(residual, np.float32)
    codebook = np.ascontiguousarray(codebook, np.float32)
    out = np.empty((pq_m, 256), np.float32)
    lib().fgo_lut(_p(residual), _p(codebook), pq_m, residual.shape[0] // pq_m, _p(out))
    return out


def batch_logic(index, queries, probe_ids, probe_dists, nthreads=0, **params):
    s, keep = make_index(index)
    p = make_params(**params)
    queries = np.ascontiguousarray(queries, np.float32)
    probe_ids = np.ascontiguousarray(probe_ids, np.uint32)
    probe_dists = np.ascontiguousarray(probe_dists, np.float32)
    nq = queries.shape[0]
    rm = p.rerank_m
    tid = np.empty((nq, rm), np.int32)
    td = np.empty((nq, rm), np.float32)
    tc = np.empty(nq, np.int32)
    st = (QStat * nq)()
    _check(lib().fgo_batch_logic(C.byref(s), _p(queries), nq, _p(probe_ids), _p(probe_dists),
                                 C.byref(p), _p(tid), _p(td), _p(tc), st, nthreads), "batch_logic")
    stats = np.array([(x.count, x.p2_overflow, x.threshold) for x in st],
                     dtype=[("count", np.int32), ("p2_overflow", np.int32), ("threshold", np.float32)])
    return tid, td, tc, stats


def rerank(queries, top_ids, top_counts, base, nthreads=0, **params):
    p = make_params(**params)
    queries = np.ascontiguousarray(queries, np.float32)
    top_ids = np.ascontiguousarray(top_ids, np.int32)
    top_counts = np.ascontiguousarray(top_counts, np.int32)
    base = np.ascontiguousarray(base, np.float32)
    nq = queries.shape[0]
    k = p.final_k
    oi = np.empty((nq, k), np.int32)
    od = np.empty((nq, k), np.float32)
    _check(lib().fgo_rerank(_p(queries), nq, queries.shape[1], _p(top_ids), _p(top_counts), _p(base),
                            C.c_int64(base.shape[0]), C.byref(p), _p(oi), _p(od), nthreads), "rerank")
    return oi, od


def search(index, base, queries, nthreads=0, **params):
    s, keep = make_index(index)
    p = make_params(**params)
    queries = np.ascontiguousarray(queries, np.float32)
    base = np.ascontiguousarray(base, np.float32)
    nq = queries.shape[0]
    oi = np.empty((nq, p.final_k), np.int32)
    od = np.empty((nq, p.final_k), np.float32)
    _check(lib().fgo_search(C.byref(s), _p(base), C.c_int64(base.shape[0]), _p(queries), nq, C.byref(p),
                            _p(oi), _p(od), nthreads), "search")
    return oi, od


def knn_exact(base, queries, k, nthreads=0):
    base = np.ascontiguousarray(base, np.float32)
    queries = np.ascontiguousarray(queries, np.float32)
    nq = queries.shape[0]
    oi = np.empty((nq, k), np.int32)
    od = np.empty((nq, k), np.float32)
    _check(lib().fgo_knn_exact(_p(base), C.c_int64(base.shape[0]), base.shape[1], _p(queries), nq, k,
                               _p(oi), _p(od), nthreads), "knn_exact")
    return oi, od


class TuneResult(C.Structure):
    _fields_ = [("top_m", C.c_int32), ("p1_lists", C.c_int32), ("limit_k", C.c_int32),
                ("threshold_coeff", C.c_float), ("coverage_at_elbow", C.c_float), ("n_ranked", C.c_int32),
                ("n_in_p1", C.c_int32), ("n_ratios", C.c_int32)]


def tune(index, base, queries, gt, nthreads=0):
    """The tuner's statistics for given sample queries and ground truth
    [nq][k].  Returns (result dict, cluster_ranks, pq_ranks, exact_ranks,
    ratios)."""
    base = np.ascontiguousarray(base, np.float32)
    queries = np.ascontiguousarray(queries, np.float32)
    gt = np.ascontiguousarray(gt, np.int32)
    nq, k = gt.shape
    ix, keep = make_index(index)
    r = TuneResult()
    cr = np.empty((nq, k), np.int32)
    pr = np.empty((nq, k), np.int32)
    er = np.empty((nq, k), np.int32)
    ra = np.empty(nq, np.float32)
    _check(lib().fgo_tune(C.byref(ix), _p(base), C.c_int64(base.shape[0]), _p(queries), nq, _p(gt), k,
                          C.byref(r), _p(cr), _p(pr), _p(er), _p(ra), nthreads), "tune")
    del keep
    res = {f: getattr(r, f) for f, _ in TuneResult._fields_}
    return res, cr, pr, er, ra


def mt19937(seed: int, skip: int = 0) -> int:
    lib().fgo_mt19937_first.restype = C.c_uint32
    return int(lib().fgo_mt19937_first(C.c_uint32(seed), skip))


def std_shuffle(n: int, seed: int) -> np.ndarray:
    """std::shuffle(0..n-1, std::mt19937(seed)) as libstdc++ performs it."""
    a = np.arange(n, dtype=np.int32)
    lib().fgo_std_shuffle(_p(a), C.c_int64(n), C.c_uint32(seed))
    return a


def pq_sample_rows(n: int, sample: int, pq_m: int) -> tuple[np.ndarray, np.ndarray]:
    """(rows [S], init [pq_m][256]) that pq_train samples and seeds with."""
    S = min(sample, n)
    rows = np.empty(S, np.int32)
    init = np.empty((pq_m, 256), np.int32)
    _check(lib().fgo_pq_sample_rows(C.c_int64(n), C.c_int64(S), pq_m, _p(rows), _p(init)), "pq_sample_rows")
    return rows, init


def ref_std_shuffle(n: int, seed: int):
    """std::shuffle from the C++ standard library itself (oracle/_ref), or None."""
    for f in sorted(os.listdir(REF_DIR)) if os.path.isdir(REF_DIR) else []:
        if f.startswith("libref_pq_"):
            L = C.CDLL(os.path.join(REF_DIR, f))
            if not hasattr(L, "ref_std_shuffle"):
                return None
            out = np.empty(n, np.int32)
            L.ref_std_shuffle(n, C.c_uint(seed), _p(out))
            return out
    return None


def kmeans(data, k, iters, seed=42, nthreads=0):
    data = np.ascontiguousarray(data, np.float32)
    cen = np.empty((k, data.shape[1]), np.float32)
    _check(lib().fgo_kmeans(_p(data), C.c_int64(data.shape[0]), data.shape[1], k, iters,
                            C.c_uint32(seed), _p(cen), nthreads), "kmeans")
    return cen


def kmeans_init(data, k, seed=42):
    data = np.ascontiguousarray(data, np.float32)
    cen = np.empty((k, data.shape[1]), np.float32)
    _check(lib().fgo_kmeans_init(_p(data), C.c_int64(data.shape[0]), data.shape[1], k,
                                 C.c_uint32(seed), _p(cen)), "kmeans_init")
    return cen


def assign(data, centroids, nthreads=0):
    data = np.ascontiguousarray(data, np.float32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    out = np.empty(data.shape[0], np.int32)
    _check(lib().fgo_assign(_p(data), C.c_int64(data.shape[0]), data.shape[1], _p(centroids),
                            centroids.shape[0], _p(out), nthreads), "assign")
    return out


def kmeans_update(data, assignment, centroids):
    data = np.ascontiguousarray(data, np.float32)
    assignment = np.ascontiguousarray(assignment, np.int32)
    cen = np.array(centroids, np.float32, copy=True, order="C")
    cnt = np.empty(cen.shape[0], np.int32)
    _check(lib().fgo_kmeans_update(_p(data), C.c_int64(data.shape[0]), data.shape[1], _p(assignment),
                                   cen.shape[0], _p(cen), _p(cnt)), "kmeans_update")
    return cen, cnt


def pq_train(data, assignment, centroids, pq_m, sample=50000, iters=8, nthreads=0):
    data = np.ascontiguousarray(data, np.float32)
    assignment = np.ascontiguousarray(assignment, np.int32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    d = data.shape[1]
    cb = np.empty((pq_m, 256, d // pq_m), np.float32)
    _check(lib().fgo_pq_train(_p(data), C.c_int64(data.shape[0]), d, _p(assignment), _p(centroids),
                              pq_m, sample, iters, _p(cb), nthreads), "pq_train")
    return cb


def pq_encode(data, assignment, centroids, codebook, nthreads=0):
    data = np.ascontiguousarray(data, np.float32)
    assignment = np.ascontiguousarray(assignment, np.int32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    codebook = np.ascontiguousarray(codebook, np.float32)
    pq_m = codebook.shape[0]
    codes = np.empty((data.shape[0], pq_m), np.uint8)
    _check(lib().fgo_pq_encode(_p(data), C.c_int64(data.shape[0]), data.shape[1], _p(assignment),
                               _p(centroids), _p(codebook), pq_m, _p(codes), nthreads), "pq_encode")
    return codes


def rebalance(data, assignment, centroids, iters=15, seed=42, nthreads=0):
    """Split oversized lists (build_global.cu:62-169).  Returns the new
    assignment and centroids."""
    data = np.ascontiguousarray(data, np.float32)
    assignment = np.ascontiguousarray(assignment, np.int32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    n, d = data.shape
    out_a = np.empty(n, np.int32)
    cap = n
    out_c = np.empty((cap, d), np.float32)
    nl = C.c_int32(0)
    _check(lib().fgo_rebalance(_p(data), C.c_int64(n), d, _p(assignment), _p(centroids), centroids.shape[0],
                               iters, C.c_uint32(seed), _p(out_a), _p(out_c), cap, C.byref(nl), nthreads),
           "rebalance")
    return out_a, np.ascontiguousarray(out_c[: nl.value])


def build_index(base, nlist, pq_m, kmeans_iters=20, pq_sample=50000, pq_iters=8, nthreads=0,
                rebalance_lists=True, rebalance_iters=15, kmeans_sample=None):
    """CPU IVF-PQ build with the oracle's semantics: k-means (on every
    (n // kmeans_sample)-th row when a sample size is given), assignment of
    all rows, list rebalancing (optional), residual PQ; lists hold ids in
    ascending order.  Returns the index dict plus the assignment."""
    base = np.ascontiguousarray(base, np.float32)
    train = base
    if kmeans_sample and kmeans_sample < base.shape[0]:
        step = max(1, base.shape[0] // kmeans_sample)
        train = np.ascontiguousarray(base[np.arange(kmeans_sample) * step])
    cen = kmeans(train, nlist, kmeans_iters, 42, nthreads)
    a = assign(base, cen, nthreads)
    if rebalance_lists:
        a, cen = rebalance(base, a, cen, rebalance_iters, 42, nthreads)
    cb = pq_train(base, a, cen, pq_m, pq_sample, pq_iters, nthreads)
    codes = pq_encode(base, a, cen, cb, nthreads)
    return assemble_lists(a, codes, cen, cb), a


def assemble_lists(assignment, codes, centroids, codebook):
    """Inverted lists in list order, ids ascending inside each list
    (build_global.cu:226-240 with buckets filled in point order)."""
    nlist = centroids.shape[0]
    order = np.argsort(assignment, kind="stable").astype(np.int32)
    counts = np.bincount(assignment, minlength=nlist)
    offsets = np.zeros(nlist + 1, np.int32)
    offsets[1:] = np.cumsum(counts)
    return dict(codebook=np.ascontiguousarray(codebook, np.float32), offsets=offsets, ids=order,
                codes=np.ascontiguousarray(codes[order]), centroids=np.ascontiguousarray(centroids, np.float32))


# ---- the reference's own code (oracle/_ref) ---------------------------------

def ref_lib(kind: str, dim: int, pq_m: int):
    """Load ``_ref/libref_{gg,pq}_<dim>_<pq_m>.so`` or return None if not built."""
    so = os.path.join(REF_DIR, f"libref_{kind}_{dim}_{pq_m}.so")
    if not os.path.exists(so):
        return None
    return C.CDLL(so)


def ref_pq_train(data, assignment, centroids, pq_m, sample=50000, iters=8):
    d = data.shape[1]
    L = ref_lib("pq", d, pq_m)
    if L is None:
        return None
    data = np.ascontiguousarray(data, np.float32)
    assignment = np.ascontiguousarray(assignment, np.int32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    cb = np.empty((pq_m, 256, d // pq_m), np.float32)
    _check(L.ref_pq_train(_p(data), data.shape[0], _p(assignment), _p(centroids), centroids.shape[0],
                          sample, iters, _p(cb)), "ref_pq_train")
    return cb


def ref_pq_encode(data, assignment, centroids, codebook):
    d = data.shape[1]
    pq_m = codebook.shape[0]
    L = ref_lib("pq", d, pq_m)
    if L is None:
        return None
    data = np.ascontiguousarray(data, np.float32)
    codes = np.empty((data.shape[0], pq_m), np.uint8)
    _check(L.ref_pq_encode(_p(data), data.shape[0], _p(np.ascontiguousarray(assignment, np.int32)),
                           _p(np.ascontiguousarray(centroids, np.float32)), centroids.shape[0],
                           _p(np.ascontiguousarray(codebook, np.float32)), _p(codes)), "ref_pq_encode")
    return codes


def graph_build(data, graph_degree=64, intermediate_degree=128, nlist=64, probe_lists=4, kmeans_iters=10, seed=42,
                metric="ip", nthreads=0, entries=False):
    """The product's graph build restated on the CPU (fp32 data).  With
    entries=True also returns the entry centroids and entry nodes."""
    data = np.ascontiguousarray(data, np.float32)
    n, dim = data.shape
    g = np.empty((n, graph_degree), np.int32)
    ec = np.empty((nlist, dim), np.float32)
    en = np.empty(nlist, np.int32)
    _check(lib().fgo_graph_build(_p(data), C.c_int64(n), dim, graph_degree, intermediate_degree, nlist, probe_lists,
                                 kmeans_iters, C.c_uint32(seed), 1 if metric == "ip" else 0, _p(g), _p(ec), _p(en),
                                 nthreads), "graph_build")
    return (g, ec, en) if entries else g


def graph_search(data, graph, queries, itopk=128, search_width=4, max_iterations=0, k=10, seed=7, metric="ip",
                 nthreads=0, entry_centroids=None, entry_nodes=None, entry_probes=0):
    """The product's graph search restated on the CPU.  data/queries are
    float32 or float16 arrays.  Returns (ids, dists, [evals, expanded])."""
    dtype = 1 if data.dtype == np.float16 else 0
    data = np.ascontiguousarray(data, np.float16 if dtype else np.float32)
    queries = np.ascontiguousarray(queries, np.float16 if dtype else np.float32)
    graph = np.ascontiguousarray(graph, np.int32)
    n, dim = data.shape
    nq = queries.shape[0]
    oi = np.empty((nq, k), np.int32)
    od = np.empty((nq, k), np.float32)
    cnt = np.zeros(2, np.uint64)
    if entry_probes:
        ec = np.ascontiguousarray(entry_centroids, np.float32)
        en = np.ascontiguousarray(entry_nodes, np.int32)
        ne = en.size
    else:
        ec = np.zeros((1, dim), np.float32)
        en = np.zeros(1, np.int32)
        ne = 0
    _check(lib().fgo_graph_search(_p(data), dtype, C.c_int64(n), dim, _p(graph), graph.shape[1], _p(ec), _p(en), ne,
                                  entry_probes, _p(queries), nq, itopk, search_width, max_iterations, k,
                                  C.c_uint32(seed), 1 if metric == "ip" else 0, _p(oi), _p(od), _p(cnt), nthreads),
           "graph_search")
    return oi, od, cnt


# ---- the reference's kmeans_gpu.cuh (oracle/_ref/libref_km.so; needs a GPU) ----

def _ref_km():
    so = os.path.join(REF_DIR, "libref_km.so")
    return C.CDLL(so) if os.path.exists(so) else None


def ref_kmeans(data, k, iters):
    """run_kmeans_gpu (kmeans_gpu.cuh:234-324) on host data, or None."""
    L = _ref_km()
    if L is None:
        return None
    data = np.ascontiguousarray(data, np.float32)
    out = np.empty((k, data.shape[1]), np.float32)
    _check(L.ref_run_kmeans(_p(data), data.shape[0], data.shape[1], k, iters, _p(out)), "ref_run_kmeans")
    return out


def ref_assign(data, centroids):
    """gpu_assign_to_centroids (kmeans_gpu.cuh:367-394), or None."""
    L = _ref_km()
    if L is None:
        return None
    data = np.ascontiguousarray(data, np.float32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    out = np.empty(data.shape[0], np.int32)
    _check(L.ref_assign(_p(data), _p(centroids), data.shape[0], data.shape[1], centroids.shape[0], _p(out)),
           "ref_assign")
    return out


def ref_encode(data, assignment, centroids, codebook):
    """encode_residuals_to_pq_gpu (kmeans_gpu.cuh:450-508), or None."""
    L = _ref_km()
    if L is None:
        return None
    data = np.ascontiguousarray(data, np.float32)
    pq_m = codebook.shape[0]
    codes = np.empty((data.shape[0], pq_m), np.uint8)
    _check(L.ref_encode(_p(data), data.shape[0], data.shape[1], _p(np.ascontiguousarray(assignment, np.int32)),
                        _p(np.ascontiguousarray(centroids, np.float32)), centroids.shape[0],
                        _p(np.ascontiguousarray(codebook, np.float32)), pq_m, _p(codes)), "ref_encode")
    return codes


def ref_kmeans_cleanup():
    L = _ref_km()
    if L is not None:
        L.ref_kmeans_cleanup()
