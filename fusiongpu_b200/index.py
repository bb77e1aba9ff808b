"""Host-side mirror of the reference's IVF-PQ interface over the C ABI.

Device memory and streams come from PyTorch (plumbing only); every kernel is
the package's own sm_100a code behind ``libfusiongpu_b200.so``.  Function
names follow the reference so a user of it finds the same entry points:

==============================  ===============================================
reference (file:line)           here
==============================  ===============================================
run_kmeans_gpu                  :func:`run_kmeans_gpu`        kmeans_gpu.cuh:234
gpu_assign_to_centroids         :func:`gpu_assign_to_centroids` kmeans_gpu.cuh:367
train_residual_pq_codebooks     :func:`train_residual_pq_codebooks` pq_utils.h:77
encode_residuals_to_pq_gpu      :func:`encode_residuals_to_pq_gpu` kmeans_gpu.cuh:450
search_cagra_index              :func:`coarse_search` (exact)  cagra_adapter.cuh:38
run_gpu_batch_logic             :func:`run_gpu_batch_logic`   gpu_global.cu:679
run_gpu_rerank                  :func:`run_gpu_rerank`        gpu_global.cu:667
IVFIndexGPU / load_ivf_index    :class:`IVFPQIndex`           defs.h:49, search_pipeline.cu:481
build_global main               :meth:`IVFPQIndex.build`      build_global.cu:21
==============================  ===============================================
"""
from __future__ import annotations

import ctypes as C
import dataclasses

import numpy as np
import torch

from . import _lib
from . import formats

INVALID_PROBE = 0xFFFFFFFF


@dataclasses.dataclass
class SearchParams:
    """Search parameters; defaults are the reference's (defs.h:17-41,
    search_pipeline.cu:562-570)."""

    top_m: int = 20
    p1_lists: int = 12
    limit_k: int = 50
    threshold_coeff: float = 1.0
    prune_ratio: float = 100.0
    rerank_m: int = 10000
    final_k: int = 10
    mini_batch: int = 128
    epsilon: float = 0.1
    beta: int = 2
    ref_compat: bool = True

    def c(self) -> _lib.SearchParams:
        return _lib.SearchParams(self.top_m, self.p1_lists, self.limit_k, self.threshold_coeff,
                                 self.prune_ratio, self.rerank_m, self.final_k, self.mini_batch,
                                 self.epsilon, self.beta, int(bool(self.ref_compat)))

    def replace(self, **kw) -> "SearchParams":
        return dataclasses.replace(self, **kw)


def _dev(x, dtype, device) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x.to(device=device, dtype=dtype).contiguous()
    return torch.from_numpy(np.ascontiguousarray(x)).to(device=device, dtype=dtype).contiguous()


def _p(t: torch.Tensor | None):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def _stream(stream: torch.cuda.Stream | None = None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


# ---- build steps ----------------------------------------------------------------

def run_kmeans_gpu(data, k: int, max_iter: int = 20, seed: int = 42, device="cuda") -> torch.Tensor:
    """Lloyd k-means (strided MT19937 seeding, exact assignment, ordered
    centroid update).  Returns centroids [k][dim] on the device."""
    x = _dev(data, torch.float32, device)
    n, d = x.shape
    cen = torch.empty((k, d), dtype=torch.float32, device=device)
    ws = _workspace(_lib.size_query("fg_kmeans_workspace_size", n, d, k), device)
    _lib.call("fg_kmeans", _p(x), n, d, k, max_iter, seed, _p(cen), _p(ws), ws.numel(), _stream())
    return cen


def gpu_assign_to_centroids(data, centroids, device="cuda") -> torch.Tensor:
    x = _dev(data, torch.float32, device)
    c = _dev(centroids, torch.float32, device)
    out = torch.empty(x.shape[0], dtype=torch.int32, device=device)
    wb = _lib.size_query("fg_assign_workspace_size", x.shape[0], x.shape[1], c.shape[0])
    ws = _workspace(wb, device)
    _lib.call("fg_assign", _p(x), x.shape[0], x.shape[1], _p(c), c.shape[0], _p(out), _p(ws), ws.numel(),
              _stream())
    return out


def sort_by_list(assign: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    n = assign.shape[0]
    order = torch.empty(n, dtype=torch.int32, device=assign.device)
    offsets = torch.empty(k + 1, dtype=torch.int32, device=assign.device)
    ws = _workspace(_lib.size_query("fg_sort_by_list_workspace_size", n, k), assign.device)
    _lib.call("fg_sort_by_list", _p(assign), n, k, _p(order), _p(offsets), _p(ws), ws.numel(), _stream())
    return order, offsets


def rebalance_lists(data, assign, centroids, iters: int = 15, seed: int = 42,
                    device="cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """Split oversized lists by local k-means (build_global.cu:62-169).
    Returns (assignment [n] int32, centroids [nlist'][dim]) on the device."""
    x = _dev(data, torch.float32, device)
    a = _dev(assign, torch.int32, device)
    c = _dev(centroids, torch.float32, device)
    n, d = x.shape
    k = c.shape[0]
    out_a = torch.empty(n, dtype=torch.int32, device=device)
    cap = min(n, 4 * k)
    while True:
        out_c = torch.empty((max(cap, 1), d), dtype=torch.float32, device=device)
        nl = C.c_int32(0)
        rc = _lib.lib().fg_rebalance(_p(x), n, d, _p(a), _p(c), k, iters, seed, _p(out_a), _p(out_c), cap,
                                     C.byref(nl), _stream())
        if rc == 3 and nl.value > cap:  # FG_ERR_WORKSPACE: more lists than cap
            cap = nl.value
            continue
        _lib.check(rc, "fg_rebalance")
        return out_a, out_c[: nl.value].contiguous()


def train_residual_pq_codebooks(data, vec_cluster_ids, clusters, pq_m: int, sample_size: int = 50000,
                                max_iter: int = 8, device="cuda") -> torch.Tensor:
    x = _dev(data, torch.float32, device)
    a = _dev(vec_cluster_ids, torch.int32, device)
    c = _dev(clusters, torch.float32, device)
    n, d = x.shape
    cb = torch.empty((pq_m, 256, d // pq_m), dtype=torch.float32, device=device)
    ws = _workspace(_lib.size_query("fg_pq_train_workspace_size", n, d, pq_m, sample_size), device)
    _lib.call("fg_pq_train", _p(x), n, d, _p(a), _p(c), pq_m, sample_size, max_iter, _p(cb), _p(ws),
              ws.numel(), _stream())
    return cb


def encode_residuals_to_pq_gpu(data, cluster_ids, centroids, codebook, device="cuda") -> torch.Tensor:
    x = _dev(data, torch.float32, device)
    a = _dev(cluster_ids, torch.int32, device)
    c = _dev(centroids, torch.float32, device)
    cb = _dev(codebook, torch.float32, device)
    pq_m = cb.shape[0]
    codes = torch.empty((x.shape[0], pq_m), dtype=torch.uint8, device=device)
    _lib.call("fg_pq_encode", _p(x), x.shape[0], x.shape[1], _p(a), _p(c), _p(cb), pq_m, _p(codes), _stream())
    return codes


# ---- search steps -----------------------------------------------------------------

def coarse_search(queries, centroids, top_m: int, device="cuda", path: str = "auto"):
    """Exact nearest `top_m` centroids (stands in for search_cagra_index).
    Returns (ids uint32 as int32 tensor, squared distances); with path="tc"
    also the number of queries that needed the exact fallback.
    path: "auto" (tensor cores when the shape allows), "tc", "simt"."""
    q = _dev(queries, torch.float32, device)
    c = _dev(centroids, torch.float32, device)
    nq, d = q.shape
    ids = torch.empty((nq, top_m), dtype=torch.int32, device=device)
    dist = torch.empty((nq, top_m), dtype=torch.float32, device=device)
    ws = _workspace(_lib.size_query("fg_coarse_workspace_size", c.shape[0], d, nq, top_m), device)
    if path == "tc":
        nfb = C.c_int32(0)
        _lib.call("fg_coarse_search_tc", _p(c), c.shape[0], d, _p(q), nq, top_m, _p(ids), _p(dist), _p(ws),
                  ws.numel(), C.byref(nfb), _stream())
        return ids, dist, int(nfb.value)
    name = "fg_coarse_search_simt" if path == "simt" else "fg_coarse_search"
    _lib.call(name, _p(c), c.shape[0], d, _p(q), nq, top_m, _p(ids), _p(dist), _p(ws), ws.numel(), _stream())
    return ids, dist


def knn_exact(base, queries, k: int, device="cuda") -> tuple[torch.Tensor, torch.Tensor]:
    b = _dev(base, torch.float32, device)
    q = _dev(queries, torch.float32, device)
    ids = torch.empty((q.shape[0], k), dtype=torch.int32, device=device)
    dist = torch.empty((q.shape[0], k), dtype=torch.float32, device=device)
    ws = _workspace(_lib.size_query("fg_knn_workspace_size", b.shape[0], b.shape[1], q.shape[0], k), device)
    _lib.call("fg_knn_exact", _p(b), b.shape[0], b.shape[1], _p(q), q.shape[0], k, _p(ids), _p(dist), _p(ws),
              ws.numel(), _stream())
    return ids, dist


def _base_tensor(base, device) -> torch.Tensor | None:
    """Raw vectors for the rerank: uint8 stays uint8 (fg_search_u8), anything
    else becomes float32."""
    if base is None:
        return None
    t = base if torch.is_tensor(base) else torch.from_numpy(np.ascontiguousarray(base))
    if t.dtype == torch.uint8:
        return t.to(device).contiguous()
    return t.to(device=device, dtype=torch.float32).contiguous()


def kmeans_sample_rows(n: int, sample: int) -> np.ndarray:
    """Rows k-means trains on when it is given a sample: every
    (n // sample)-th row, `sample` of them."""
    step = max(1, n // sample)
    return (np.arange(min(n, sample), dtype=np.int64) * step)


class IVFPQIndex:
    """A device-resident IVF-PQ index (the reference's IVFIndexGPU plus the raw
    base vectors SearchPipeline keeps for the rerank; float32, or uint8 for
    byte-valued datasets)."""

    def __init__(self, centroids, codebook, offsets, ids, codes, base=None, device="cuda"):
        self.device = torch.device(device)
        self.centroids = _dev(centroids, torch.float32, device)
        self.codebook = _dev(codebook, torch.float32, device)
        self.offsets = _dev(offsets, torch.int32, device)
        self.ids = _dev(ids, torch.int32, device)
        self.codes = _dev(codes, torch.uint8, device)
        self.base = _base_tensor(base, device)
        self.nlist, self.dim = self.centroids.shape
        self.pq_m = self.codes.shape[1]
        self.total = self.ids.shape[0]
        lens = self.offsets[1:] - self.offsets[:-1]
        self.max_list_len = int(lens.max().item()) if self.nlist else 0
        self._view = _lib.IvfpqView(self.codebook.data_ptr(), self.offsets.data_ptr(), self.codes.data_ptr(),
                                    self.ids.data_ptr(), self.centroids.data_ptr(), self.nlist, self.dim,
                                    self.pq_m, self.total, self.max_list_len)
        self._ws = None

    # -- construction ----------------------------------------------------------
    @classmethod
    def from_arrays(cls, index: dict, base=None, device="cuda") -> "IVFPQIndex":
        return cls(index["centroids"], index["codebook"], index["offsets"], index["ids"], index["codes"], base,
                   device)

    @classmethod
    def build(cls, base, nlist: int, pq_m: int, kmeans_iters: int = 20, pq_sample: int = 50000,
              pq_iters: int = 8, seed: int = 42, keep_base: bool = True, rebalance: bool = True,
              rebalance_iters: int = 15, kmeans_sample: int | None = None, device="cuda") -> "IVFPQIndex":
        """k-means -> assignment -> list rebalancing -> residual PQ training ->
        encoding -> lists (build_global.cu:21-258 without the CAGRA graph over
        centroids, which the exact coarse quantizer replaces).  The index has
        nlist lists or more when rebalancing splits some.  kmeans_sample:
        train the centroids on that many strided rows (kmeans_sample_rows),
        then assign every row (the reference trains on all rows)."""
        x = _dev(base, torch.float32, device)
        xk = x
        if kmeans_sample and kmeans_sample < x.shape[0]:
            xk = x[torch.from_numpy(kmeans_sample_rows(x.shape[0], kmeans_sample)).to(x.device)].contiguous()
        cen = run_kmeans_gpu(xk, nlist, kmeans_iters, seed, device)
        del xk
        a = gpu_assign_to_centroids(x, cen, device)
        if rebalance:
            a, cen = rebalance_lists(x, a, cen, rebalance_iters, seed, device)
            nlist = cen.shape[0]
        cb = train_residual_pq_codebooks(x, a, cen, pq_m, pq_sample, pq_iters, device)
        codes = encode_residuals_to_pq_gpu(x, a, cen, cb, device)
        order, offsets = sort_by_list(a, nlist)
        lcodes = torch.empty_like(codes)
        lids = torch.empty(x.shape[0], dtype=torch.int32, device=x.device)
        _lib.call("fg_gather_lists", _p(codes), x.shape[0], pq_m, _p(order), _p(lcodes), _p(lids), _stream())
        keep = None
        if keep_base:
            keep = base if (torch.is_tensor(base) and base.dtype == torch.uint8) or \
                (isinstance(base, np.ndarray) and base.dtype == np.uint8) else x
        idx = cls(cen, cb, offsets, lids, lcodes, keep, device)
        idx.assignment = a
        return idx

    @classmethod
    def load(cls, res_dir: str, pq_m: int, dim: int, base=None, device="cuda") -> "IVFPQIndex":
        """load_ivf_index_to_gpu (search_pipeline.cu:481-529)."""
        return cls.from_arrays(formats.load_index(res_dir, pq_m, dim), base, device)

    def save(self, res_dir: str) -> None:
        formats.save_index(res_dir, self.to_numpy())

    def to_numpy(self) -> dict:
        return dict(codebook=self.codebook.cpu().numpy(), offsets=self.offsets.cpu().numpy(),
                    ids=self.ids.cpu().numpy(), codes=self.codes.cpu().numpy(),
                    centroids=self.centroids.cpu().numpy())

    @property
    def view(self) -> _lib.IvfpqView:
        return self._view

    # -- search ------------------------------------------------------------------
    def workspace_bytes(self, nq: int, params: SearchParams) -> int:
        return _lib.size_query("fg_search_workspace_size", C.byref(self._view), C.byref(params.c()), nq)

    def workspace(self, nq: int, params: SearchParams) -> torch.Tensor:
        need = self.workspace_bytes(nq, params)
        if self._ws is None or self._ws.numel() < need:
            self._ws = _workspace(need, self.device)
        return self._ws

    def search(self, queries, params: SearchParams | None = None, out=None, stream=None, ws=None):
        """Full search: exact coarse -> candidate generation -> rerank.
        Returns (ids [nq][final_k] int32, dists [nq][final_k] float32).
        `ws` is a caller-owned uint8 device workspace of at least
        workspace_bytes(nq, params); without it the index's shared one is used
        (grown on demand, so a captured graph must pass its own)."""
        params = params or SearchParams()
        if self.base is None:
            raise ValueError("search needs the raw base vectors (build with keep_base=True)")
        q = _dev(queries, torch.float32, self.device)
        nq = q.shape[0]
        if out is None:
            ids = torch.empty((nq, params.final_k), dtype=torch.int32, device=self.device)
            dist = torch.empty((nq, params.final_k), dtype=torch.float32, device=self.device)
        else:
            ids, dist = out
        if ws is None:
            ws = self.workspace(nq, params)
        cp = params.c()
        fn = "fg_search_u8" if self.base.dtype == torch.uint8 else "fg_search"
        _lib.call(fn, C.byref(self._view), _p(self.base), self.base.shape[0], _p(q), nq, C.byref(cp),
                  _p(ids), _p(dist), _p(ws), ws.numel(), _stream(stream))
        return ids, dist

    def search_host(self, queries, params: SearchParams | None = None, out=None, chunks: int = 2,
                    zero_copy: bool | None = None, graph: bool = False, _mapped: bool | None = None,
                    _state=None):
        """Search host-resident queries into host-resident results with the
        copies overlapped: the batch is cut into `chunks` pieces on two
        streams, each stream with its own device buffers and workspace, so one
        piece's upload and download run on the copy engines while another
        piece's kernels run.  Pinned host buffers keep the copies asynchronous;
        `out` = (ids, dists) host tensors [nq][final_k].  When both are
        page-locked, contiguous and mapped into the device's address space
        (fg_host_memory_mapped), the rerank kernel writes the results into
        them directly and no download follows the search (zero_copy=None
        decides by that check, True requires it, False always copies).
        Returns them once the current stream has been made to wait for every
        piece (synchronise before reading them on the host).

        graph=True replays the whole step -- uploads, kernels and result
        writes -- as one CUDA graph, captured on the first call for these
        host buffers and parameters (the graph holds their addresses: keep
        the same pinned query and result tensors between calls and overwrite
        their contents; other buffers capture another graph).  One launch per
        call then replaces about a dozen, so host delays no longer stall the
        GPU between them."""
        params = params or SearchParams()
        if graph:
            return self._search_host_graph(queries, params, out, chunks, zero_copy)
        if self.base is None:
            raise ValueError("search needs the raw base vectors (build with keep_base=True)")
        hq = queries if isinstance(queries, torch.Tensor) and queries.dtype == torch.float32 else \
            torch.as_tensor(queries, dtype=torch.float32)
        if hq.device.type != "cpu":
            raise ValueError("search_host takes host queries")
        nq = hq.shape[0]
        chunks = max(1, min(int(chunks), nq)) if nq else 1
        per = (nq + chunks - 1) // chunks if nq else 0
        dev = self.device
        # streams, device buffers, workspaces and the C parameter block are
        # kept for the next call with the same piece size and parameters
        # (a captured graph passes the state it owns instead)
        hs = _state
        if hs is None:
            hs = getattr(self, "_host_state", None)
            if hs is None or hs[0] != self._host_key(per, params):
                self._host_state = hs = self._new_host_state(per, params)
        state, cp = hs[1], hs[2]
        cur = torch.cuda.current_stream(dev)
        for st in state:
            st["stream"].wait_stream(cur)
        pieces = [(lo, min(nq, lo + per)) for lo in range(0, nq, max(per, 1))]
        # each stream's first upload goes out before the per-call checks below
        for c, (lo, hi) in enumerate(pieces[:2]):
            st = state[c % 2]
            with torch.cuda.stream(st["stream"]):
                st["q"][:hi - lo].copy_(hq[lo:hi], non_blocking=True)
        if out is None:
            out = (torch.empty((nq, params.final_k), dtype=torch.int32).pin_memory(),
                   torch.empty((nq, params.final_k), dtype=torch.float32).pin_memory())
        hid, hdd = out
        mapped = _mapped if _mapped is not None else (_host_mapped(hid) and _host_mapped(hdd))
        if zero_copy and not mapped:
            raise ValueError("zero_copy needs contiguous, page-locked, device-mapped result tensors")
        zc = mapped if zero_copy is None else bool(zero_copy)
        fn = "fg_search_u8" if self.base.dtype == torch.uint8 else "fg_search"
        for c, (lo, hi) in enumerate(pieces):
            n = hi - lo
            st = state[c % 2]
            with torch.cuda.stream(st["stream"]):
                if c >= 2:
                    st["q"][:n].copy_(hq[lo:hi], non_blocking=True)
                oi, od = (hid[lo:hi], hdd[lo:hi]) if zc else (st["ids"], st["dd"])
                _lib.call(fn, C.byref(self._view), _p(self.base), self.base.shape[0], _p(st["q"]), n, C.byref(cp),
                          _p(oi), _p(od), _p(st["ws"]), st["ws"].numel(), _stream(st["stream"]))
                if not zc:
                    hid[lo:hi].copy_(st["ids"][:n], non_blocking=True)
                    hdd[lo:hi].copy_(st["dd"][:n], non_blocking=True)
        for st in state:
            cur.wait_stream(st["stream"])
        return hid, hdd

    @staticmethod
    def _host_key(per: int, params: SearchParams):
        return (per, *vars(params).values())

    def _new_host_state(self, per: int, params: SearchParams):
        """Two streams, each with its own device query/result buffers and
        workspace for pieces of `per` queries, plus the C parameter block."""
        dev = self.device
        ws_bytes = self.workspace_bytes(max(per, 1), params)
        state = []
        for _ in range(2):
            state.append(dict(stream=torch.cuda.Stream(device=dev),
                              q=torch.empty((max(per, 1), self.dim), dtype=torch.float32, device=dev),
                              ids=torch.empty((max(per, 1), params.final_k), dtype=torch.int32, device=dev),
                              dd=torch.empty((max(per, 1), params.final_k), dtype=torch.float32, device=dev),
                              ws=_workspace(ws_bytes, dev)))
        return (self._host_key(per, params), state, params.c())

    def _search_host_graph(self, queries, params: SearchParams, out, chunks: int, zero_copy: bool | None):
        hq = queries if isinstance(queries, torch.Tensor) and queries.dtype == torch.float32 else None
        if hq is None or hq.device.type != "cpu" or not hq.is_pinned() or not hq.is_contiguous():
            raise ValueError("search_host(graph=True) takes a contiguous pinned float32 query tensor")
        nq = hq.shape[0]
        if out is None:
            raise ValueError("search_host(graph=True) needs the result tensors (out=) it is captured for")
        hid, hdd = out
        if not (hid.is_pinned() and hdd.is_pinned()):
            raise ValueError("search_host(graph=True) needs pinned result tensors")
        key = (hq.data_ptr(), nq, hid.data_ptr(), hdd.data_ptr(), tuple(hid.shape), int(chunks), zero_copy,
               *vars(params).values())
        graphs = self.__dict__.setdefault("_host_graphs", {})
        entry = graphs.get(key)
        if entry is None:
            mapped = _host_mapped(hid) and _host_mapped(hdd)
            nch = max(1, min(int(chunks), nq)) if nq else 1
            per = (nq + nch - 1) // nch if nq else 0
            # the graph owns its streams, buffers and workspace: the addresses it
            # replays stay valid whatever other calls do with theirs
            state = self._new_host_state(per, params)
            # an eager call first: it sets the kernels' shared-memory attributes
            self.search_host(hq, params, out, chunks, zero_copy, _mapped=mapped, _state=state)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.search_host(hq, params, out, chunks, zero_copy, _mapped=mapped, _state=state)
            if len(graphs) >= 8:
                graphs.pop(next(iter(graphs)))
            graphs[key] = entry = (g, state)
        entry[0].replay()
        return hid, hdd

    def capture(self, nq: int, params: SearchParams | None = None) -> "SearchGraph":
        """A CUDA graph of one search of `nq` queries with these parameters,
        for replay in launch-bound (small-batch) serving: the search needs no
        allocation and no host synchronisation once its workspace exists."""
        return SearchGraph(self, nq, params or SearchParams())

    def coarse(self, queries, top_m: int):
        return coarse_search(queries, self.centroids, top_m, self.device)

    def batch_logic(self, queries, probe_ids, probe_dists, params: SearchParams):
        return run_gpu_batch_logic(self, queries, probe_ids, probe_dists, params)

    def rerank(self, queries, top_ids, top_counts, params: SearchParams):
        return run_gpu_rerank(queries, top_ids, top_counts, self.base, params, self.device)


def _host_mapped(t) -> bool:
    """Whether kernels can write host tensor t in place: contiguous,
    page-locked and mapped at its own address (fg_host_memory_mapped)."""
    if t.device.type != "cpu" or not t.is_contiguous() or not t.is_pinned() or t.numel() == 0:
        return False
    m = C.c_int32(0)
    _lib.call("fg_host_memory_mapped", C.c_void_p(t.data_ptr()), C.byref(m))
    return m.value == 1


class SearchGraph:
    """One captured search: copy queries into `self.queries`, call replay(),
    read `self.ids` / `self.dists` (all on the index's device)."""

    def __init__(self, index: IVFPQIndex, nq: int, params: SearchParams):
        self.index, self.params = index, params
        dev = index.device
        self.queries = torch.zeros((nq, index.dim), dtype=torch.float32, device=dev)
        self.ids = torch.empty((nq, params.final_k), dtype=torch.int32, device=dev)
        self.dists = torch.empty((nq, params.final_k), dtype=torch.float32, device=dev)
        # the graph's own workspace, allocated before capture and held as long as
        # the graph: the index's shared workspace may be replaced by a larger
        # search, and eager searches on other streams use it concurrently
        self.ws = _workspace(index.workspace_bytes(nq, params), dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # warm up (attributes, tensor maps) outside the graph
            index.search(self.queries, params, out=(self.ids, self.dists), ws=self.ws)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            index.search(self.queries, params, out=(self.ids, self.dists), ws=self.ws)

    def replay(self, queries=None):
        if queries is not None:
            self.queries.copy_(queries, non_blocking=True)
        self.graph.replay()
        return self.ids, self.dists


def run_gpu_batch_logic(index: IVFPQIndex, queries, probe_ids, probe_dists, params: SearchParams):
    """Candidate generation (gpu_global.cu:679-874).  Returns (top_ids,
    top_dists [nq][rerank_m], top_counts [nq], candidate_counts [nq])."""
    dev = index.device
    q = _dev(queries, torch.float32, dev)
    pid = _dev(probe_ids, torch.int32, dev)
    pd = _dev(probe_dists, torch.float32, dev)
    nq = q.shape[0]
    rm = params.rerank_m
    tid = torch.empty((nq, rm), dtype=torch.int32, device=dev)
    td = torch.empty((nq, rm), dtype=torch.float32, device=dev)
    tc = torch.empty(nq, dtype=torch.int32, device=dev)
    cc = torch.empty(nq, dtype=torch.int32, device=dev)
    cp = params.c()
    wb = _lib.size_query("fg_batch_logic_workspace_size", C.byref(index.view), C.byref(cp), nq)
    ws = _workspace(wb, dev)
    _lib.call("fg_batch_logic_ws", C.byref(index.view), _p(q), nq, _p(pid), _p(pd), C.byref(cp), _p(tid), _p(td),
              _p(tc), _p(cc), _p(ws), ws.numel(), _stream())
    return tid, td, tc, cc


def run_gpu_rerank(queries, top_ids, top_counts, base, params: SearchParams, device="cuda"):
    """Exact rerank (gpu_global.cu:603-673).  Returns (ids, dists) [nq][final_k]."""
    q = _dev(queries, torch.float32, device)
    tid = _dev(top_ids, torch.int32, device)
    tc = _dev(top_counts, torch.int32, device)
    b = _base_tensor(base, device)
    nq = q.shape[0]
    ids = torch.empty((nq, params.final_k), dtype=torch.int32, device=device)
    dist = torch.empty((nq, params.final_k), dtype=torch.float32, device=device)
    cp = params.c()
    fn = "fg_rerank_u8" if b.dtype == torch.uint8 else "fg_rerank"
    _lib.call(fn, _p(q), nq, q.shape[1], _p(tid), _p(tc), _p(b), b.shape[0], C.byref(cp), _p(ids),
              _p(dist), _stream())
    return ids, dist


def recall_at(results: np.ndarray, gt: np.ndarray, k: int) -> float:
    """compute_recall (search_pipeline.cu:531-557): hits of the first k
    predicted ids (deduplicated) in the ground-truth rows, over nq*k."""
    nq = results.shape[0]
    hits = 0
    for i in range(nq):
        g = set(gt[i].tolist())
        seen = set()
        for v in results[i, :k].tolist():
            if v in seen:
                continue
            seen.add(v)
            hits += v in g
    return hits / (nq * k)
