"""Graph index (C4): fixed-degree k-NN graph build and CAGRA-style search on
the GPU, through the C ABI (fg_graph_build / fg_graph_search).

The reference has no graph index of its own (it searches a cuVS CAGRA graph
over its centroids, cagra_adapter.cuh:10-68); this follows the CAGRA design
for the C4 configuration: 1M fp16 vectors, inner product, degree 64, itopk
128, search width 4.
"""
from __future__ import annotations

import ctypes as C
import dataclasses

import torch

from . import _lib
from .index import _p, _stream

METRICS = {"l2": 0, "ip": 1}
DTYPES = {torch.float32: 0, torch.float16: 1}


@dataclasses.dataclass
class GraphBuildParams:
    graph_degree: int = 64
    intermediate_degree: int = 128
    nlist: int = 1024
    probe_lists: int = 8
    kmeans_iters: int = 10
    seed: int = 42
    metric: str = "ip"

    def c(self) -> _lib.GraphBuildParams:
        return _lib.GraphBuildParams(self.graph_degree, self.intermediate_degree, self.nlist, self.probe_lists,
                                     self.kmeans_iters, self.seed, METRICS[self.metric])


@dataclasses.dataclass
class GraphSearchParams:
    itopk: int = 128
    search_width: int = 4
    max_iterations: int = 0
    k: int = 10
    seed: int = 7
    metric: str = "ip"
    entry_probes: int = 0  # seeds from the nearest IVF lists of the build (0: random seeds only)

    def c(self) -> _lib.GraphSearchParams:
        return _lib.GraphSearchParams(self.itopk, self.search_width, self.max_iterations, self.k, self.seed,
                                      METRICS[self.metric], self.entry_probes)

    def replace(self, **kw) -> "GraphSearchParams":
        return dataclasses.replace(self, **kw)


class GraphIndex:
    """Vectors [n][dim] (fp16 or fp32, on the GPU), their graph [n][degree]
    and, from the build, the entry points (IVF centroids and list medoids)."""

    def __init__(self, data: torch.Tensor, graph: torch.Tensor, entry_centroids: torch.Tensor | None = None,
                 entry_nodes: torch.Tensor | None = None):
        if data.dtype not in DTYPES:
            raise TypeError("graph vectors must be float16 or float32")
        self.data = data.contiguous()
        self.graph = graph.contiguous().to(torch.int32)
        self.degree = int(graph.shape[1])
        self.entry_centroids = entry_centroids
        self.entry_nodes = entry_nodes
        self._ws = None

    @classmethod
    def build(cls, data: torch.Tensor, params: GraphBuildParams | None = None) -> "GraphIndex":
        params = params or GraphBuildParams()
        data = data.contiguous()
        n, dim = data.shape
        graph = torch.empty((n, params.graph_degree), dtype=torch.int32, device=data.device)
        ec = torch.empty((params.nlist, dim), dtype=torch.float32, device=data.device)
        en = torch.empty(params.nlist, dtype=torch.int32, device=data.device)
        _lib.call("fg_graph_build", _p(data), DTYPES[data.dtype], n, dim, C.byref(params.c()), _p(graph), _p(ec),
                  _p(en), _stream())
        return cls(data, graph, ec, en)

    def search(self, queries: torch.Tensor, params: GraphSearchParams | None = None, counters: bool = False):
        """Top-k ids [nq][k] and distances (IP: -dot), optionally the device
        counters (distance evaluations, expanded nodes, failed index checks)."""
        params = params or GraphSearchParams()
        q = queries.to(self.data.dtype).contiguous()
        nq = q.shape[0]
        ids = torch.empty((nq, params.k), dtype=torch.int32, device=self.data.device)
        d = torch.empty((nq, params.k), dtype=torch.float32, device=self.data.device)
        cnt = torch.zeros(3, dtype=torch.int64, device=self.data.device) if counters else None
        n, dim = self.data.shape
        ne = 0 if self.entry_nodes is None else int(self.entry_nodes.numel())
        if params.entry_probes and not ne:
            raise ValueError("entry_probes needs the entry points of GraphIndex.build")
        cp = params.c()
        need = _lib.size_query("fg_graph_search_workspace_size", DTYPES[self.data.dtype], dim, nq, ne, C.byref(cp))
        if need and (self._ws is None or self._ws.numel() < need):
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.data.device)
        ws = self._ws if need else None
        _lib.call("fg_graph_search", _p(self.data), DTYPES[self.data.dtype], n, dim, _p(self.graph), self.degree,
                  _p(self.entry_centroids), _p(self.entry_nodes), ne, _p(q), nq, C.byref(cp), _p(ids), _p(d),
                  _p(cnt), _p(ws), 0 if ws is None else ws.numel(), _stream())
        return (ids, d, cnt) if counters else (ids, d)


def knn_ip(base: torch.Tensor, queries: torch.Tensor, k: int):
    """Exact inner-product ground truth (fp32 arithmetic on the vectors as given)."""
    b = base.float().contiguous()
    q = queries.float().contiguous()
    ws = torch.empty(_lib.size_query("fg_knn_workspace_size", b.shape[0], b.shape[1], q.shape[0], k),
                     dtype=torch.uint8, device=b.device)
    ids = torch.empty((q.shape[0], k), dtype=torch.int32, device=b.device)
    d = torch.empty((q.shape[0], k), dtype=torch.float32, device=b.device)
    _lib.call("fg_knn", _p(b), b.shape[0], b.shape[1], _p(q), q.shape[0], k, METRICS["ip"], _p(ids), _p(d), _p(ws),
              ws.numel(), _stream())
    return ids, d
