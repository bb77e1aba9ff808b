"""ctypes binding of libfusiongpu_b200.so (the C ABI in include/fusiongpu.h).

Loading fails loudly: there is no CPU or eager fallback behind this module.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
# FG_LIBRARY names another build of the same library (a variant under test)
LIB_PATH = os.environ.get("FG_LIBRARY") or os.path.join(PKG, "libfusiongpu_b200.so")

FG_OK = 0
STATUS = {0: "FG_OK", 1: "FG_ERR_INVALID_ARG", 2: "FG_ERR_CUDA", 3: "FG_ERR_WORKSPACE",
          4: "FG_ERR_UNSUPPORTED", 5: "FG_ERR_DEVICE"}


class FgError(RuntimeError):
    def __init__(self, status: int, what: str, msg: str):
        super().__init__(f"{what}: {STATUS.get(status, status)}: {msg}")
        self.status = status


class IvfpqView(C.Structure):
    _fields_ = [("pq_codebook", C.c_void_p), ("list_offsets", C.c_void_p), ("pq_codes", C.c_void_p),
                ("vector_ids", C.c_void_p), ("centroids", C.c_void_p), ("nlist", C.c_int32),
                ("dim", C.c_int32), ("pq_m", C.c_int32), ("total", C.c_int32), ("max_list_len", C.c_int32)]


class SearchParams(C.Structure):
    _fields_ = [("top_m", C.c_int32), ("p1_lists", C.c_int32), ("limit_k", C.c_int32),
                ("threshold_coeff", C.c_float), ("prune_ratio", C.c_float), ("rerank_m", C.c_int32),
                ("final_k", C.c_int32), ("mini_batch", C.c_int32), ("epsilon", C.c_float),
                ("beta", C.c_int32), ("ref_compat", C.c_int32)]


class TuneResult(C.Structure):
    _fields_ = [("top_m", C.c_int32), ("p1_lists", C.c_int32), ("limit_k", C.c_int32),
                ("threshold_coeff", C.c_float), ("coverage_at_elbow", C.c_float), ("n_ranked", C.c_int32),
                ("n_in_p1", C.c_int32), ("n_ratios", C.c_int32)]


class GraphBuildParams(C.Structure):
    _fields_ = [("graph_degree", C.c_int32), ("intermediate_degree", C.c_int32), ("nlist", C.c_int32),
                ("probe_lists", C.c_int32), ("kmeans_iters", C.c_int32), ("seed", C.c_uint32), ("metric", C.c_int32)]


class GraphSearchParams(C.Structure):
    _fields_ = [("itopk", C.c_int32), ("search_width", C.c_int32), ("max_iterations", C.c_int32), ("k", C.c_int32),
                ("seed", C.c_uint32), ("metric", C.c_int32), ("entry_probes", C.c_int32)]


# name -> argtypes (all return int status unless noted)
_P, _I32, _I64, _U32, _F, _SZ = C.c_void_p, C.c_int32, C.c_int64, C.c_uint32, C.c_float, C.c_size_t
_SIGS = {
    "fg_coarse_workspace_size": [_I32, _I32, _I32, _I32, C.POINTER(_SZ)],
    "fg_coarse_search": [_P, _I32, _I32, _P, _I32, _I32, _P, _P, _P, _SZ, _P],
    "fg_coarse_search_simt": [_P, _I32, _I32, _P, _I32, _I32, _P, _P, _P, _SZ, _P],
    "fg_coarse_search_tc": [_P, _I32, _I32, _P, _I32, _I32, _P, _P, _P, _SZ, _P, _P],
    "fg_coarse_search_noalloc": [_P, _I32, _I32, _P, _I32, _I32, _P, _P, _P],
    "fg_batch_logic": [C.POINTER(IvfpqView), _P, _I32, _P, _P, C.POINTER(SearchParams), _P, _P, _P, _P, _P],
    "fg_batch_logic_workspace_size": [C.POINTER(IvfpqView), C.POINTER(SearchParams), _I32, C.POINTER(_SZ)],
    "fg_batch_logic_ws": [C.POINTER(IvfpqView), _P, _I32, _P, _P, C.POINTER(SearchParams), _P, _P, _P, _P, _P, _SZ,
                          _P],
    "fg_probe_budget": [_P, _I32, _P, _P, _I32, _I32, _F, _P, _P, _P],
    "fg_rerank": [_P, _I32, _I32, _P, _P, _P, _I64, C.POINTER(SearchParams), _P, _P, _P],
    "fg_rerank_u8": [_P, _I32, _I32, _P, _P, _P, _I64, C.POINTER(SearchParams), _P, _P, _P],
    "fg_search_u8": [C.POINTER(IvfpqView), _P, _I64, _P, _I32, C.POINTER(SearchParams), _P, _P, _P, _SZ, _P],
    "fg_search_workspace_size": [C.POINTER(IvfpqView), C.POINTER(SearchParams), _I32, C.POINTER(_SZ)],
    "fg_search": [C.POINTER(IvfpqView), _P, _I64, _P, _I32, C.POINTER(SearchParams), _P, _P, _P, _SZ, _P],
    "fg_host_memory_mapped": [_P, C.POINTER(C.c_int32)],
    "fg_map_ids": [_P, _I64, _P, _I64, _P, _P],
    "fg_merge_topk": [_P, _P, _I32, _I32, _I32, _P, _P, _P],
    "fg_pack_topk": [_P, _P, _I32, _I32, _P, _I64, _P, _P],
    "fg_merge_topk_keys": [_P, _I32, _I32, _I32, _P, _P, _P],
    "fg_kmeans_init": [_P, _I64, _I32, _I32, _U32, _P, _P, _SZ, _P],
    "fg_assign_workspace_size": [_I64, _I32, _I32, _P],
    "fg_assign": [_P, _I64, _I32, _P, _I32, _P, _P, _SZ, _P],
    "fg_sort_by_list_workspace_size": [_I64, _I32, C.POINTER(_SZ)],
    "fg_sort_by_list": [_P, _I64, _I32, _P, _P, _P, _SZ, _P],
    "fg_kmeans_update": [_P, _I32, _P, _P, _I32, _P, _P],
    "fg_kmeans_workspace_size": [_I64, _I32, _I32, C.POINTER(_SZ)],
    "fg_kmeans": [_P, _I64, _I32, _I32, _I32, _U32, _P, _P, _SZ, _P],
    "fg_pq_train_workspace_size": [_I64, _I32, _I32, _I32, C.POINTER(_SZ)],
    "fg_pq_train": [_P, _I64, _I32, _P, _P, _I32, _I32, _I32, _P, _P, _SZ, _P],
    "fg_pq_encode": [_P, _I64, _I32, _P, _P, _P, _I32, _P, _P],
    "fg_gather_lists": [_P, _I64, _I32, _P, _P, _P, _P],
    "fg_rebalance": [_P, _I64, _I32, _P, _P, _I32, _I32, _U32, _P, _P, _I32, C.POINTER(_I32), _P],
    "fg_tune": [C.POINTER(IvfpqView), _P, _I64, _P, _I32, _P, _I32, C.POINTER(TuneResult), _P, _P, _P, _P, _P],
    "fg_tune_elbow": [_P, _I32, _I64, C.POINTER(_I32), C.POINTER(_F)],
    "fg_knn_workspace_size": [_I64, _I32, _I32, _I32, C.POINTER(_SZ)],
    "fg_graph_build": [_P, _I32, _I64, _I32, C.POINTER(GraphBuildParams), _P, _P, _P, _P],
    "fg_graph_search_workspace_size": [_I32, _I32, _I32, _I32, C.POINTER(GraphSearchParams), C.POINTER(_SZ)],
    "fg_graph_search": [_P, _I32, _I64, _I32, _P, _I32, _P, _P, _I32, _P, _I32, C.POINTER(GraphSearchParams), _P, _P,
                        _P, _P, _SZ, _P],
    "fg_knn": [_P, _I64, _I32, _P, _I32, _I32, _I32, _P, _P, _P, _SZ, _P],
    "fg_knn_exact": [_P, _I64, _I32, _P, _I32, _I32, _P, _P, _P, _SZ, _P],
}

_lib = None


def lib() -> C.CDLL:
    """Load the in-tree library (raises if it is missing: run fusiongpu_b200.build)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -m fusiongpu_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = C.c_int
        L.fg_version.restype = C.c_char_p
        L.fg_last_error.restype = C.c_char_p
        L.fg_search_params_default.argtypes = [C.POINTER(SearchParams)]
        L.fg_search_params_default.restype = None
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return ["fg_version", "fg_last_error", "fg_search_params_default", *_SIGS.keys()]


def check(status: int, what: str) -> None:
    if status != FG_OK:
        raise FgError(status, what, lib().fg_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def size_query(name: str, *args) -> int:
    out = C.c_size_t(0)
    call(name, *args, C.byref(out))
    return int(out.value)
