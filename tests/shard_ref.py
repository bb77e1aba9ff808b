"""TEST INFRASTRUCTURE: host statements of the sharded search's exchange step
(the merge that fg_merge_topk performs on the GPU) and of the sharded
semantics with the CPU oracle."""
import numpy as np

from fusiongpu_b200.sharded import partition_lists, shard_arrays


def merge_topk_host(dists: np.ndarray, ids: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Host statement of fg_merge_topk: [nshards][nq][k] -> [nq][k] by
    (distance, id as unsigned, so padding id -1 sorts last)."""
    ns, nq, kk = dists.shape
    d = np.transpose(dists, (1, 0, 2)).reshape(nq, ns * kk)
    i = np.transpose(ids, (1, 0, 2)).reshape(nq, ns * kk)
    out_i = np.empty((nq, k), np.int32)
    out_d = np.empty((nq, k), np.float32)
    for q in range(nq):
        order = np.lexsort((i[q].astype(np.uint32), d[q]))[:k]
        out_i[q] = i[q][order]
        out_d[q] = d[q][order]
    return out_i, out_d


def pack_keys_host(ids: np.ndarray, dists: np.ndarray) -> np.ndarray:
    """Host statement of fg_pack_topk (without a map): orderable distance bits
    in the high word (sign set: all bits flipped; else the sign bit set), the
    id as unsigned in the low word."""
    u = np.ascontiguousarray(dists, np.float32).view(np.uint32).astype(np.uint64)
    hi = np.where(u & 0x80000000, ~u & 0xFFFFFFFF, u | 0x80000000)
    return ((hi << np.uint64(32)) | ids.astype(np.uint32).astype(np.uint64)).view(np.int64)


def merge_keys_host(keys: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Host statement of fg_merge_topk_keys: [nshards][nq][k] keys -> the k
    smallest per query, unpacked."""
    ns, nq, kk = keys.shape
    u = np.transpose(keys.view(np.uint64), (1, 0, 2)).reshape(nq, ns * kk)
    top = np.sort(u, axis=1)[:, :k]
    hi = (top >> np.uint64(32)).astype(np.uint32)
    bits = np.where(hi & 0x80000000, hi & 0x7FFFFFFF, ~hi).astype(np.uint32)
    return (top & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.int32), bits.view(np.float32)


def oracle_sharded_search(index: dict, base: np.ndarray, queries: np.ndarray, world: int, **params):
    """The sharded semantics restated with the CPU oracle: per-shard search,
    global ids, host merge."""
    import oracle
    owner = partition_lists(np.diff(np.asarray(index["offsets"], dtype=np.int64)), world)
    ds, is_ = [], []
    for r in range(world):
        shard, sbase, l2g = shard_arrays(index, base, owner, r)
        if l2g.size == 0:
            nq, k = queries.shape[0], params["final_k"]
            ds.append(np.full((nq, k), np.finfo(np.float32).max, np.float32))
            is_.append(np.full((nq, k), -1, np.int32))
            continue
        li, ld = oracle.search(shard, sbase, queries, **params)
        gi = np.where((li >= 0) & (li < l2g.size), l2g[np.clip(li, 0, l2g.size - 1)], -1).astype(np.int32)
        ds.append(ld)
        is_.append(gi)
    return merge_topk_host(np.stack(ds), np.stack(is_), params["final_k"])


def oracle_sharded_graph(data: np.ndarray, queries: np.ndarray, world: int, build: dict, search: dict):
    """Graph sharded by rows, restated with the CPU oracle: each shard's graph
    and entry points built on its own rows (IVF lists capped at rows/4),
    per-shard search, global ids = local + first row, host merge."""
    import oracle
    from fusiongpu_b200.sharded import graph_shard_rows
    n = data.shape[0]
    ds, is_ = [], []
    for r in range(world):
        lo, hi = graph_shard_rows(n, world, r)
        part = np.ascontiguousarray(data[lo:hi])
        b = dict(build, nlist=max(1, min(build["nlist"], part.shape[0] // 4)))
        g, ec, en = oracle.graph_build(part.astype(np.float32), entries=True, **b)
        li, ld, _ = oracle.graph_search(part, g, queries, entry_centroids=ec, entry_nodes=en, **search)
        ds.append(ld)
        is_.append(np.where(li >= 0, li + lo, -1).astype(np.int32))
    return merge_topk_host(np.stack(ds), np.stack(is_), search["k"])
