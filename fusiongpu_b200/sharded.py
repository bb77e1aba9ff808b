"""List-sharded search across the GPUs of one box (one process per GPU).

The reference runs on one GPU only (search_pipeline.cu:560).  For a database
that is sharded by inverted list:

* every GPU keeps all centroids and the codebook (so each computes the same
  global probe list) but only the lists it owns, with their codes, ids and raw
  vectors -- lists are dealt out by longest-processing-time on list length;
* queries are broadcast; each GPU runs the whole search on its lists
  (``fg_search``: probes it does not own are empty lists), maps its shard-local
  vector ids to global ids (``fg_map_ids``) and returns its local top-k;
* ``fg_pack_topk`` maps its shard-local vector ids to global ids and packs
  each (distance, id) into one 64-bit key; ONE all-gather (NCCL over NVLink)
  puts the per-GPU [nq][k] keys side by side and ``fg_merge_topk_keys`` keeps
  the k best per query by (distance, global id).

Per-shard semantics: phase 1 / threshold / phase 2 run over each shard's share
of the probes (a probed list owned elsewhere counts as empty, as a pruned or
empty list does in the reference), so results equal "the search on each shard,
merged" -- which is what the oracle checks.
"""
from __future__ import annotations

import numpy as np


def partition_lists(list_sizes: np.ndarray, nshards: int) -> np.ndarray:
    """Owner shard of every list: longest list first to the least-loaded
    shard (ties: lower list id first, lower shard first)."""
    sizes = np.asarray(list_sizes, dtype=np.int64)
    order = np.lexsort((np.arange(sizes.size), -sizes))
    load = np.zeros(nshards, dtype=np.int64)
    owner = np.empty(sizes.size, dtype=np.int32)
    for c in order:
        s = int(np.argmin(load))
        owner[c] = s
        load[s] += sizes[c]
    return owner


def shard_arrays(index: dict, base: np.ndarray, owner: np.ndarray, rank: int):
    """The shard index of ``rank`` (same centroids/codebook, lists it does not
    own emptied), its raw vectors, and the local -> global id map."""
    off = np.asarray(index["offsets"], dtype=np.int64)
    lens = np.diff(off)
    own = owner == rank
    new_lens = np.where(own, lens, 0)
    new_off = np.zeros_like(off)
    new_off[1:] = np.cumsum(new_lens)
    sel = np.concatenate([np.arange(off[c], off[c + 1]) for c in np.flatnonzero(own)] or [np.zeros(0, np.int64)])
    l2g = np.asarray(index["ids"])[sel].astype(np.int32)
    shard = dict(codebook=index["codebook"], centroids=index["centroids"], offsets=new_off.astype(np.int32),
                 ids=np.arange(sel.size, dtype=np.int32), codes=np.ascontiguousarray(np.asarray(index["codes"])[sel]))
    return shard, np.ascontiguousarray(base[l2g]), l2g


def exchange(ids, dists, l2g, world, group, device, timings=None):
    """The exchange step shared by both sharded indexes: pack this GPU's
    [nq][k] (shard-local id, distance) into global keys, all-gather them in
    one NCCL call, merge on the device.  `timings` (a dict) receives CUDA
    events around the all-gather and the merge."""
    import torch
    import torch.distributed as dist
    from . import _lib
    from .index import _p, _stream
    nq, k = dists.shape
    keys = torch.empty((nq * k,), dtype=torch.int64, device=device)
    nmap = 0 if l2g is None else l2g.numel()
    _lib.call("fg_pack_topk", _p(ids), _p(dists), nq, k, _p(l2g), nmap, _p(keys), _stream())
    if world == 1:
        allk = keys
    else:
        allk = torch.empty((world * nq * k,), dtype=torch.int64, device=device)
        ev = _events(timings, "allgather")
        dist.all_gather_into_tensor(allk, keys, group=group)
        _events_end(ev)
    out_i = torch.empty((nq, k), dtype=torch.int32, device=device)
    out_d = torch.empty((nq, k), dtype=torch.float32, device=device)
    ev = _events(timings, "merge")
    _lib.call("fg_merge_topk_keys", _p(allk), world, nq, k, _p(out_i), _p(out_d), _stream())
    _events_end(ev)
    return out_i, out_d


def _events(timings, name):
    if timings is None:
        return None
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    timings.setdefault(name, []).append((e0, e1))
    return e1


def _events_end(e1):
    if e1 is not None:
        e1.record()


def elapsed_ms(timings) -> dict:
    """Mean milliseconds per stage of a `timings` dict (after a synchronize)."""
    return {k: sum(a.elapsed_time(b) for a, b in v) / len(v) for k, v in timings.items() if v}


class ShardedIndex:
    """This process's shard of a list-sharded IVF-PQ index on one GPU."""

    def __init__(self, index: dict, base: np.ndarray, rank: int, world: int, device="cuda", group=None):
        import torch
        from .index import IVFPQIndex
        self.rank, self.world, self.group = rank, world, group
        self.owner = partition_lists(np.diff(np.asarray(index["offsets"], dtype=np.int64)), world)
        shard, sbase, l2g = shard_arrays(index, base, self.owner, rank)
        self.local = IVFPQIndex.from_arrays(shard, sbase, device)
        self.device = self.local.device
        self.l2g = torch.from_numpy(l2g).to(self.device)
        self.n_local = int(l2g.size)

    def local_search(self, queries, params):
        """This GPU's top-k with global ids."""
        import torch
        from . import _lib
        from .index import _p, _stream
        ids, d = self.local.search(queries, params)
        gids = torch.empty_like(ids)
        _lib.call("fg_map_ids", _p(ids), ids.numel(), _p(self.l2g), self.l2g.numel(), _p(gids), _stream())
        return gids, d

    def search(self, queries, params, timings=None):
        """Global top-k on every rank: local search, one all-gather of packed
        keys, device merge.  `timings` (a dict) receives CUDA events per
        stage ("local", "allgather", "merge")."""
        import torch
        if self.n_local == 0:
            nq = queries.shape[0]
            d = torch.full((nq, params.final_k), float(np.finfo(np.float32).max), device=self.device)
            ids = torch.full((nq, params.final_k), -1, dtype=torch.int32, device=self.device)
        else:
            ev = _events(timings, "local")
            ids, d = self.local.search(queries, params)
            _events_end(ev)
        return exchange(ids, d, self.l2g, self.world, self.group, self.device, timings)


def graph_shard_rows(n: int, nshards: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of shard `rank`: contiguous, sizes differ by at most one."""
    lo = n * rank // nshards
    hi = n * (rank + 1) // nshards
    return lo, hi


class ShardedGraphIndex:
    """This process's slice of a graph index partitioned by rows across GPUs.

    Every GPU builds the graph over its own rows (fg_graph_build), searches the
    whole query batch on it (fg_graph_search), turns its local ids into global
    ones (fg_map_ids) and the per-GPU top-k lists are merged after one
    all-gather (fg_merge_topk, ascending (distance, global id); inner-product
    distances are -dot, so ascending is best first)."""

    def __init__(self, data, rank: int, world: int, build_params=None, device="cuda", group=None):
        import torch
        from .graph import GraphBuildParams, GraphIndex
        self.rank, self.world, self.group = rank, world, group
        n = data.shape[0]
        self.lo, self.hi = graph_shard_rows(n, world, rank)
        part = data[self.lo:self.hi]
        dev = torch.device(device) if not isinstance(device, torch.device) else device
        part = torch.as_tensor(part).to(dev).contiguous() if not torch.is_tensor(part) else part.to(dev).contiguous()
        bp = build_params or GraphBuildParams()
        bp = type(bp)(**{**bp.__dict__, "nlist": max(1, min(bp.nlist, part.shape[0] // 4))})
        self.local = GraphIndex.build(part, bp)
        self.device = part.device
        self.l2g = torch.arange(self.lo, self.hi, dtype=torch.int32, device=self.device)

    def local_search(self, queries, params):
        import torch
        from . import _lib
        from .index import _p, _stream
        ids, d = self.local.search(queries, params)
        gids = torch.empty_like(ids)
        _lib.call("fg_map_ids", _p(ids), ids.numel(), _p(self.l2g), self.l2g.numel(), _p(gids), _stream())
        return gids, d

    def search(self, queries, params, timings=None):
        ev = _events(timings, "local")
        ids, d = self.local.search(queries, params)
        _events_end(ev)
        return exchange(ids, d, self.l2g, self.world, self.group, self.device, timings)
