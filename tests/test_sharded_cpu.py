"""Host logic of the list-sharded search: partitioning, shard construction,
and the exchange step with world_size 2 over gloo (CPU processes), checked
against the single-process statement of the same semantics."""
import os
import socket
import tempfile

import numpy as np
import pytest

import oracle
from fusiongpu_b200 import sharded
from fusiongpu_b200 import datasets as ds
from tests import shard_ref

P = dict(top_m=10, p1_lists=4, limit_k=40, threshold_coeff=1.0, prune_ratio=100.0, rerank_m=120, final_k=10,
         mini_batch=64, epsilon=0.1, beta=2, ref_compat=False)


def _data():
    base, q = ds.generate(ds.scaled(ds.C1, 6000, 48, n_centres=24, seed=41))
    index, _ = oracle.build_index(base, 48, 32, kmeans_iters=4, pq_sample=3000, pq_iters=4)
    return index, base, q


def test_partition_is_balanced_and_deterministic():
    rng = np.random.default_rng(0)
    sizes = rng.integers(0, 500, size=1000)
    for n in (1, 2, 3, 8):
        o = sharded.partition_lists(sizes, n)
        assert np.array_equal(o, sharded.partition_lists(sizes, n))
        load = np.bincount(o, weights=sizes, minlength=n)
        assert load.max() - load.min() <= sizes.max()


def test_shards_cover_every_vector_once():
    index, base, q = _data()
    owner = sharded.partition_lists(np.diff(index["offsets"]), 3)
    seen = []
    for r in range(3):
        shard, sbase, l2g = sharded.shard_arrays(index, base, owner, r)
        assert shard["codes"].shape[0] == l2g.size == sbase.shape[0]
        np.testing.assert_array_equal(sbase, base[l2g])
        seen.append(l2g)
    allv = np.concatenate(seen)
    assert np.array_equal(np.sort(allv), np.arange(base.shape[0]))


def test_packed_key_merge_equals_pair_merge():
    """Packing (distance, id) into one 64-bit word and merging the words
    selects what the pair merge selects, with negative distances (inner
    product), ties and -1 padding."""
    rng = np.random.default_rng(9)
    ns, nq, k = 4, 60, 12
    d = np.sort(rng.integers(-8, 8, size=(ns, nq, k)).astype(np.float32) * 0.5, axis=2)
    i = rng.permutation(ns * nq * k).reshape(ns, nq, k).astype(np.int32)
    d[:, :, -2:] = np.finfo(np.float32).max
    i[:, :, -2:] = -1
    keys = np.stack([shard_ref.pack_keys_host(i[s], d[s]) for s in range(ns)])
    ki, kd = shard_ref.merge_keys_host(keys, k)
    ei, ed = shard_ref.merge_topk_host(d, i, k)
    np.testing.assert_array_equal(ki, ei)
    np.testing.assert_array_equal(kd, ed)


def test_merge_host_orders_by_distance_then_id():
    d = np.array([[[1.0, 2.0, 3.0]], [[1.0, 1.5, np.finfo(np.float32).max]]], np.float32)
    i = np.array([[[7, 3, 4]], [[2, 9, -1]]], np.int32)
    mi, md = shard_ref.merge_topk_host(d, i, 4)
    np.testing.assert_array_equal(mi[0], [2, 7, 9, 3])
    np.testing.assert_array_equal(md[0], [1.0, 1.0, 1.5, 2.0])


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    index, base, q = _data()
    owner = sharded.partition_lists(np.diff(index["offsets"]), world)
    shard, sbase, l2g = sharded.shard_arrays(index, base, owner, rank)
    li, ld = oracle.search(shard, sbase, q, **P)
    gi = np.where(li >= 0, l2g[np.clip(li, 0, l2g.size - 1)], -1).astype(np.int32)
    # the exchange is one all-gather of packed (distance key, global id) words
    tk = torch.from_numpy(shard_ref.pack_keys_host(gi, ld))
    all_k = torch.empty((world * tk.numel(),), dtype=torch.int64)
    dist.all_gather_into_tensor(all_k, tk.reshape(-1))
    mi, md = shard_ref.merge_keys_host(all_k.numpy().reshape((world,) + tuple(tk.shape)), P["final_k"])
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), ids=mi, dists=md)
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_two_rank_exchange_over_gloo():
    import torch.multiprocessing as mp
    index, base, q = _data()
    ei, ed = shard_ref.oracle_sharded_search(index, base, q, 2, **P)
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, _free_port(), d), nprocs=2, join=True)
        for r in range(2):
            f = np.load(os.path.join(d, f"rank{r}.npz"))
            np.testing.assert_array_equal(f["ids"], ei)
            np.testing.assert_array_equal(f["dists"], ed)
    # sharding changes the per-shard thresholds, not the quality much
    gt, _ = oracle.knn_exact(base, q, 10)
    rec = np.mean([len(set(ei[i]) & set(gt[i])) / 10 for i in range(q.shape[0])])
    assert rec > 0.9


# ---- graph sharded by rows --------------------------------------------------------

GB = dict(graph_degree=16, intermediate_degree=32, nlist=16, probe_lists=3, kmeans_iters=3, seed=42, metric="ip")
GS = dict(itopk=32, search_width=2, k=10, seed=5, metric="ip", entry_probes=4)


def _graph_data():
    rng = np.random.default_rng(21)
    x = rng.normal(size=(1500, 32)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    q = rng.normal(size=(12, 32)).astype(np.float32)
    return x.astype(np.float16), q.astype(np.float16)


def test_graph_shard_rows_partition():
    for n, w in ((10, 3), (1000, 8), (7, 7)):
        rows = [sharded.graph_shard_rows(n, w, r) for r in range(w)]
        assert rows[0][0] == 0 and rows[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(rows, rows[1:]))
        assert max(h - l for l, h in rows) - min(h - l for l, h in rows) <= 1


def _graph_worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    x, q = _graph_data()
    lo, hi = sharded.graph_shard_rows(x.shape[0], world, rank)
    part = np.ascontiguousarray(x[lo:hi])
    b = dict(GB, nlist=max(1, min(GB["nlist"], part.shape[0] // 4)))
    g, ec, en = oracle.graph_build(part.astype(np.float32), entries=True, **b)
    li, ld, _ = oracle.graph_search(part, g, q, entry_centroids=ec, entry_nodes=en, **GS)
    gi = np.where(li >= 0, li + lo, -1).astype(np.int32)
    tk = torch.from_numpy(shard_ref.pack_keys_host(gi, ld))
    all_k = torch.empty((world * tk.numel(),), dtype=torch.int64)
    dist.all_gather_into_tensor(all_k, tk.reshape(-1))
    mi, md = shard_ref.merge_keys_host(all_k.numpy().reshape((world,) + tuple(tk.shape)), GS["k"])
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), ids=mi, dists=md)
    dist.barrier()
    dist.destroy_process_group()


def test_graph_two_rank_exchange_over_gloo():
    import torch.multiprocessing as mp
    x, q = _graph_data()
    ei, ed = shard_ref.oracle_sharded_graph(x, q, 2, GB, GS)
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_graph_worker, args=(2, _free_port(), d), nprocs=2, join=True)
        for r in range(2):
            f = np.load(os.path.join(d, f"rank{r}.npz"))
            np.testing.assert_array_equal(f["ids"], ei)
            np.testing.assert_array_equal(f["dists"], ed)
    # the merged result is close to the exact inner-product top-10
    xf, qf = x.astype(np.float64), q.astype(np.float64)
    gt = np.argsort(-(qf @ xf.T), axis=1)[:, :10]
    rec = np.mean([len(set(ei[i]) & set(gt[i])) / 10 for i in range(len(q))])
    assert rec >= 0.8, rec
