"""GPU side of the list-sharded search: the merge kernel, shards simulated on
one GPU, and (with 2+ GPUs) the real NCCL all-gather, each against the
oracle's statement of the sharded semantics."""
import ctypes as C
import os
import socket
import tempfile

import numpy as np
import pytest

import oracle
from fusiongpu_b200 import datasets as ds
from tests import shard_ref
from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]
torch = pytest.importorskip("torch")

P = dict(top_m=10, p1_lists=4, limit_k=40, threshold_coeff=1.0, prune_ratio=100.0, rerank_m=120, final_k=10,
         mini_batch=64, epsilon=0.1, beta=2, ref_compat=False)


def _data():
    base, q = ds.generate(ds.scaled(ds.C1, 12000, 96, n_centres=32, seed=43))
    index, _ = oracle.build_index(base, 64, 32, kmeans_iters=4, pq_sample=4000, pq_iters=4)
    return index, base, q


def _merge_gpu(d, i, k):
    from fusiongpu_b200 import _lib
    from fusiongpu_b200.index import _p, _stream
    ns, nq, kk = d.shape
    td = torch.from_numpy(np.ascontiguousarray(d)).cuda()
    ti = torch.from_numpy(np.ascontiguousarray(i)).cuda()
    oi = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    od = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    _lib.call("fg_merge_topk", _p(td), _p(ti), ns, nq, k, _p(oi), _p(od), _stream())
    return oi.cpu().numpy(), od.cpu().numpy()


def _merge_keys_gpu(d, i, k):
    """Pack each shard's [nq][k] on the GPU, then merge the stacked keys."""
    from fusiongpu_b200 import _lib
    from fusiongpu_b200.index import _p, _stream
    ns, nq, kk = d.shape
    keys = torch.empty((ns, nq, kk), dtype=torch.int64, device="cuda")
    for s in range(ns):
        td = torch.from_numpy(np.ascontiguousarray(d[s])).cuda()
        ti = torch.from_numpy(np.ascontiguousarray(i[s])).cuda()
        _lib.call("fg_pack_topk", _p(ti), _p(td), nq, kk, None, 0, _p(keys[s]), _stream())
    oi = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    od = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    _lib.call("fg_merge_topk_keys", _p(keys), ns, nq, k, _p(oi), _p(od), _stream())
    return keys.cpu().numpy(), oi.cpu().numpy(), od.cpu().numpy()


@pytest.mark.parametrize("ns,nq,k", [(6, 150, 20), (1, 33, 7), (2, 70, 100), (8, 40, 100), (3, 9, 1)])
def test_packed_key_merge_matches_host_statements(ns, nq, k):
    rng = np.random.default_rng(4 + ns + k)
    d = np.sort(rng.integers(-10, 10, size=(ns, nq, k)).astype(np.float32) * 0.25, axis=2)  # ties, negatives
    i = rng.permutation(ns * nq * k).reshape(ns, nq, k).astype(np.int32)
    d[:, :, -3:] = np.finfo(np.float32).max
    i[:, :, -3:] = -1
    keys, oi, od = _merge_keys_gpu(d, i, k)
    want = np.stack([np.sort(shard_ref.pack_keys_host(i[s], d[s]).view(np.uint64), axis=1) for s in range(ns)])
    np.testing.assert_array_equal(keys.view(np.uint64), want)
    ei, ed = shard_ref.merge_topk_host(d, i, k)
    np.testing.assert_array_equal(oi, ei)
    np.testing.assert_array_equal(od, ed)


def test_pack_maps_local_ids():
    from fusiongpu_b200 import _lib
    from fusiongpu_b200.index import _p, _stream
    ids = torch.tensor([0, 3, -1, 7, 2], dtype=torch.int32, device="cuda")
    d = torch.tensor([1.0, 2.0, 3.0, 4.0, 0.5], device="cuda")
    m = torch.tensor([10, 11, 12, 13], dtype=torch.int32, device="cuda")
    keys = torch.empty(5, dtype=torch.int64, device="cuda")
    _lib.call("fg_pack_topk", _p(ids), _p(d), 1, 5, _p(m), 4, _p(keys), _stream())
    want = shard_ref.pack_keys_host(np.array([10, 13, -1, -1, 12], np.int32), d.cpu().numpy())
    np.testing.assert_array_equal(keys.cpu().numpy().view(np.uint64), np.sort(want.view(np.uint64)))


def test_merge_kernel_matches_host_statement():
    rng = np.random.default_rng(3)
    ns, nq, k = 5, 200, 16
    d = np.sort(rng.integers(0, 20, size=(ns, nq, k)).astype(np.float32), axis=2)  # many ties
    i = rng.permutation(ns * nq * k).reshape(ns, nq, k).astype(np.int32)
    d[:, :, -3:] = np.finfo(np.float32).max
    i[:, :, -3:] = -1
    oi, od = _merge_gpu(d, i, k)
    ei, ed = shard_ref.merge_topk_host(d, i, k)
    np.testing.assert_array_equal(od, ed)
    np.testing.assert_array_equal(oi, ei)


@pytest.mark.parametrize("world", [2, 3])
def test_shards_on_one_gpu_match_oracle(world):
    from fusiongpu_b200.index import SearchParams
    from fusiongpu_b200.sharded import ShardedIndex
    index, base, q = _data()
    p = SearchParams(**P)
    qd = torch.from_numpy(q).cuda()
    ds_, is_ = [], []
    for r in range(world):
        sh = ShardedIndex(index, base, r, world)
        gi, d = sh.local_search(qd, p)
        ds_.append(d.cpu().numpy())
        is_.append(gi.cpu().numpy())
    oi, od = _merge_gpu(np.stack(ds_), np.stack(is_), P["final_k"])
    ei, ed = shard_ref.oracle_sharded_search(index, base, q, world, **P)
    np.testing.assert_array_equal(od, ed)
    np.testing.assert_array_equal(oi, ei)


def _nccl_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    from fusiongpu_b200.index import SearchParams
    from fusiongpu_b200.sharded import ShardedIndex
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    index, base, q = _data()
    sh = ShardedIndex(index, base, rank, world, device=f"cuda:{rank}")
    ids, d = sh.search(torch.from_numpy(q).to(f"cuda:{rank}"), SearchParams(**P))
    torch.cuda.synchronize()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), ids=ids.cpu().numpy(), dists=d.cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not cuda_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpus_nccl_all_gather_matches_oracle():
    import torch.multiprocessing as mp
    index, base, q = _data()
    ei, ed = shard_ref.oracle_sharded_search(index, base, q, 2, **P)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_nccl_worker, args=(2, port, d), nprocs=2, join=True)
        for r in range(2):
            f = np.load(os.path.join(d, f"rank{r}.npz"))
            np.testing.assert_array_equal(f["dists"], ed)
            np.testing.assert_array_equal(f["ids"], ei)


# ---- graph sharded by rows --------------------------------------------------------

GB = dict(graph_degree=16, intermediate_degree=32, nlist=24, probe_lists=3, kmeans_iters=3, seed=42, metric="ip")
GS = dict(itopk=48, search_width=2, k=10, seed=5, metric="ip", entry_probes=4)


def _graph_data():
    rng = np.random.default_rng(22)
    x = rng.normal(size=(6000, 64)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    q = rng.normal(size=(40, 64)).astype(np.float32)
    return x.astype(np.float16), q.astype(np.float16)


@pytest.mark.parametrize("world", [1, 3])
def test_graph_shards_on_one_gpu_match_oracle(world):
    from fusiongpu_b200.graph import GraphBuildParams, GraphSearchParams
    from fusiongpu_b200.sharded import ShardedGraphIndex
    x, q = _graph_data()
    qd = torch.from_numpy(q).cuda()
    ds_, is_ = [], []
    for r in range(world):
        sh = ShardedGraphIndex(torch.from_numpy(x).cuda(), r, world, GraphBuildParams(**GB))
        gi, d = sh.local_search(qd, GraphSearchParams(**GS))
        ds_.append(d.cpu().numpy())
        is_.append(gi.cpu().numpy())
    oi, od = _merge_gpu(np.stack(ds_), np.stack(is_), GS["k"])
    ei, ed = shard_ref.oracle_sharded_graph(x, q, world, GB, GS)
    np.testing.assert_array_equal(od, ed)
    np.testing.assert_array_equal(oi, ei)


def _graph_nccl_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    from fusiongpu_b200.graph import GraphBuildParams, GraphSearchParams
    from fusiongpu_b200.sharded import ShardedGraphIndex
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    x, q = _graph_data()
    dev = f"cuda:{rank}"
    sh = ShardedGraphIndex(torch.from_numpy(x).to(dev), rank, world, GraphBuildParams(**GB), device=dev)
    ids, d = sh.search(torch.from_numpy(q).to(dev), GraphSearchParams(**GS))
    torch.cuda.synchronize()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), ids=ids.cpu().numpy(), dists=d.cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not cuda_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_graph_two_gpus_nccl_matches_oracle():
    import torch.multiprocessing as mp
    x, q = _graph_data()
    ei, ed = shard_ref.oracle_sharded_graph(x, q, 2, GB, GS)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_graph_nccl_worker, args=(2, port, d), nprocs=2, join=True)
        for r in range(2):
            f = np.load(os.path.join(d, f"rank{r}.npz"))
            np.testing.assert_array_equal(f["dists"], ed)
            np.testing.assert_array_equal(f["ids"], ei)


def test_shard_of_long_lists_keeps_the_split_path():
    """A shard owns a quarter of the lists but keeps every list slot, so the
    mean over all slots understates its lists; the scan dispatch still sees
    long lists (typical length = max(mean, longest / 2)) and runs the split
    path, with the oracle's per-shard results."""
    import ctypes as C
    from fusiongpu_b200 import _lib
    from fusiongpu_b200.index import SearchParams
    from fusiongpu_b200.sharded import ShardedIndex
    base, q = ds.generate(ds.scaled(ds.C1, 24000, 64, n_centres=16, seed=44))
    index, _ = oracle.build_index(base, 16, 32, kmeans_iters=4, pq_sample=6000, pq_iters=4, rebalance_lists=False)
    lens = np.diff(index["offsets"])
    assert lens.mean() > 400
    p = SearchParams(**dict(P, top_m=8, p1_lists=2))
    shards = [ShardedIndex(index, base, r, 4) for r in range(4)]
    for sh in shards:
        local = sh.local
        assert local.total / local.nlist <= 400 < local.max_list_len / 2
        need = _lib.size_query("fg_batch_logic_workspace_size", C.byref(local.view), C.byref(p.c()), q.shape[0])
        assert need > 0
    qd = torch.from_numpy(q).cuda()
    ds_, is_ = [], []
    for sh in shards:
        gi, d = sh.local_search(qd, p)
        ds_.append(d.cpu().numpy())
        is_.append(gi.cpu().numpy())
    oi, od = _merge_gpu(np.stack(ds_), np.stack(is_), P["final_k"])
    ei, ed = shard_ref.oracle_sharded_search(index, base, q, 4, **dict(P, top_m=8, p1_lists=2))
    np.testing.assert_array_equal(od, ed)
    np.testing.assert_array_equal(oi, ei)
