"""Generate golden vectors from the reference's own search kernels.

Runs on a machine with a GPU and the reference built into oracle/_ref
(`make -C oracle ref`): the reference's run_gpu_batch_logic and
run_gpu_rerank (gpu_global.cu:667-874, compiled from source for sm_100a) on a
small seeded index with injected probe lists.  Writes ref_<name>.npz holding
the index, the probes and the reference's outputs; tests/test_golden_cpu.py
checks the CPU oracle against them without a GPU.

    python tests/golden/make_golden.py [out_dir]
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from fusiongpu_b200 import datasets as ds  # noqa: E402

SPEC = dict(n_base=8000, n_query=64, n_centres=32, seed=31)
INDEX = dict(nlist=64, pq_m=32, kmeans_iters=6, pq_sample=4000, pq_iters=6)
PARAMS = {
    "c1": dict(top_m=12, p1_lists=5, limit_k=50, threshold_coeff=1.0, prune_ratio=100.0, rerank_m=100,
               final_k=10, mini_batch=128, epsilon=0.1, beta=2),
    "deep": dict(top_m=16, p1_lists=6, limit_k=40, threshold_coeff=1.1, prune_ratio=100.0, rerank_m=300,
                 final_k=20, mini_batch=64, epsilon=0.1, beta=3),
}


def workload():
    spec = ds.scaled(ds.C1, SPEC["n_base"], SPEC["n_query"], n_centres=SPEC["n_centres"], seed=SPEC["seed"])
    return ds.generate(spec)


def main(out_dir):
    import torch
    import ctypes as C
    base, q = workload()
    index, _ = oracle.build_index(base, INDEX["nlist"], INDEX["pq_m"], kmeans_iters=INDEX["kmeans_iters"],
                                  pq_sample=INDEX["pq_sample"], pq_iters=INDEX["pq_iters"])
    L = oracle.ref_lib("gg", base.shape[1], INDEX["pq_m"])
    assert L is not None, "oracle/_ref not built"
    dev = "cuda"
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in index.items()}
    tq = torch.from_numpy(q).to(dev)
    tb = torch.from_numpy(base).to(dev)
    P = lambda x: C.c_void_p(x.data_ptr())  # noqa: E731
    for name, p in PARAMS.items():
        pid, pdist = oracle.coarse(index["centroids"], q, p["top_m"])
        nq, rm, k = q.shape[0], p["rerank_m"], p["final_k"]
        # the reference writes each query's candidates into a region sized by the
        # summed lengths of its probed lists; run it only where the oracle shows
        # its writes stay inside that region
        _, _, _, st = oracle.batch_logic(index, q, pid, pdist, **p, ref_compat=True)
        lens = np.diff(index["offsets"])
        budget = np.where(pdist > pdist[:, :1] * np.float32(p["prune_ratio"]), 0, lens[pid.astype(np.int64)]).sum(1)
        assert (st["count"] <= budget).all()
        tpid = torch.from_numpy(pid.view(np.int32).copy()).to(dev)
        tpd = torch.from_numpy(pdist).to(dev)
        top_i = torch.zeros((nq, rm), dtype=torch.int32, device=dev)
        top_d = torch.zeros((nq, rm), dtype=torch.float32, device=dev)
        top_c = torch.zeros(nq, dtype=torch.int32, device=dev)
        cnt = torch.zeros(nq, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        rc = L.ref_run_batch_logic(P(t["codebook"]), P(t["offsets"]), P(t["codes"]), P(t["ids"]),
                                   P(t["centroids"]), index["centroids"].shape[0], P(tq), P(tpid), P(tpd), nq,
                                   p["top_m"], rm, k, C.c_float(p["prune_ratio"]), p["p1_lists"], p["limit_k"],
                                   C.c_float(p["threshold_coeff"]), P(top_i), P(top_d), P(top_c), P(cnt))
        assert rc == 0, rc
        fi = torch.zeros((nq, k), dtype=torch.int32, device=dev)
        fd = torch.zeros((nq, k), dtype=torch.float32, device=dev)
        rc = L.ref_run_rerank(P(tq), P(top_i), P(top_c), P(tb), P(fi), P(fd), nq, rm, k, base.shape[0],
                              p["mini_batch"], C.c_float(p["epsilon"]), p["beta"])
        assert rc == 0, rc
        np.savez_compressed(
            os.path.join(out_dir, f"ref_{name}.npz"),
            base_sum=np.float64(base.astype(np.float64).sum()), queries=q, probe_ids=pid, probe_dists=pdist,
            **{f"index_{k_}": v for k_, v in index.items()},
            params=np.array([repr(p)]),
            ref_top_ids=top_i.cpu().numpy(), ref_top_dists=top_d.cpu().numpy(), ref_top_counts=top_c.cpu().numpy(),
            ref_counts=cnt.cpu().numpy(), ref_final_ids=fi.cpu().numpy(), ref_final_dists=fd.cpu().numpy())
        print("wrote", name)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
