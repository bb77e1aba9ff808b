"""Golden vectors from the reference's own tuner (tune_parameters.cu).

Runs on a machine with a GPU and oracle/_ref built (`make -C oracle ref`):
the reference's tune_search_parameters (compiled from source, its sampler
seeded through the wrapper) on a small seeded index.  Writes ref_tune.npz
with the base, the index, the sample rows the reference drew and its
recommendations and per-neighbour statistics; tests/test_tune_cpu.py checks
the CPU oracle against them without a GPU.

    python tests/golden/make_golden_tune.py [out_dir]
"""
import ctypes as C
import dataclasses
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from fusiongpu_b200 import datasets as ds  # noqa: E402

DIM, PQ_M = 64, 16
INDEX = dict(nlist=48, pq_m=PQ_M, kmeans_iters=6, pq_sample=4000, pq_iters=5)
TUNE = dict(n_samples=200, k=10, seed=1234)


def workload():
    spec = dataclasses.replace(ds.scaled(ds.C1, 6000, 8, n_centres=24, seed=41), dim=DIM)
    base, _ = ds.generate(spec)
    return base


def ref_tune_lib():
    return oracle.ref_lib("tune", DIM, PQ_M)


def ref_sample(L, seed, n_base, n):
    rows = np.empty(n, np.int32)
    L.ref_tune_sample(C.c_uint(seed), n_base, n, C.c_void_p(rows.ctypes.data))
    return rows


def run_ref(L, base, index, n_samples, k, seed):
    P = lambda a: C.c_void_p(np.ascontiguousarray(a).ctypes.data)  # noqa: E731
    out_i = np.zeros(6, np.int32)
    coeff = C.c_float(0)
    cr = np.zeros(n_samples * k, np.int32)
    pr = np.zeros(n_samples * k, np.int32)
    er = np.zeros(n_samples * k, np.int32)
    ra = np.zeros(n_samples, np.float32)
    keep = [np.ascontiguousarray(x) for x in (base, index["centroids"], index["offsets"], index["ids"],
                                              index["codes"], index["codebook"])]
    rc = L.ref_tune(P(keep[0]), base.shape[0], P(keep[1]), index["centroids"].shape[0], P(keep[2]), P(keep[3]),
                    P(keep[4]), P(keep[5]), n_samples, k, C.c_uint(seed), P(out_i), C.byref(coeff), P(cr), P(pr),
                    P(er), P(ra))
    assert rc == 0, rc
    return dict(top_m=int(out_i[0]), p1_lists=int(out_i[1]), limit_k=int(out_i[2]), threshold_coeff=coeff.value,
                cluster_ranks=cr[:out_i[3]], pq_ranks=pr[:out_i[4]], exact_ranks=er[:out_i[4]], ratios=ra[:out_i[5]])


def main(out_dir):
    base = workload()
    index, _ = oracle.build_index(base, INDEX["nlist"], PQ_M, kmeans_iters=INDEX["kmeans_iters"],
                                  pq_sample=INDEX["pq_sample"], pq_iters=INDEX["pq_iters"])
    L = ref_tune_lib()
    assert L is not None, "oracle/_ref not built"
    rows = ref_sample(L, TUNE["seed"], base.shape[0], TUNE["n_samples"])
    r = run_ref(L, base, index, TUNE["n_samples"], TUNE["k"], TUNE["seed"])
    np.savez_compressed(
        os.path.join(out_dir, "ref_tune.npz"), base=base, rows=rows, seed=TUNE["seed"], k=TUNE["k"],
        **{f"index_{k_}": v for k_, v in index.items()},
        ref_top_m=r["top_m"], ref_p1_lists=r["p1_lists"], ref_limit_k=r["limit_k"],
        ref_threshold_coeff=np.float32(r["threshold_coeff"]), ref_cluster_ranks=r["cluster_ranks"],
        ref_pq_ranks=r["pq_ranks"], ref_exact_ranks=r["exact_ranks"], ref_ratios=r["ratios"])
    print("wrote ref_tune.npz", {k_: r[k_] for k_ in ("top_m", "p1_lists", "limit_k", "threshold_coeff")})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
