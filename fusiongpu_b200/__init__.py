"""fusiongpu_b200: an IVF-PQ search engine for NVIDIA B200 (sm_100a).

The compute path is ``libfusiongpu_b200.so`` (hand-written CUDA behind the C
ABI in ``include/fusiongpu.h``); this package is the host-side mirror of the
reference's interface over it.  Importing the package does not need a GPU;
calling into the library does, and fails loudly without one.
"""
from . import datasets, formats  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    # the torch-backed API loads lazily so that CPU-only users of the data
    # and format helpers do not pay for importing torch
    if name in ("IVFPQIndex", "SearchParams", "run_gpu_batch_logic", "run_gpu_rerank", "coarse_search",
                "knn_exact", "run_kmeans_gpu", "gpu_assign_to_centroids", "train_residual_pq_codebooks",
                "encode_residuals_to_pq_gpu", "sort_by_list", "recall_at"):
        from . import index
        return getattr(index, name)
    raise AttributeError(name)
