/*
 * ref_build_global_wrap.cu -- TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference's index-build program (build_global.cu, included by
 * path through REF_SRC, with its kmeans_gpu.cuh, pq_utils.h and utils.h) into
 * an executable with the compile-time constants of one workload (REF_DIM,
 * REF_PQ_M, REF_K_CLUSTERS; see ref_defs.h).  It runs the reference's own
 * build unchanged: GPU k-means (cuBLAS), assignment, the FIFO rebalancing
 * loop, CPU residual-PQ training, GPU encoding, and writes ../res/ivf_data.bin
 * and ../res/global_pq_codebook.bin relative to its working directory.
 *
 * One step cannot run here: the cuVS CAGRA graph over the final centroids
 * (build_global.cu:175-183, cagra_adapter.cuh:10-26) needs RAFT/cuVS, which
 * this image does not have.  Its header is skipped by defining its include
 * guard, and the stub below takes the call and writes no graph file; the
 * search side injects exact probe lists in its place.
 */
#include "ref_defs.h"

#define CAGRA_ADAPTER_CUH
inline void build_cagra_index(const float*, int, int, const char*) {}

#include REF_SRC
