"""The build's k-means steps against the reference's own kmeans_gpu.cuh
(compiled from source into oracle/_ref/libref_km.so: cuBLAS SGEMM assignment,
atomic centroid update, GPU encoder), run on the same data.

The reference's assignment forms ||x||^2 + ||c||^2 - 2 x.c with an SGEMM
(kmeans_gpu.cuh:54-78, 197-229), whose summation order is cuBLAS's; this
build sums (x - c)^2 in dimension order.  On integer-valued vectors every
partial sum is an integer below 2^24, both are exact, and the choices are
identical; on general floats they may differ only between near-equal
distances."""
import numpy as np
import pytest

import oracle
from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def fg():
    if oracle._ref_km() is None:
        pytest.skip("oracle/_ref/libref_km.so not built (reference sources absent)")
    import fusiongpu_b200.index as fgi
    yield fgi
    oracle.ref_kmeans_cleanup()


def _ints(n, dim, seed):
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, size=(n, dim)).astype(np.float32)


@pytest.mark.parametrize("n,k,dim", [(20000, 300, 128), (9000, 4096, 128), (5000, 64, 96)])
def test_assign_equals_reference_on_integer_vectors(fg, n, k, dim):
    x = _ints(n, dim, n + k)
    c = x[np.random.default_rng(k).choice(n, k, replace=False)].copy()
    c[k // 2] = c[1]  # a duplicated centroid: both pick the lower index
    got = fg.gpu_assign_to_centroids(torch.from_numpy(x).cuda(), torch.from_numpy(c).cuda())
    np.testing.assert_array_equal(got.cpu().numpy(), oracle.ref_assign(x, c))


def test_assign_agrees_with_reference_on_floats(fg):
    rng = np.random.default_rng(5)
    x = rng.normal(size=(30000, 96)).astype(np.float32)
    c = rng.normal(size=(500, 96)).astype(np.float32)
    got = fg.gpu_assign_to_centroids(torch.from_numpy(x).cuda(), torch.from_numpy(c).cuda()).cpu().numpy()
    ref = oracle.ref_assign(x, c)
    assert (got == ref).mean() > 0.999
    diff = np.flatnonzero(got != ref)
    d = lambda i, j: float(((x[i].astype(np.float64) - c[j]) ** 2).sum())
    for i in diff:  # only near-ties may differ
        assert abs(d(i, got[i]) - d(i, ref[i])) <= 1e-5 * d(i, ref[i])


def test_kmeans_first_step_matches_reference(fg):
    """Same strided MT19937(42) seeding (kmeans_gpu.cuh:259-267), so after one
    Lloyd step the assignment is identical on integer vectors and the
    centroids agree within the reference's float arithmetic (atomic sums
    scaled by a float reciprocal, kmeans_gpu.cuh:81-116, against double sums
    divided here).  A centroid left without points becomes zero in the
    reference (kmeans_gpu.cuh:291-293 zero the centroids before the sums) and
    keeps its previous value here."""
    x = _ints(12000, 64, 3)
    k = 400
    ref1 = oracle.ref_kmeans(x, k, 1)
    got1 = fg.run_kmeans_gpu(torch.from_numpy(x).cuda(), k, 1).cpu().numpy()
    init = fg.run_kmeans_gpu(torch.from_numpy(x).cuda(), k, 0).cpu().numpy()
    a = oracle.assign(x, init)
    empty = np.setdiff1d(np.arange(k), a)
    full = np.setdiff1d(np.arange(k), empty)
    np.testing.assert_allclose(got1[full], ref1[full], rtol=1e-6, atol=1e-4)
    assert (ref1[empty] == 0).all()
    np.testing.assert_array_equal(got1[empty], init[empty])


def test_encoder_equals_reference(fg):
    from fusiongpu_b200 import datasets as ds
    base, _ = ds.generate(ds.scaled(ds.C3, 20000, 10, n_centres=64, seed=5))
    cen = oracle.kmeans(base, 48, 3)
    a = oracle.assign(base, cen)
    cb = oracle.pq_train(base, a, cen, 48, 8000, 4)
    got = fg.encode_residuals_to_pq_gpu(torch.from_numpy(base).cuda(), torch.from_numpy(a).cuda(),
                                        torch.from_numpy(cen).cuda(), torch.from_numpy(cb).cuda())
    np.testing.assert_array_equal(got.cpu().numpy(), oracle.ref_encode(base, a, cen, cb))
