"""The allocation-free coarse search (fg_coarse_search_noalloc).

It exists for callers that cannot pass device memory at call time -- plugins
whose host runtime owns every device pool, serving loops that must not reach
cudaMalloc or cudaFree.  It must return exactly what the
workspace-based exact path (fg_coarse_search_simt) returns, on consecutive
calls that reuse its built-in scratch array.  This file sorts last so that a
run stopping at the first failure has run every other test already.
"""
import ctypes as C

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]
torch = pytest.importorskip("torch")


def _p(t):
    return C.c_void_p(t.data_ptr())


def _simt(L, cen, q, top_m):
    nlist, dim = cen.shape
    nq = q.shape[0]
    ids = torch.empty((nq, top_m), dtype=torch.int32, device="cuda")
    d = torch.empty((nq, top_m), dtype=torch.float32, device="cuda")
    need = C.c_size_t(0)
    assert L.fg_coarse_workspace_size(nlist, dim, nq, top_m, C.byref(need)) == 0
    ws = torch.empty(max(need.value, 256), dtype=torch.uint8, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.fg_coarse_search_simt(_p(cen), nlist, dim, _p(q), nq, top_m, _p(ids), _p(d), _p(ws), ws.numel(), stream)
    assert rc == 0, L.fg_last_error()
    return ids, d


def _noalloc(L, cen, q, top_m):
    nlist, dim = cen.shape
    nq = q.shape[0]
    ids = torch.full((nq, top_m), -7, dtype=torch.int32, device="cuda")
    d = torch.full((nq, top_m), -7.0, dtype=torch.float32, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.fg_coarse_search_noalloc(_p(cen), nlist, dim, _p(q), nq, top_m, _p(ids), _p(d), stream)
    assert rc == 0, L.fg_last_error()
    return ids, d


@pytest.mark.parametrize("nlist,dim,nq,top_m", [(4096, 128, 3000, 32), (10000, 32, 700, 64)])
def test_noalloc_equals_workspace_path_on_consecutive_calls(nlist, dim, nq, top_m):
    from fusiongpu_b200 import _lib
    L = _lib.lib()
    g = torch.Generator(device="cuda").manual_seed(nlist)
    cen = torch.randn((nlist, dim), generator=g, device="cuda")
    q = torch.randn((nq, dim), generator=g, device="cuda")
    ei, ed = _simt(L, cen, q, top_m)
    for _ in range(2):  # the second call reuses the scratch the first one left behind
        ids, d = _noalloc(L, cen, q, top_m)
        torch.cuda.synchronize()
        # exact equality: both paths compute the same fp32 expressions in the same order
        np.testing.assert_array_equal(ids.cpu().numpy(), ei.cpu().numpy())
        np.testing.assert_array_equal(d.cpu().numpy(), ed.cpu().numpy())


def test_noalloc_rejects_rows_beyond_its_scratch():
    from fusiongpu_b200 import _lib
    L = _lib.lib()
    nlist, dim = 5_000_000, 1  # one distance row alone is 20 MB > 16 MiB
    cen = torch.zeros((nlist, dim), device="cuda")
    q = torch.zeros((2, dim), device="cuda")
    ids = torch.empty((2, 4), dtype=torch.int32, device="cuda")
    d = torch.empty((2, 4), dtype=torch.float32, device="cuda")
    rc = L.fg_coarse_search_noalloc(_p(cen), nlist, dim, _p(q), 2, 4, _p(ids), _p(d),
                                    C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 1
    assert b"scratch" in L.fg_last_error()
