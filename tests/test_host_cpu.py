"""CPU tests of the host side: formats, generators, and the C-ABI library
(load + exported symbols only; no compute call without a GPU)."""
import ctypes
import os
import re

import numpy as np

from fusiongpu_b200 import datasets as ds
from fusiongpu_b200 import formats

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_generator_is_deterministic_and_integer_valued():
    spec = ds.scaled(ds.C1, 3000, 20, n_centres=8)
    b1, q1 = ds.generate(spec)
    b2, q2 = ds.generate(spec)
    np.testing.assert_array_equal(b1, b2)
    np.testing.assert_array_equal(q1, q2)
    assert b1.dtype == np.float32 and b1.shape == (3000, 128)
    assert (b1 == np.rint(b1)).all() and b1.min() >= 0 and b1.max() <= 255


def test_generator_unit_and_uint8():
    b, _ = ds.generate(ds.scaled(ds.C3, 500, 5, n_centres=4))
    np.testing.assert_allclose(np.linalg.norm(b, axis=1), 1.0, rtol=1e-5)
    b, _ = ds.generate(ds.scaled(ds.C5, 500, 5, n_centres=4))
    assert b.dtype == np.uint8


def test_fvecs_ivecs_roundtrip(tmp_path):
    x = np.random.default_rng(0).normal(size=(7, 5)).astype(np.float32)
    formats.write_vecs(str(tmp_path / "a.fvecs"), x)
    np.testing.assert_array_equal(formats.read_vecs(str(tmp_path / "a.fvecs")), x)
    g = np.arange(12, dtype=np.int32).reshape(3, 4)
    formats.write_vecs(str(tmp_path / "g.ivecs"), g)
    np.testing.assert_array_equal(formats.read_vecs(str(tmp_path / "g.ivecs"), np.int32), g)
    raw = np.fromfile(str(tmp_path / "g.ivecs"), np.int32)
    assert raw[0] == 4 and raw[5] == 4  # per-row dimension header (utils.h:56-58)


def test_ivf_file_layout(tmp_path):
    rng = np.random.default_rng(0)
    nlist, dim, pq_m = 5, 8, 4
    lens = np.array([3, 0, 2, 4, 1])
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    idx = dict(codebook=rng.normal(size=(pq_m, 256, dim // pq_m)).astype(np.float32), offsets=off,
               ids=rng.permutation(10).astype(np.int32), codes=rng.integers(0, 256, (10, pq_m)).astype(np.uint8),
               centroids=rng.normal(size=(nlist, dim)).astype(np.float32))
    formats.save_index(str(tmp_path), idx)
    raw = np.fromfile(str(tmp_path / "ivf_data.bin"), np.uint8)
    hdr = raw[:8].view(np.int32)
    assert list(hdr) == [10, nlist]
    assert raw.size == 8 + 4 * (nlist + 1) + 4 * 10 + 10 * pq_m + 4 * nlist * dim
    back = formats.load_index(str(tmp_path), pq_m, dim)
    for k in idx:
        np.testing.assert_array_equal(back[k], idx[k])


def _declared_symbols():
    h = open(os.path.join(ROOT, "include", "fusiongpu.h")).read()
    h = re.sub(r"/\*.*?\*/", "", h, flags=re.S)
    return sorted(set(re.findall(r"\b(fg_[a-z0-9_]+)\s*\(", h)))


def test_library_exports_every_declared_symbol():
    from fusiongpu_b200 import _lib
    L = ctypes.CDLL(_lib.LIB_PATH)
    declared = _declared_symbols()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(L, name), name
    # the binding covers the whole header
    assert sorted(_lib.exported_symbols()) == declared
    L.fg_version.restype = ctypes.c_char_p
    assert b"sm_100a" in L.fg_version()


def test_library_defaults_match_reference():
    from fusiongpu_b200 import _lib
    p = _lib.SearchParams()
    _lib.lib().fg_search_params_default(ctypes.byref(p))
    assert (p.top_m, p.p1_lists, p.limit_k, p.rerank_m, p.final_k, p.mini_batch, p.beta) == (
        20, 12, 50, 10000, 10, 128, 2)
    assert abs(p.epsilon - 0.1) < 1e-7 and p.prune_ratio == 100.0 and p.threshold_coeff == 1.0


def test_scan_dispatch_by_list_length_and_probe_count(monkeypatch):
    """fg_batch_logic_workspace_size states which candidate-generation path a
    search takes (host logic only, no GPU): short lists with fewer than 8
    probes run the team kernel (no workspace); short lists with 8 or more
    probes, all in phase 1, the group kernel (top_m * limit_k candidate keys
    per query); long lists, or a shard whose longest list is long, the split
    path (max(4096, 2 * rerank_m) keys per query)."""
    from fusiongpu_b200 import _lib
    monkeypatch.delenv("FG_SCAN_KERNEL", raising=False)

    def ws(total, max_len, top_m, p1_lists, nq=1000, rerank_m=1000, limit_k=50):
        v = _lib.IvfpqView(0, 0, 0, 0, 0, 4104, 128, 64, total, max_len)
        p = _lib.SearchParams()
        _lib.lib().fg_search_params_default(ctypes.byref(p))
        p.top_m, p.p1_lists, p.rerank_m, p.limit_k = top_m, p1_lists, rerank_m, limit_k
        return _lib.size_query("fg_batch_logic_workspace_size", ctypes.byref(v), ctypes.byref(p), nq)

    c2 = dict(total=1_000_000, max_len=488)  # C2: 4,104 lists of ~244
    assert ws(**c2, top_m=2, p1_lists=12) == 0
    assert ws(**c2, top_m=4, p1_lists=12) == 0
    assert ws(**c2, top_m=16, p1_lists=12) == 0  # phase 2: the team kernel
    g8 = ws(**c2, top_m=8, p1_lists=12)
    assert 1000 * 8 * 50 * 8 <= g8 < 1000 * 4096 * 8  # the group path's keys, not the split path's
    assert ws(**c2, top_m=12, p1_lists=12) > g8
    s = ws(total=4_000_000, max_len=1400, top_m=64, p1_lists=12)  # lists of ~975
    assert s >= 1000 * 4096 * 8
    shard = ws(total=250_000, max_len=1400, top_m=64, p1_lists=12)  # a quarter of the lists owned
    assert shard >= 1000 * 4096 * 8
    monkeypatch.setenv("FG_SCAN_KERNEL", "team")
    assert ws(**c2, top_m=8, p1_lists=12) == 0
