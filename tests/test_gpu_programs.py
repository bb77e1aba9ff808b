"""GPU tests of the C++ host layer: the three programs that mirror the
reference's executables (fg_build_global, fg_search_pipeline,
fg_tune_parameters), a caller of the reference's C++ signatures compiled
against include/fusiongpu_compat.hpp, and the tuner through the C ABI --
each against the CPU oracle (bit-exact) and, where oracle/_ref is built, the
tuner against the reference's own."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

import oracle
from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "fusiongpu_b200", "bin")
DIM, PQ_M, NLIST = 64, 16, 32
BUILD = dict(kmeans_iters=2, pq_sample=4000, pq_iters=3)
SEARCH = dict(top_m=8, rerank_m=300, final_k=10, p1_lists=12, limit_k=50, threshold_coeff=1.0, prune_ratio=100.0,
              mini_batch=128, epsilon=0.1, beta=2)


def _run(args, cwd, timeout=600):
    r = subprocess.run(args, cwd=cwd, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, f"{args[0]} failed ({r.returncode}):\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    return r.stdout


def _data():
    # blobs of unequal spread so that the build rebalances lists; queries are
    # fresh draws from the same blobs
    rng = np.random.default_rng(7)
    centres = rng.normal(0, 4, size=(3, DIM))
    spread = (0.5, 1.0, 3.0)
    x = np.concatenate([rng.normal(centres[i], spread[i], size=(n, DIM))
                        for i, n in enumerate((5000, 2000, 1000))]).astype(np.float32)
    base = np.ascontiguousarray(x[rng.permutation(x.shape[0])])
    qr = np.random.default_rng(8)
    pick = qr.integers(0, 3, size=300)
    q = np.stack([qr.normal(centres[i], spread[i]) for i in pick]).astype(np.float32)
    return base, np.ascontiguousarray(q)


@pytest.fixture(scope="module")
def work(tmp_path_factory):
    from fusiongpu_b200 import build, formats
    build.programs()
    d = tmp_path_factory.mktemp("programs")
    base, q = _data()
    formats.write_vecs(str(d / "base.fvecs"), base)
    formats.write_vecs(str(d / "q.fvecs"), q)
    gt, _ = oracle.knn_exact(base, q, 10)
    formats.write_vecs(str(d / "gt.ivecs"), gt)
    os.makedirs(d / "res")
    out = _run([os.path.join(BIN, "fg_build_global"), "base.fvecs", "--nlist", str(NLIST), "--pq_m", str(PQ_M),
                "--out", "res", "--kmeans_iters", str(BUILD["kmeans_iters"]), "--pq_sample",
                str(BUILD["pq_sample"]), "--pq_iters", str(BUILD["pq_iters"])], cwd=d)
    index, _ = oracle.build_index(base, NLIST, PQ_M, **BUILD)
    return dict(dir=d, base=base, q=q, gt=gt, index=index, build_log=out)


def test_build_global_program_bit_exact(work):
    from fusiongpu_b200 import formats
    got = formats.load_index(str(work["dir"] / "res"), PQ_M, DIM)
    exp = work["index"]
    assert exp["centroids"].shape[0] > NLIST  # rebalancing split lists
    for k in ("centroids", "codebook", "offsets", "ids", "codes"):
        np.testing.assert_array_equal(got[k], exp[k])
    rows = open(work["dir"] / "cluster_distribution.csv").read().split()[1:]
    counts = np.array([int(r.split(",")[1]) for r in rows])
    np.testing.assert_array_equal(counts, np.diff(exp["offsets"]))


@pytest.mark.parametrize("mode", ["reference", "intended", "fused", "graph"])
def test_search_pipeline_program_bit_exact(work, mode):
    d = work["dir"]
    args = [os.path.join(BIN, "fg_search_pipeline"), "base.fvecs", "q.fvecs", "gt.ivecs", "--res", "res", "--pq_m",
            str(PQ_M), "-b", "64", "-s", "2", "-m", str(SEARCH["top_m"]), "-r", str(SEARCH["rerank_m"]), "-k",
            str(SEARCH["final_k"]), "--out", f"out_{mode}.ivecs"]
    if mode not in ("reference", "graph"):
        args.append("--intended")
    if mode == "fused":
        args.append("--fused")
    if mode == "graph":
        args += ["--graph", "-b", "50"]  # 300 queries: six full batches, all replayed
    out = _run(args, cwd=d)
    from fusiongpu_b200 import formats
    ids = formats.read_vecs(str(d / f"out_{mode}.ivecs"), np.int32)
    exp, _ = oracle.search(work["index"], work["base"], work["q"], ref_compat=(mode in ("reference", "graph")),
                           **SEARCH)
    np.testing.assert_array_equal(ids, exp)
    m = re.search(r"RESULT qps=(\S+) recall1=(\S+) recall10=(\S+)", out)
    assert m, out
    hits = sum(len(set(exp[i, :10]) & set(work["gt"][i, :10])) for i in range(exp.shape[0]))
    assert abs(float(m.group(3)) - hits / (10 * exp.shape[0])) < 1e-5
    assert float(m.group(1)) > 0


def test_tune_api_bit_exact(work):
    import fusiongpu_b200.index as fgi
    from fusiongpu_b200 import tune
    idx = fgi.IVFPQIndex.from_arrays(work["index"], work["base"])
    rows = tune.sample_rows(work["base"].shape[0], 200, 42)
    q = np.ascontiguousarray(work["base"][rows])
    gt, _ = oracle.knn_exact(work["base"], q, 10)
    got = tune.tune_parameters(idx, q, gt)
    exp, cr, pr, er, ra = oracle.tune(work["index"], work["base"], q, gt)
    for k in ("top_m", "p1_lists", "limit_k", "threshold_coeff", "coverage_at_elbow", "n_ranked", "n_in_p1",
              "n_ratios"):
        assert got[k] == exp[k], k
    np.testing.assert_array_equal(got["cluster_ranks"], cr)
    np.testing.assert_array_equal(got["pq_ranks"], pr)
    np.testing.assert_array_equal(got["exact_ranks"], er)
    np.testing.assert_array_equal(got["ratios"], ra)


def test_tune_parameters_program(work):
    from fusiongpu_b200 import tune
    d = work["dir"]
    out = _run([os.path.join(BIN, "fg_tune_parameters"), "base.fvecs", "-n", "200", "-k", "10", "--res", "res",
                "--pq_m", str(PQ_M), "-o", "cfg.txt", "--seed", "42", "--sweep", "--target", "0.5"], cwd=d)
    rows = tune.sample_rows(work["base"].shape[0], 200, 42)
    q = np.ascontiguousarray(work["base"][rows])
    gt, _ = oracle.knn_exact(work["base"], q, 10)
    exp = oracle.tune(work["index"], work["base"], q, gt)[0]
    m = re.search(r"TUNE top_m=(\d+) p1_lists=(\d+) limit_k=(\d+) threshold_coeff=(\S+)", out)
    assert m, out
    assert (int(m.group(1)), int(m.group(2)), int(m.group(3))) == (exp["top_m"], exp["p1_lists"], exp["limit_k"])
    assert abs(float(m.group(4)) - exp["threshold_coeff"]) <= 1e-5 * exp["threshold_coeff"]
    cfg = tune.load_config(str(d / "cfg.txt"))
    assert cfg["top_m"] == exp["top_m"] and cfg["limit_k"] == exp["limit_k"]
    assert "SWEEP best" in out or "SWEEP no grid point" in out


def test_tune_matches_reference_tuner(work):
    L = oracle.ref_lib("tune", DIM, PQ_M)
    if L is None:
        pytest.skip("oracle/_ref not built")
    import sys
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_golden_tune as mg
    import fusiongpu_b200.index as fgi
    from fusiongpu_b200 import tune
    base, index = work["base"], work["index"]
    seed, n, k = 99, 150, 10
    rows = mg.ref_sample(L, seed, base.shape[0], n)
    ref = mg.run_ref(L, base, index, n, k, seed)
    q = np.ascontiguousarray(base[rows])
    idx = fgi.IVFPQIndex.from_arrays(index, base)
    gt, _ = fgi.knn_exact(idx.base, torch.from_numpy(q).cuda(), k)
    got = tune.tune_parameters(idx, q, gt)
    for key in ("top_m", "p1_lists", "limit_k"):
        assert got[key] == ref[key], key
    assert np.float32(got["threshold_coeff"]) == np.float32(ref["threshold_coeff"])
    cr, pr, er, ra = got["cluster_ranks"], got["pq_ranks"], got["exact_ranks"], got["ratios"]
    np.testing.assert_array_equal(cr[cr > 0], ref["cluster_ranks"])
    np.testing.assert_array_equal(pr[pr > 0], ref["pq_ranks"])
    np.testing.assert_array_equal(er[er > 0], ref["exact_ranks"])
    np.testing.assert_array_equal(ra[~np.isnan(ra)], ref["ratios"])


def _compile_compat(tmp_path):
    exe = str(tmp_path / "compat_search")
    subprocess.run(["/usr/bin/g++", "-O2", "-std=c++17", f"-DDIM={DIM}", f"-DPQ_M={PQ_M}",
                    "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "fusiongpu_b200", "host"),
                    "-I", "/usr/local/cuda/include", os.path.join(ROOT, "tests", "compat", "compat_search.cpp"),
                    "-o", exe, "-L", os.path.join(ROOT, "fusiongpu_b200"), "-lfusiongpu_b200",
                    "-L", "/usr/local/cuda/lib64", "-lcudart",
                    "-Wl,-rpath," + os.path.join(ROOT, "fusiongpu_b200"), "-Wl,-rpath,/usr/local/cuda/lib64"],
                   check=True, timeout=300)
    return exe


def test_compat_header_reference_signatures(work, tmp_path):
    from fusiongpu_b200 import formats
    exe = _compile_compat(tmp_path)
    d = work["dir"]
    _run([exe, "res", "q.fvecs", "base.fvecs", str(tmp_path / "r"), str(SEARCH["top_m"]), str(SEARCH["rerank_m"]),
          str(SEARCH["final_k"])], cwd=d)
    ids = formats.read_vecs(str(tmp_path / "r.ids.ivecs"), np.int32)
    dists = formats.read_vecs(str(tmp_path / "r.dists.fvecs"), np.float32)
    exp_i, exp_d = oracle.search(work["index"], work["base"], work["q"], ref_compat=True, **SEARCH)
    np.testing.assert_array_equal(ids, exp_i)
    np.testing.assert_array_equal(dists, exp_d)
    # the host-pointer build helpers
    sub = np.ascontiguousarray(work["base"][:3000])
    formats.write_vecs(str(tmp_path / "sub.fvecs"), sub)
    _run([exe, "--kmeans", str(tmp_path / "sub.fvecs"), "16", "5", str(tmp_path / "cen.fvecs")], cwd=d)
    cen = formats.read_vecs(str(tmp_path / "cen.fvecs"), np.float32)
    np.testing.assert_array_equal(cen, oracle.kmeans(sub, 16, 5))
    a = formats.read_vecs(str(tmp_path / "cen.fvecs.assign.ivecs"), np.int32)[0]
    np.testing.assert_array_equal(a, oracle.assign(sub, cen))


def test_probe_budget(work):
    from fusiongpu_b200 import _lib
    from fusiongpu_b200.index import _p
    index = work["index"]
    off = index["offsets"].astype(np.int64)
    nlist = off.size - 1
    rng = np.random.default_rng(3)
    nq, top_m = 300, 12
    pid = np.stack([rng.permutation(nlist)[:top_m] for _ in range(nq)]).astype(np.uint32)
    pd = np.sort(rng.uniform(1, 10, size=(nq, top_m)).astype(np.float32), axis=1)
    pid[5, 3] = 0xFFFFFFFF
    ratio = np.float32(2.0)
    keep = ~(pd > pd[:, :1] * ratio) & (pid != 0xFFFFFFFF)
    lens = np.where(keep, np.diff(off)[np.minimum(pid, nlist - 1).astype(np.int64)], 0)
    exp = lens.sum(1).astype(np.int32)
    t_off = torch.from_numpy(index["offsets"]).cuda()
    t_pid = torch.from_numpy(pid.view(np.int32)).cuda()
    t_pd = torch.from_numpy(pd).cuda()
    cnt = torch.empty(nq, dtype=torch.int32, device="cuda")
    offs = torch.empty(nq + 1, dtype=torch.int32, device="cuda")
    _lib.call("fg_probe_budget", _p(t_off), nlist, _p(t_pid), _p(t_pd), nq, top_m, C.c_float(ratio), _p(cnt),
              _p(offs), None)
    np.testing.assert_array_equal(cnt.cpu().numpy(), exp)
    np.testing.assert_array_equal(offs.cpu().numpy(), np.concatenate([[0], np.cumsum(exp)]).astype(np.int32))
