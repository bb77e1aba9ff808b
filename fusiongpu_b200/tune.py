"""Search-parameter tuning (tune_parameters.cu), on the GPU through the C ABI.

``tune_parameters`` derives the reference's four recommendations (top_m,
p1_lists, limit_k, threshold_coeff) from sampled base vectors used as queries
and their exact neighbours; ``sweep`` then measures recall and throughput
over a grid of nprobe (top_m) and rerank depth, as a user picks the operating
point.  ``save_config`` writes the reference's search_config.txt keys.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from .index import IVFPQIndex, SearchParams, _dev, _p, _stream, knn_exact, recall_at


def mt19937_raw(seed: int, n: int) -> np.ndarray:
    """The first n outputs of MT19937 seeded with init_genrand(seed) (the
    generator of std::mt19937)."""
    rs = np.random.RandomState(seed & 0xFFFFFFFF)
    _, key, pos, _, _ = rs.get_state()
    bg = np.random.MT19937()
    bg.state = {"bit_generator": "MT19937", "state": {"key": key, "pos": pos}}
    return bg.random_raw(n).astype(np.uint32)


def sample_rows(n_base: int, n_samples: int, seed: int = 42) -> np.ndarray:
    """Rows of the base set used as tuning queries: MT19937(seed) output i
    modulo n_base.  (The reference draws them from an unseeded
    std::random_device, tune_parameters.cu:477-484; a seed makes runs
    repeatable.)"""
    return (mt19937_raw(seed, n_samples) % np.uint32(n_base)).astype(np.int64)


def tune_parameters(index: IVFPQIndex, queries, gt, base=None) -> dict:
    """The four recommendations plus the per-neighbour statistics.  ``gt`` is
    [nq][k] int32 (exact neighbours, ascending distance)."""
    dev = index.device
    q = _dev(queries, torch.float32, dev)
    g = _dev(gt, torch.int32, dev)
    b = index.base if base is None else _dev(base, torch.float32, dev)
    if b is None:
        raise ValueError("tuning needs the raw base vectors")
    nq, k = g.shape
    r = _lib.TuneResult()
    cr = np.empty((nq, k), np.int32)
    pr = np.empty((nq, k), np.int32)
    er = np.empty((nq, k), np.int32)
    ra = np.empty(nq, np.float32)
    hp = lambda a: C.c_void_p(a.ctypes.data)  # noqa: E731
    _lib.call("fg_tune", C.byref(index.view), _p(b), b.shape[0], _p(q), nq, _p(g), k, C.byref(r), hp(cr), hp(pr),
              hp(er), hp(ra), _stream())
    out = {f: getattr(r, f) for f, _ in _lib.TuneResult._fields_}
    out.update(cluster_ranks=cr, pq_ranks=pr, exact_ranks=er, ratios=ra)
    return out


def tune_from_base(index: IVFPQIndex, n_samples: int = 1000, k: int = 10, seed: int = 42) -> dict:
    """tune_search_parameters end to end: sample base rows, exact k-NN on the
    GPU, statistics.  Returns the recommendations, the sample rows and the
    ground truth."""
    if index.base is None:
        raise ValueError("tuning needs the raw base vectors")
    rows = sample_rows(index.base.shape[0], n_samples, seed)
    q = index.base[torch.from_numpy(rows).to(index.device)].contiguous()
    gt, _ = knn_exact(index.base, q, k, index.device)
    res = tune_parameters(index, q, gt)
    res.update(rows=rows, queries=q, gt=gt)
    return res


def save_config(path: str, res: dict) -> None:
    """The keys of the reference's search_config.txt (tune_parameters.cu:1015-1053)."""
    with open(path, "w") as f:
        f.write("# search parameters recommended by the tuner\n")
        f.write(f"RECOMMENDED_TOP_M={res['top_m']}\n")
        f.write(f"RECOMMENDED_P1_LISTS={res['p1_lists']}\n")
        f.write(f"RECOMMENDED_LIMIT_K={res['limit_k']}\n")
        f.write(f"THRESHOLD_COEFF={res['threshold_coeff']:.3f}\n")


def load_config(path: str) -> dict:
    keys = {"RECOMMENDED_TOP_M": "top_m", "RECOMMENDED_P1_LISTS": "p1_lists", "RECOMMENDED_LIMIT_K": "limit_k",
            "THRESHOLD_COEFF": "threshold_coeff"}
    out = {}
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line or line.startswith("#") or "=" not in line:
                continue
            k, v = line.split("=", 1)
            if k in keys:
                out[keys[k]] = float(v) if k == "THRESHOLD_COEFF" else int(v)
    return out


def sweep(index: IVFPQIndex, queries, gt: np.ndarray, params: SearchParams, top_ms, rerank_ms, k: int = 10,
          reps: int = 3) -> list[dict]:
    """Recall@k and device-timed QPS of the full search for each (top_m,
    rerank_m); inputs resident on the GPU."""
    q = _dev(queries, torch.float32, index.device)
    gt = np.asarray(gt)
    rows = []
    for tm in top_ms:
        for rm in rerank_ms:
            p = params.replace(top_m=int(tm), rerank_m=int(rm), p1_lists=min(params.p1_lists, int(tm)))
            ids, _ = index.search(q, p)
            rec = recall_at(ids.cpu().numpy(), gt, k)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                index.search(q, p)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            rows.append(dict(top_m=int(tm), rerank_m=int(rm), recall=rec, qps=q.shape[0] / (ms / 1e3), ms=ms))
    return rows


def best_at_recall(rows: list[dict], target: float) -> dict | None:
    ok = [r for r in rows if r["recall"] >= target]
    return max(ok, key=lambda r: r["qps"]) if ok else None


__all__ = ["mt19937_raw", "sample_rows", "tune_parameters", "tune_from_base", "save_config", "load_config", "sweep",
           "best_at_recall"]
