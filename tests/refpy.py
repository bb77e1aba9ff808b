"""Pure-Python loops restating the reference's search semantics, for tiny
integer-valued cases only (every sum stays below 2**24, so float32 arithmetic
is exact and fused multiply-adds need no emulation).  Used to cross-check the
C oracle, including its tie-breaking and ref_compat quirks.

Follows gpu_global.cu:31-77 (prune), 321-390 (phase 1), 394-426 (threshold),
428-527 (phase 2 with overflow), 838-871 (sort + gather), 603-673 (rerank).
"""
from __future__ import annotations

import numpy as np

FLT_MAX = float(np.finfo(np.float32).max)
INVALID = 0xFFFFFFFF


def toy_index(seed: int, dim: int = 16, pq_m: int = 4, lens=(0, 5, 40, 130, 300, 1100, 60, 200)):
    """Integer centroids/codebook/codes/base so that every distance is exact."""
    rng = np.random.default_rng(seed)
    nlist = len(lens)
    sd = dim // pq_m
    centroids = rng.integers(0, 16, size=(nlist, dim)).astype(np.float32)
    codebook = rng.integers(-3, 4, size=(pq_m, 256, sd)).astype(np.float32)
    total = int(sum(lens))
    offsets = np.zeros(nlist + 1, np.int32)
    offsets[1:] = np.cumsum(lens)
    # few distinct codes per subspace -> many exact distance ties
    codes = rng.integers(0, 6, size=(total, pq_m)).astype(np.uint8)
    ids = rng.permutation(total).astype(np.int32)
    base = rng.integers(0, 16, size=(total, dim)).astype(np.float32)
    index = dict(codebook=codebook, offsets=offsets, ids=ids, codes=codes, centroids=centroids)
    return index, base


def lut(res, codebook):
    pq_m, _, sd = codebook.shape
    t = np.zeros((pq_m, 256), np.float64)
    for m in range(pq_m):
        diff = res[m * sd:(m + 1) * sd][None, :].astype(np.float64) - codebook[m].astype(np.float64)
        t[m] = (diff * diff).sum(1)
    return t


def adc(code, t):
    d = 0.0
    for m in range(len(code)):
        d += t[m, code[m]]
    return d


def batch_logic(index, queries, probe_ids, probe_dists, p):
    cb, off, ids, codes, cen = (index[k] for k in ("codebook", "offsets", "ids", "codes", "centroids"))
    nq = queries.shape[0]
    P, rm = p["top_m"], p["rerank_m"]
    P1 = min(P, p["p1_lists"])
    rc = bool(p["ref_compat"])
    top_ids = np.zeros((nq, rm), np.int32)
    top_d = np.zeros((nq, rm), np.float32)
    counts = np.zeros(nq, np.int32)
    ncand = np.zeros(nq, np.int32)
    for q in range(nq):
        best = float(np.float32(probe_dists[q, 0]))
        pthr = float(np.float32(best * np.float32(p["prune_ratio"])))
        pid = [INVALID if float(probe_dists[q, j]) > pthr else int(probe_ids[q, j]) for j in range(P)]
        cands = []  # (dist, seq, id)
        cut = [0.0] * P1
        for j in range(P1):
            c = pid[j]
            if c == INVALID:
                continue
            s, e = int(off[c]), int(off[c + 1])
            ln = e - s
            if ln == 0:
                continue
            wc = min(ln, p["limit_k"])
            scan = min(ln, 1024) if rc else ln
            t = lut(queries[q] - cen[c], cb)
            ds = sorted((adc(codes[s + i], t), i) for i in range(scan))
            for r in range(min(wc, scan)):
                d, i = ds[r]
                cands.append((d, (j << 20) | i, int(ids[s + i])))
            if wc - 1 < scan:
                cut[j] = ds[wc - 1][0]
        pos = [x for x in cut if x > 0.0]
        thr = float(np.float32(np.float32(min(pos)) * np.float32(p["threshold_coeff"]))) if pos else FLT_MAX
        for j in range(P1, P):
            c = pid[j]
            if c == INVALID:
                continue
            s, e = int(off[c]), int(off[c + 1])
            ln = e - s
            if ln == 0:
                continue
            t = lut(queries[q] - cen[c], cb)
            d = [adc(codes[s + i], t) for i in range(ln)]
            passing = [i for i in range(ln) if d[i] <= thr]
            if not rc or len(passing) <= 128:
                for i in passing:
                    cands.append((d[i], (j << 20) | i, int(ids[s + i])))
            else:
                for i in passing[:128]:
                    cands.append((d[i], (j << 20) | i, int(ids[s + i])))
                quota = len(passing) - 128
                # thread t of 128 walks i = t, t+128, ... re-emitting its first `quota` passing
                per_t = {}
                for i in passing:
                    per_t.setdefault(i % 128, []).append(i)
                re = sorted(i for t_, lst in per_t.items() for i in lst[:quota])
                for i in re:
                    cands.append((d[i], (j << 20) | (1 << 19) | i, int(ids[s + i])))
        cands.sort(key=lambda x: (x[0], x[1]))
        n = len(cands)
        ak = min(n, rm)
        counts[q] = ak
        ncand[q] = n
        for r in range(rm):
            if rc and r >= 128:
                top_ids[q, r], top_d[q, r] = 0, 0.0
            elif r < ak:
                top_ids[q, r], top_d[q, r] = cands[r][2], cands[r][0]
            else:
                top_ids[q, r], top_d[q, r] = -1, FLT_MAX
    return top_ids, top_d, counts, ncand


def rerank(queries, top_ids, top_counts, base, p):
    k, mb, rm = p["final_k"], p["mini_batch"], p["rerank_m"]
    nw = min(128, k + mb) if p["ref_compat"] else k + mb
    nq = queries.shape[0]
    out_i = np.zeros((nq, k), np.int32)
    out_d = np.zeros((nq, k), np.float32)
    for q in range(nq):
        fid = [-1] * k
        fd = [FLT_MAX] * k
        stab = 0
        total = int(top_counts[q])
        off = 0
        while off < rm:
            if off >= total:
                break
            eff = min(mb, total - off)
            w = [(fd[i], i, fid[i]) for i in range(k)]
            for i in range(mb):
                if k + i >= nw:
                    break
                vid, dist = -1, FLT_MAX
                if i < eff:
                    vid = int(top_ids[q, off + i])
                    if 0 <= vid < base.shape[0]:
                        df = queries[q].astype(np.float64) - base[vid].astype(np.float64)
                        dist = float((df * df).sum())
                w.append((dist, k + i, vid))
            w.sort(key=lambda x: (x[0], x[1]))
            new = w[:k]
            chg = sum(1 for (_, _, nid) in new if nid != -1 and nid not in fid)
            stab = stab + 1 if np.float32(chg) / np.float32(k) <= np.float32(p["epsilon"]) else 0
            fid = [x[2] for x in new]
            fd = [x[0] for x in new]
            off += mb
            if stab >= p["beta"]:
                break
        out_i[q] = fid
        out_d[q] = fd
    return out_i, out_d


def rebalance(data, assignment, centroids, kmeans, assign, iters=15, seed=42):
    """The FIFO split loop of build_global.cu:62-169 in plain Python, with the
    k-means and assignment steps passed in (the oracle's).  Returns the new
    assignment and centroids."""
    from collections import deque
    n = data.shape[0]
    k = centroids.shape[0]
    avg = n / k
    split_above = int(avg * 2)
    queue = deque()
    for c in range(k):
        members = np.flatnonzero(assignment == c)
        if members.size:
            queue.append((members, centroids[c]))
    done = []
    while queue:
        ids, cen = queue.popleft()
        if ids.size <= split_above or ids.size < 32:
            done.append((ids, cen))
            continue
        sub_k = max(2, int(np.ceil(ids.size / avg)))
        sub_k = min(sub_k, ids.size // 2)
        sc = kmeans(data[ids], sub_k, iters, seed)
        sa = assign(data[ids], sc)
        kids = [(ids[sa == c], sc[c]) for c in range(sub_k) if np.any(sa == c)]
        (done if len(kids) == 1 else queue).extend(kids)
    out_a = np.empty(n, np.int32)
    for c, (ids, _) in enumerate(done):
        out_a[ids] = c
    return out_a, np.stack([c for _, c in done]).astype(np.float32)
