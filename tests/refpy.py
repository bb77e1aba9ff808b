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


# ---- graph index (the product's CAGRA-style build and search) ----------------
# Integer-valued vectors keep every distance exact in float32, so plain numpy
# arithmetic gives the same values as the kernels' fmaf chains; what these
# loops check is the control logic: candidate lists, pruning, reverse edges,
# visited-set resets, parent choice, merging and termination.

def _mix32(h):
    h &= 0xFFFFFFFF
    h ^= h >> 16
    h = (h * 0x85EBCA6B) & 0xFFFFFFFF
    h ^= h >> 13
    h = (h * 0xC2B2AE35) & 0xFFFFFFFF
    h ^= h >> 16
    return h


def graph_seed_node(seed, q, s, S, n):
    x = _mix32(seed ^ _mix32((((q * S + s) & 0xFFFFFFFF) * 0x9E3779B9 + 0x7F4A7C15) & 0xFFFFFFFF))
    return x % n


def _dist(a, b, metric):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(-(a @ b)) if metric == "ip" else float(((a - b) ** 2).sum())


def graph_build(data, D, I, L, P, iters, seed, metric, kmeans, assign, coarse):
    """Steps 1-5 of the graph build with the oracle's k-means/assign/coarse."""
    n = data.shape[0]
    cen = kmeans(data, L, iters, seed)
    a = assign(data, cen)
    lists = [np.flatnonzero(a == c) for c in range(L)]
    nn, _ = coarse(cen, cen, P)
    g0 = -np.ones((n, I), np.int64)
    for c in range(L):
        chosen = [c] + [int(x) for x in nn[c] if int(x) != c][: P - 1]
        cand = np.sort(np.concatenate([lists[l] for l in chosen]))
        kk = min(len(cand), I + 1)
        for u in lists[c]:
            d = sorted((_dist(data[u], data[v], metric), int(v)) for v in cand)[:kk]
            row = [v for _, v in d if v != u][:I]
            g0[u, :len(row)] = row
    pr = -np.ones((n, D), np.int64)
    for u in range(n):
        nb = g0[u]
        keys = []
        for i in range(I):
            if nb[i] < 0:
                keys.append((0xFFFF, i))
                continue
            cnt = sum(1 for j in range(i) if nb[j] >= 0 and nb[i] in g0[nb[j], :i])
            keys.append((cnt, i))
        keys.sort()
        pr[u] = [nb[i] for _, i in keys[:D]]
    rev = [[] for _ in range(n)]
    for i in range(D):
        for u in range(n):
            if pr[u, i] >= 0:
                rev[pr[u, i]].append(u)
    out = -np.ones((n, D), np.int64)
    for u in range(n):
        row = []
        for v in pr[u, :D // 2]:
            if v >= 0 and v not in row:
                row.append(int(v))
        taken = 0
        for v in rev[u]:
            if taken >= D - D // 2 or len(row) >= D:
                break
            if v not in row:
                row.append(v)
                taken += 1
        for v in pr[u, D // 2:]:
            if len(row) >= D:
                break
            if v >= 0 and v not in row:
                row.append(int(v))
        out[u, :len(row)] = row
    return out.astype(np.int32)


def graph_search(data, graph, queries, itopk, width, max_iter, k, seed, metric, hash_slots=4096,
                 entry_centroids=None, entry_nodes=None, entry_probes=0):
    n, D = graph.shape
    if max_iter == 0:
        max_iter = 2 * ((itopk + width - 1) // width) + 10
    WD = width * D
    out_i = -np.ones((len(queries), k), np.int32)
    out_d = np.full((len(queries), k), FLT_MAX, np.float32)
    evals = expanded = 0
    for q, qv in enumerate(queries):
        top = []        # [(dist, id, explored)]
        vis = set()
        for it in range(-1, max_iter):
            if it < 0:
                S = 0
                if entry_probes:
                    S = min(entry_probes, len(entry_nodes), WD)
                    ed = sorted((_dist(qv, c, metric), ci) for ci, c in enumerate(entry_centroids))
                    first = [int(entry_nodes[ci]) for _, ci in ed[:S]]
                else:
                    first = []
                slots = first + [graph_seed_node(seed, q, s, WD, n) for s in range(S, WD)]
            else:
                par = []
                for e in top:
                    if len(par) == width:
                        break
                    if not e[2]:
                        par.append(e[1])
                        e[2] = True
                if not par:
                    break
                expanded += len(par)
                if len(vis) > hash_slots // 2:
                    vis = {e[1] for e in top}
                slots = [int(graph[par[s // D], s % D]) if s // D < len(par) else -1 for s in range(WD)]
            fresh = []
            for v in slots:
                if 0 <= v < n and v not in vis:
                    vis.add(v)
                    fresh.append(v)
            evals += len(fresh)
            cand = [[np.float32(_dist(data[v], qv, metric)), v, False] for v in fresh]
            top = sorted(top + cand, key=lambda e: (e[0], e[1]))[:itopk]
        for r, e in enumerate(top[:k]):
            out_i[q, r] = e[1]
            out_d[q, r] = e[0]
    return out_i, out_d, (evals, expanded)
