#!/usr/bin/env python
"""Benchmark: QPS at recall@10 = 0.95 on the C2 workload (1M x 128 IVF-PQ,
nlist 4096, PQ 64x8, k=100, exact rerank of the top 1000), nprobe swept over
{8,16,32,64,128} and QPS interpolated at the recall target.

A step is one search of the whole 10,000-query batch at one nprobe.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl fusiongpu|reference]

Under torchrun every rank holds a full replica of the index and searches its
own copy of the batch (replicas; per-GPU work is fixed, scaling "weak").
`--impl reference` times the CPU restatement of the reference's search (the
oracle) on the host cores instead; only rank 0 works.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

RECALL_TARGET = 0.95
# BASELINE's sweep is {8..128}; 1/2/4 extend it downwards so the QPS at the
# recall target is interpolated between points that bracket it
SWEEP = (1, 2, 4, 8, 16, 32, 64, 128)
CONFIG = dict(workload="C2: 1,000,000 x 128 fp32 integer-valued Gaussian mixture (4096 centres, sigma 10), "
                       "10,000 queries, L2",
              nlist=4096, pq_m=64, k=100, rerank_m=1000, p1_lists=12, limit_k=50, threshold_coeff=1.0,
              mini_batch=128, epsilon=0.1, beta=2, nprobe_sweep=list(SWEEP), recall="recall@10",
              mode="intended (full rerank_m gather, k+mini_batch rerank window)")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="fusiongpu", choices=["fusiongpu", "reference"])
    ap.add_argument("--cpu-sample", type=int, default=4000, help="queries in the CPU-baseline sample")
    ap.add_argument("--nprobe", type=int, default=0, help="time this nprobe only (profiling)")
    ap.add_argument("--profile", default="", choices=["", "scan", "coarse", "rerank", "search", "graph"],
                    help="build the index, then run only this stage warmup+1 times (for ncu)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--quick", action="store_true", help="small workload (development only)")
    ap.add_argument("--index-dir", default="", help="--profile: load the C2 index from here (build and save it "
                                                   "there when absent), so a profiler sees only the search")
    ap.add_argument("--workload", default="C2", choices=["C2", "C3", "C4", "C5"],
                    help="C2: IVF-PQ headline (default); C3: 10M x 96 IVF-PQ (HBM-bound scan); "
                         "C4: graph index (1M x 768 fp16, IP); C5: 100M x 128 uint8, lists sharded across GPUs")
    return ap.parse_args()


def interp_at_recall(points, target=RECALL_TARGET):
    """points: [(nprobe, recall, qps)] in nprobe order.  QPS at `target` by
    linear interpolation in recall between the bracketing sweep points."""
    pts = sorted(points, key=lambda p: p[0])
    if pts[0][1] >= target:
        return pts[0][2], True
    for a, b in zip(pts, pts[1:]):
        if a[1] < target <= b[1]:
            t = (target - a[1]) / (b[1] - a[1])
            return a[2] + t * (b[2] - a[2]), True
    best = max(pts, key=lambda p: p[1])
    return best[2], False


def search_params(nprobe, SearchParams, ref_compat=False):
    return SearchParams(top_m=nprobe, p1_lists=CONFIG["p1_lists"], limit_k=CONFIG["limit_k"],
                        threshold_coeff=CONFIG["threshold_coeff"], prune_ratio=100.0,
                        rerank_m=CONFIG["rerank_m"], final_k=CONFIG["k"], mini_batch=CONFIG["mini_batch"],
                        epsilon=CONFIG["epsilon"], beta=CONFIG["beta"], ref_compat=ref_compat)


def oracle_kw(p):
    return dict(top_m=p.top_m, p1_lists=p.p1_lists, limit_k=p.limit_k, threshold_coeff=p.threshold_coeff,
                prune_ratio=p.prune_ratio, rerank_m=p.rerank_m, final_k=p.final_k, mini_batch=p.mini_batch,
                epsilon=p.epsilon, beta=p.beta, ref_compat=bool(p.ref_compat))


def compare_results(gi, gd, oi, od):
    """(ids differing where the distances differ by more than 1e-5 relative,
    the largest relative distance difference) between two [nq][k] results."""
    gd = gd.astype(np.float64)
    od = od.astype(np.float64)
    with np.errstate(invalid="ignore", divide="ignore"):
        rel = np.where(gd == od, 0.0, np.abs(gd - od) / np.maximum(np.abs(od), 1e-30))
    rel = np.nan_to_num(rel, nan=np.inf)
    mism = int(((gi != oi) & (rel > 1e-5)).sum())
    return mism, float(rel.max()) if rel.size else 0.0


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.05)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


def workload(quick: bool):
    from fusiongpu_b200 import datasets as ds
    if quick:
        return ds.scaled(ds.C2, 200_000, 2_000, n_centres=1024), 1024
    return ds.C2, CONFIG["nlist"]


def setup(device, quick):
    """Data, GPU-built index and exact ground truth (untimed)."""
    import torch
    from fusiongpu_b200 import datasets as ds
    from fusiongpu_b200.index import IVFPQIndex, knn_exact
    spec, nlist = workload(quick)
    t0 = time.time()
    base, queries = ds.generate(spec)
    xb = torch.from_numpy(base).to(device)
    idx = IVFPQIndex.build(xb, nlist, CONFIG["pq_m"], kmeans_iters=20, pq_sample=50000, pq_iters=8, device=device)
    # the ground truth both arms use (exact_gt), and the library's own exact
    # k-NN beside it as a check
    gt = exact_gt(base, queries, 10, device)
    g2, _ = knn_exact(xb, torch.from_numpy(queries).to(device), 10, device=device)
    torch.cuda.synchronize(device)
    return dict(spec=spec, base=base, queries=queries, index=idx, gt=gt, setup_s=time.time() - t0,
                gt_equals_knn_exact=bool(np.array_equal(gt, g2.cpu().numpy())))


def main():
    args = parse()
    if args.workload == "C4":
        return main_c4(args)
    if args.workload == "C3":
        return main_c3(args)
    if args.workload == "C5":
        return main_c5(args)
    if args.impl == "reference":
        return main_reference(args)
    import torch
    import torch.distributed as dist
    from fusiongpu_b200.index import SearchParams, recall_at

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.profile:
        return profile_stage(args, device)
    if world > 1:
        return main_sharded(args, rank, world, local, device, barrier, max_over_ranks)
    W = setup(device, args.quick)
    idx, queries, gt = W["index"], W["queries"], W["gt"]
    nq = queries.shape[0]
    qd = torch.from_numpy(queries).to(device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)  # > 126 MB L2
    stream = torch.cuda.current_stream(device)
    sweep = []
    def launches_per_step(nprobe):
        # two bf16 splits + coarse GEMM + finish (top_m <= 4), or splits + prefix GEMM
        # + bound + filter GEMM + finish; then the scan (the team kernel, or from 8 probes
        # with every probe in phase 1 the group path: pair count, scan, scatter, group cut,
        # group kernel, selection) and the rerank
        scan = 6 if 8 <= nprobe <= CONFIG["p1_lists"] else 1
        return (4 if nprobe <= 4 else 6) + scan + 1
    clocks = ClockSampler(local)

    def run_sweep(ref_compat):
        out = []
        for nprobe in (SWEEP if not args.nprobe else (args.nprobe,)):
            p = search_params(nprobe, SearchParams, ref_compat)
            ids = torch.empty((nq, p.final_k), dtype=torch.int32, device=device)
            dd = torch.empty((nq, p.final_k), dtype=torch.float32, device=device)
            for _ in range(args.warmup):
                idx.search(qd, p, out=(ids, dd))
            torch.cuda.synchronize(device)
            rec = recall_at(ids[:, :10].cpu().numpy(), gt[:, :10], 10)
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.steps)]
            barrier()
            torch.cuda.synchronize(device)
            for e0, e1 in ev:
                flush.zero_()  # L2 flush between steps, outside the timed region
                e0.record(stream)
                idx.search(qd, p, out=(ids, dd))
                e1.record(stream)
            torch.cuda.synchronize(device)
            barrier()
            ms = sum(e0.elapsed_time(e1) for e0, e1 in ev) / args.steps
            ms = max_over_ranks(ms)
            out.append(dict(nprobe=nprobe, recall=rec, ms_per_step=ms, qps=world * nq / (ms / 1e3)))
        return out

    with clocks:
        sweep = run_sweep(False)
        # the reference's own output semantics (128-entry gather and rerank window)
        sweep_rc = run_sweep(True)

    pts = [(s["nprobe"], s["recall"], s["qps"]) for s in sweep]
    value, met = interp_at_recall(pts)
    op = next((s for s in sweep if s["recall"] >= RECALL_TARGET), max(sweep, key=lambda s: s["recall"]))
    rc_value, rc_met = interp_at_recall([(s["nprobe"], s["recall"], s["qps"]) for s in sweep_rc])
    op_rc = next((s for s in sweep_rc if s["recall"] >= RECALL_TARGET), max(sweep_rc, key=lambda s: s["recall"]))

    # ---- end to end through the public API: pinned host queries in, host results out
    E2E_CHUNKS = int(os.environ.get("FG_E2E_CHUNKS", "2"))
    E2E_GRAPH = os.environ.get("FG_E2E_GRAPH", "1") != "0"  # one graph launch per step
    e2e_pts = []
    hq = torch.from_numpy(queries).pin_memory()
    for s in sweep:
        p = search_params(s["nprobe"], SearchParams)
        hid = torch.empty((nq, p.final_k), dtype=torch.int32).pin_memory()
        hdd = torch.empty((nq, p.final_k), dtype=torch.float32).pin_memory()

        def one():
            # the public host-buffer call: uploads, kernels and result writes replayed
            # as one CUDA graph (captured in the first warm-up call)
            idx.search_host(hq, p, out=(hid, hdd), chunks=E2E_CHUNKS, graph=E2E_GRAPH)

        for _ in range(max(1, args.warmup)):
            one()
        torch.cuda.synchronize(device)
        barrier()
        tot = 0.0
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            one()
            e1.record(stream)
            e1.synchronize()
            tot += e0.elapsed_time(e1)
        barrier()
        ms = max_over_ranks(tot / args.steps)
        e2e_pts.append((s["nprobe"], s["recall"], world * nq / (ms / 1e3)))
        s["e2e_ms_per_step"] = ms
    e2e_value, _ = interp_at_recall(e2e_pts)

    # ---- roofline of the dominant kernel (ADC scan = candidate generation) at the operating point
    roof = roofline(idx, qd, op["nprobe"], args, device, SearchParams, flush)

    out = {
        "metric": "QPS at recall@10=0.95 (C2 1M x 128 IVF-PQ)",
        "value": value,
        "unit": "queries/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": op["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture standing in for a dataset; index built on the GPU)",
        "config": dict(CONFIG, parallelism=f"replicas x{world} (full index per GPU, own 10k-query batch)",
                       l2="flushed (256 MB write) between timed steps",
                       recall_target_met=met, operating_nprobe=op["nprobe"],
                       quick=bool(args.quick), lists=idx.nlist,
                       recall_on=f"all {nq} queries (exact float64 ground truth; equals fg_knn_exact: "
                                 f"{W['gt_equals_knn_exact']})"),
        "sweep": sweep,
        "ref_compat": {"mode": "reference output semantics (ref_compat=1: 128-lane gather, 128-entry rerank "
                               "window, phase-1 clamp, phase-2 overflow re-emission)",
                       "value": rc_value, "recall_target_met": rc_met, "operating_nprobe": op_rc["nprobe"],
                       "ms_per_step": op_rc["ms_per_step"], "sweep": sweep_rc},
        "e2e": {"value": e2e_value, "unit": "queries/s", "h2d_bytes_per_step": int(queries.nbytes),
                "d2h_bytes_per_step": int(nq * CONFIG["k"] * 8)},
        # this library's kernels inside timed regions: the two device sweeps, the
        # host-buffer sweep (E2E_CHUNKS searches per step), the scan-only timing
        "gpu_launches": (sum(launches_per_step(s["nprobe"]) for s in sweep + sweep_rc)
                         + E2E_CHUNKS * sum(launches_per_step(s["nprobe"]) for s in sweep) + 1) * args.steps,
        "gpu_launches_per_step": launches_per_step(op["nprobe"]),
        "roofline": roof,
        "clocks": clocks.summary(),
        "setup_s": W["setup_s"],
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        out["cpu_baseline"], out["parity"] = cpu_baseline_and_parity(W, idx, qd, op["nprobe"], args.cpu_sample,
                                                                     SearchParams)
        out["ref_gpu"] = ref_gpu_block(W, idx, qd, args, device, SearchParams, flush)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main_sharded(args, rank, world, local, device, barrier, max_over_ranks):
    """C2 on N GPUs as the list-sharded search: every rank builds the same
    (deterministic) index and keeps the lists LPT deals it, with their codes,
    ids and raw vectors; the 10,000 queries go to every rank; each rank runs
    the exact coarse search (centroids replicated), scans and reranks its own
    lists, and one NCCL all-gather of packed (distance, global id) keys feeds
    the device merge.  Strong scaling: the batch is the same at every N.
    Times are CUDA events per rank, the max over ranks."""
    import torch
    import torch.distributed as dist
    from fusiongpu_b200.index import SearchParams, recall_at
    from fusiongpu_b200.sharded import ShardedIndex, elapsed_ms
    W = setup(device, args.quick)
    idx, queries, gt = W["index"], W["queries"], W["gt"]
    host = idx.to_numpy()
    nlists = idx.nlist
    del idx, W["index"]
    torch.cuda.empty_cache()
    sh = ShardedIndex(host, W["base"], rank, world, device=device)
    nq = queries.shape[0]
    qd = torch.from_numpy(queries).to(device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    sweep = []
    clocks = ClockSampler(local)
    with clocks:
        for nprobe in (SWEEP if not args.nprobe else (args.nprobe,)):
            p = search_params(nprobe, SearchParams)
            for _ in range(args.warmup):
                ids, dd = sh.search(qd, p)
            torch.cuda.synchronize(device)
            rec = recall_at(ids[:, :10].cpu().numpy(), gt[:, :10], 10)
            barrier()
            torch.cuda.synchronize(device)
            tot = 0.0
            stages = {}
            for _ in range(args.steps):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                sh.search(qd, p, timings=stages)
                e1.record(stream)
                e1.synchronize()
                tot += e0.elapsed_time(e1)
            barrier()
            ms = max_over_ranks(tot / args.steps)
            st = {k: max_over_ranks(v) for k, v in sorted(elapsed_ms(stages).items())}
            sweep.append(dict(nprobe=nprobe, recall=rec, ms_per_step=ms, qps=nq / (ms / 1e3), stage_ms=st))
    pts = [(s_["nprobe"], s_["recall"], s_["qps"]) for s_ in sweep]
    value, met = interp_at_recall(pts)
    op = next((s_ for s_ in sweep if s_["recall"] >= RECALL_TARGET), max(sweep, key=lambda s_: s_["recall"]))
    # end to end: pinned host queries in, every rank's merged result back to pinned host memory
    hq = torch.from_numpy(queries).pin_memory()
    e2e_pts = []
    for s_ in sweep:
        p = search_params(s_["nprobe"], SearchParams)
        hid = torch.empty((nq, p.final_k), dtype=torch.int32).pin_memory()
        hdd = torch.empty((nq, p.final_k), dtype=torch.float32).pin_memory()
        qdev = torch.empty_like(qd)
        barrier()
        tot = 0.0
        for i in range(args.warmup + args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            qdev.copy_(hq, non_blocking=True)
            r_ids, r_d = sh.search(qdev, p)
            hid.copy_(r_ids, non_blocking=True)
            hdd.copy_(r_d, non_blocking=True)
            e1.record(stream)
            e1.synchronize()
            if i >= args.warmup:
                tot += e0.elapsed_time(e1)
        barrier()
        ms = max_over_ranks(tot / args.steps)
        s_["e2e_ms_per_step"] = ms
        e2e_pts.append((s_["nprobe"], s_["recall"], nq / (ms / 1e3)))
    e2e_value, _ = interp_at_recall(e2e_pts)
    n_local = torch.tensor([sh.n_local], dtype=torch.int64, device=device)
    all_local = [torch.zeros_like(n_local) for _ in range(world)]
    dist.all_gather(all_local, n_local)
    out = {
        "metric": "QPS at recall@10=0.95 (C2 1M x 128 IVF-PQ)",
        "value": value,
        "unit": "queries/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": op["ms_per_step"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture standing in for a dataset; index built on the GPU)",
        "config": dict(CONFIG, parallelism=f"inverted lists dealt to {world} GPUs by length (LPT); queries "
                                           "broadcast; exact coarse replicated; one NCCL all-gather of packed "
                                           "(distance, global id) keys; device merge",
                       vectors_per_gpu=[int(t.item()) for t in all_local], lists=nlists,
                       l2="flushed (256 MB write) between timed steps", recall_target_met=met,
                       operating_nprobe=op["nprobe"], quick=bool(args.quick),
                       allgather_bytes_per_rank=int(nq * CONFIG["k"] * 8)),
        "sweep": sweep,
        "e2e": {"value": e2e_value, "unit": "queries/s", "h2d_bytes_per_step": int(queries.nbytes),
                "d2h_bytes_per_step": int(nq * CONFIG["k"] * 8)},
        # per search: the coarse stage (4 or 6), scan, rerank, pack, merge; device and e2e sweeps
        "gpu_launches": sum((4 if s_["nprobe"] <= 4 else 6) + 4 for s_ in sweep) * args.steps * 2,
        "clocks": clocks.summary(),
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
    dist.destroy_process_group()


def profile_stage(args, device):
    """Index build, coarse probes, then warmup+1 launches of one stage alone:
    the target of `ncu -k regex:<kernel> -s <warmup> -c 1`."""
    import torch
    from fusiongpu_b200 import datasets as ds
    from fusiongpu_b200.index import IVFPQIndex, SearchParams, run_gpu_batch_logic, run_gpu_rerank
    spec, nlist = workload(args.quick)
    base, queries = ds.generate(spec)
    d = args.index_dir
    if d and os.path.exists(os.path.join(d, "ivf_data.bin")):
        idx = IVFPQIndex.load(d, CONFIG["pq_m"], spec.dim, base=base, device=device)
    else:
        idx = IVFPQIndex.build(torch.from_numpy(base).to(device), nlist, CONFIG["pq_m"], device=device)
        if d:
            os.makedirs(d, exist_ok=True)
            idx.save(d)
    qd = torch.from_numpy(queries).to(device)
    nprobe = args.nprobe or 8
    p = search_params(nprobe, SearchParams)
    pid, pd = idx.coarse(qd, nprobe)
    ti, td, tc, cc = run_gpu_batch_logic(idx, qd, pid, pd, p)
    torch.cuda.synchronize(device)
    torch.cuda.profiler.start()  # ncu --profile-from-start off: skip the build's launches
    for _ in range(args.warmup + 1):
        if args.profile == "scan":
            run_gpu_batch_logic(idx, qd, pid, pd, p)
        elif args.profile == "coarse":
            idx.coarse(qd, nprobe)
        elif args.profile == "rerank":
            run_gpu_rerank(qd, ti, tc, idx.base, p, device)
        else:
            idx.search(qd, p)
    torch.cuda.synchronize(device)
    print(json.dumps({"profile": args.profile, "nprobe": nprobe, "nq": int(queries.shape[0]),
                      "max_list_len": idx.max_list_len}))


def roofline(idx, qd, nprobe, args, device, SearchParams, flush):
    """Algorithmic bytes of the scan kernel per launch (code bytes of every
    probed list + 4 bytes per emitted candidate) over its CUDA-event time."""
    import torch
    from fusiongpu_b200.index import run_gpu_batch_logic
    p = search_params(nprobe, SearchParams)
    pid, pd = idx.coarse(qd, nprobe)
    lens = (idx.offsets[1:] - idx.offsets[:-1]).to(torch.int64)
    code_bytes = int(lens[pid.long()].sum().item()) * idx.pq_m
    for _ in range(args.warmup):
        ti, td, tc, cc = run_gpu_batch_logic(idx, qd, pid, pd, p)
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    tot = 0.0
    for _ in range(args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ti, td, tc, cc = run_gpu_batch_logic(idx, qd, pid, pd, p)
        e1.record(stream)
        e1.synchronize()
        tot += e0.elapsed_time(e1)
    ms = tot / args.steps
    cand_bytes = 4 * int(cc.to(torch.int64).sum().item())
    alg = code_bytes + cand_bytes
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = alg / (ms / 1e3) / 1e9
    traffic = None
    try:
        tr = json.load(open(os.path.join(ROOT, "profiles", "scan_traffic.json")))
        if tr.get("nprobe") == nprobe and tr.get("workload") == "C2":
            traffic = tr["dram_bytes_per_launch"]
    except Exception:
        pass
    # the library's scan dispatch: the team kernel on short lists (typical length <= 400: the larger of the
    # mean and half the longest list), else the split path
    typical = max(idx.total / max(idx.nlist, 1), 0.5 * idx.max_list_len)
    kernel = "ivfpq_team_kernel" if typical <= 400 else "split_phase_kernel (phase 1 + phase 2)"
    return {"kernel": kernel, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
            "traffic": traffic, "algorithmic_bytes": alg, "ms_per_launch": ms, "nprobe": nprobe}


def cpu_baseline_and_parity(W, idx, qd, nprobe, sample, SearchParams):
    """The oracle (C restatement of the reference search, OpenMP over all
    host cores) on the first `sample` queries at the operating nprobe: its
    time is the CPU baseline, and its results -- in the intended and in the
    reference (ref_compat) mode -- are compared with the GPU search of the
    same queries on the same index: ids that differ where the distances
    differ by more than 1e-5 relative, the largest relative distance error,
    and recall@10 of both on this one query set."""
    import oracle
    from fusiongpu_b200.index import recall_at
    index = W["index"].to_numpy()
    q = np.ascontiguousarray(W["queries"][:sample])
    gt = W["gt"][:sample, :10]
    cores = os.cpu_count() or 1
    parity = {"queries": int(sample), "nprobe": int(nprobe), "tie_rule": "ids may differ where distances are "
              "within 1e-5 relative", "index": "the GPU arm's index", "modes": {}}
    cpu = None
    for mode, rc in (("intended", False), ("ref_compat", True)):
        p = search_params(nprobe, SearchParams, rc)
        kw = oracle_kw(p)
        if cpu is None:
            oracle.search(index, W["base"], q[:8], nthreads=cores, **kw)  # warm caches
        t0 = time.perf_counter()
        oi, od = oracle.search(index, W["base"], q, nthreads=cores, **kw)
        dt = time.perf_counter() - t0
        if cpu is None:
            cpu = {"value": sample / dt, "unit": "queries/s", "cores": cores, "kind": "port",
                   "sample": f"first {sample} of {W['queries'].shape[0]} queries at nprobe={nprobe}, same index "
                             "(intended mode)", "seconds": dt}
        gi, gd = idx.search(qd[:sample].contiguous(), p)
        gi, gd = gi.cpu().numpy(), gd.cpu().numpy()
        mism, rel = compare_results(gi, gd, oi, od)
        parity["modes"][mode] = {"id_mismatches_beyond_1e-5_ties": mism, "max_rel_dist_err": rel,
                                 "bit_exact": bool(np.array_equal(gi, oi) and np.array_equal(gd, od)),
                                 "recall_gpu": recall_at(gi[:, :10], gt, 10),
                                 "recall_oracle": recall_at(oi[:, :10], gt, 10)}
    return cpu, parity


REF_GPU_NPROBE = (1, 2, 4, 8, 16, 32)
REF_GPU_BATCHES = (128, 10000)
# the reference's LUT buffer holds bs * top_m * M * 256 floats (gpu_global.cu:108-160)
REF_GPU_TABLE_LIMIT = 24 << 30


def _ref_gg(dim, pq_m):
    """The reference's gpu_global.cu built for (dim, pq_m) under oracle/_ref,
    with the timing-context entry points typed, or None."""
    import ctypes as C
    import oracle
    L = oracle.ref_lib("gg", dim, pq_m)
    if L is None or not hasattr(L, "ref_ctx_create"):
        return None
    P, I, F = C.c_void_p, C.c_int, C.c_float
    L.ref_ctx_create.restype = P
    L.ref_ctx_create.argtypes = [I, I, I, I, I]
    L.ref_ctx_destroy.argtypes = [P]
    L.ref_ctx_stream.restype = P
    L.ref_ctx_stream.argtypes = [P]
    L.ref_ctx_search.restype = I
    L.ref_ctx_search.argtypes = [P, P, P, P, P, P, I, P, I, P, P, P, I, I, F, I, I, F, I, F, I, P, P, P]
    return L


def ref_gpu_block(W, idx, qd, args, device, SearchParams, flush):
    """The reference's own search kernels (gpu_global.cu:667-874, compiled for
    sm_100a under oracle/_ref) on this GPU, on the GPU arm's index, with the
    exact probe lists injected where the reference calls CAGRA
    (search_pipeline.cu:341): run_gpu_batch_logic + run_gpu_rerank per batch
    of 128 (the reference's default, search_pipeline.cu:562) and of the whole
    10,000, on one stream (its function-static scratch is shared by all
    streams), timed with CUDA events on that stream.  Beside each: this
    engine's candidate generation + rerank (fg_batch_logic + fg_rerank,
    ref_compat mode) on the same probes and batch, and how many query rows
    return other ids than ours.  A point with probes beyond p1_lists runs
    the reference's phase 2, whose overflow re-emission can write past a
    query's candidate region: it runs only where the oracle shows every
    query's candidate count within its region."""
    import ctypes as C
    import torch
    import oracle
    from fusiongpu_b200.index import recall_at, run_gpu_batch_logic, run_gpu_rerank
    L = _ref_gg(idx.dim, idx.pq_m)
    if L is None:
        return {"unavailable": f"oracle/_ref/libref_gg_{idx.dim}_{idx.pq_m}.so not built (reference sources absent)"}
    nq = qd.shape[0]
    gt = W["gt"][:, :10]
    index_np = None
    P = lambda t: C.c_void_p(t.data_ptr())
    steps = max(1, min(args.steps, 5))
    lens = (idx.offsets[1:] - idx.offsets[:-1]).to(torch.int64)
    res = {"what": "reference run_gpu_batch_logic + run_gpu_rerank (no coarse stage: exact probes injected) vs "
                   "fg_batch_logic + fg_rerank (ref_compat) on the same probes",
           "steps": steps, "stream": "one (the reference's static scratch is shared across streams)", "points": []}
    for nprobe in REF_GPU_NPROBE:
        p = search_params(nprobe, SearchParams, True)
        pid, pd = idx.coarse(qd, nprobe)
        torch.cuda.synchronize(device)
        point = {"nprobe": nprobe}
        if nprobe > p.p1_lists:
            if index_np is None:
                index_np = idx.to_numpy()
            pid_np, pd_np = pid.cpu().numpy().view(np.uint32), pd.cpu().numpy()
            _, _, _, st = oracle.batch_logic(index_np, W["queries"], pid_np, pd_np, nthreads=os.cpu_count() or 1,
                                             **oracle_kw(p))
            budget = np.where(pd_np > pd_np[:, :1] * np.float32(p.prune_ratio), 0,
                              lens.cpu().numpy()[pid_np.astype(np.int64)]).sum(1)
            if not (st["count"] <= budget).all():
                point["skipped"] = "candidate count beyond its region for some query (phase-2 overflow)"
                res["points"].append(point)
                continue
        # ours, same probes, whole batch
        ours = []
        for _ in range(args.warmup):
            ti, td, tc, cc = run_gpu_batch_logic(idx, qd, pid, pd, p)
            oi, od = run_gpu_rerank(qd, ti, tc, idx.base, p, device)
        stream = torch.cuda.current_stream(device)
        for _ in range(steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            ti, td, tc, cc = run_gpu_batch_logic(idx, qd, pid, pd, p)
            oi, od = run_gpu_rerank(qd, ti, tc, idx.base, p, device)
            e1.record(stream)
            e1.synchronize()
            ours.append(e0.elapsed_time(e1))
        oi, od = oi.cpu().numpy(), od.cpu().numpy()
        point["fusiongpu_ms_per_10k"] = sum(ours) / len(ours)
        point["recall_fusiongpu"] = recall_at(oi[:, :10], gt, 10)
        for bs in REF_GPU_BATCHES:
            key = f"batch_{bs}"
            if bs * nprobe * idx.pq_m * 256 * 4 > REF_GPU_TABLE_LIMIT:
                point[key] = {"skipped": "the reference's LUT buffer would exceed 24 GB"}
                continue
            ctx = L.ref_ctx_create(bs, nprobe, p.rerank_m, p.final_k, p.p1_lists)
            if not ctx:
                point[key] = {"skipped": "allocation failed"}
                continue
            try:
                rs = torch.cuda.ExternalStream(L.ref_ctx_stream(ctx), device=device)
                fi = torch.zeros((nq, p.final_k), dtype=torch.int32, device=device)
                fd = torch.zeros((nq, p.final_k), dtype=torch.float32, device=device)
                cnt = torch.zeros(nq, dtype=torch.int32, device=device)
                pid_u = pid.contiguous()

                def one_pass():
                    for lo in range(0, nq, bs):
                        hi = min(nq, lo + bs)
                        rc = L.ref_ctx_search(ctx, P(idx.codebook), P(idx.offsets), P(idx.codes), P(idx.ids),
                                              P(idx.centroids), idx.nlist, P(idx.base), idx.base.shape[0],
                                              C.c_void_p(qd[lo].data_ptr()), C.c_void_p(pid_u[lo].data_ptr()),
                                              C.c_void_p(pd[lo].data_ptr()), hi - lo, nprobe, p.prune_ratio,
                                              p.p1_lists, p.limit_k, p.threshold_coeff, p.mini_batch, p.epsilon,
                                              p.beta, C.c_void_p(fi[lo].data_ptr()), C.c_void_p(fd[lo].data_ptr()),
                                              C.c_void_p(cnt[lo].data_ptr()))
                        if rc != 0:
                            raise RuntimeError(f"reference search failed: cuda error {rc}")

                torch.cuda.synchronize(device)
                one_pass()  # grows the reference's pools (its own cudaMalloc) outside the timing
                torch.cuda.synchronize(device)
                tms = []
                for _ in range(steps):
                    flush.zero_()
                    torch.cuda.synchronize(device)
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(rs)
                    one_pass()
                    e1.record(rs)
                    e1.synchronize()
                    tms.append(e0.elapsed_time(e1))
                ri, rd = fi.cpu().numpy(), fd.cpu().numpy()
                mism, rel = compare_results(ri, rd, oi, od)
                ms = sum(tms) / len(tms)
                point[key] = {"ms_per_10k": ms, "qps": nq / (ms / 1e3), "recall": recall_at(ri[:, :10], gt, 10),
                              "rows_with_other_ids": int((ri != oi).any(1).sum()),
                              "id_mismatches_beyond_1e-5_ties": mism, "max_rel_dist_err": rel,
                              "candidate_counts_equal": bool(np.array_equal(cnt.cpu().numpy(), cc.cpu().numpy())),
                              "speedup_fusiongpu": ms / point["fusiongpu_ms_per_10k"]}
            finally:
                torch.cuda.synchronize(device)
                L.ref_ctx_destroy(ctx)
        res["points"].append(point)
    return res


def recall10(results, gt):
    """compute_recall (search_pipeline.cu:531-557): hits of the first 10
    predicted ids (deduplicated) in the ground-truth rows, over nq*10."""
    hits = 0
    for r, g in zip(results[:, :10].tolist(), gt[:, :10].tolist()):
        hits += len(set(r) & set(g))
    return hits / (results.shape[0] * 10)


def exact_gt(base, queries, k, device, chunk=1000):
    """Exact L2 k-NN in float64 on the GPU (torch matmul), ties by lower id.
    The C2 vectors are integers in [0, 255], so every distance is an integer
    below 2^25 and float64 holds it exactly whatever the summation order;
    the key distance * 2^20 + id (ids < 2^20) is then exact too."""
    import torch
    b = torch.from_numpy(np.ascontiguousarray(base)).to(device, torch.float64)
    bn = (b * b).sum(1)
    ids = torch.arange(b.shape[0], device=device, dtype=torch.float64)
    out = []
    for lo in range(0, queries.shape[0], chunk):
        q = torch.from_numpy(np.ascontiguousarray(queries[lo:lo + chunk])).to(device, torch.float64)
        d = bn[None, :] + (q * q).sum(1)[:, None] - 2.0 * (q @ b.T)
        key = d * float(1 << 20) + ids[None, :]
        out.append(torch.topk(key, k, dim=1, largest=False).indices.to(torch.int32).cpu())
        del d, key
    return torch.cat(out).numpy()


def reference_build(base, nlist, pq_m):
    """The index the reference's own build_global writes for this data:
    oracle/_ref/ref_build_global_<dim>_<pq_m>_<nlist> (build_global.cu
    compiled from its sources with these constants) runs in a scratch
    directory on a .fvecs copy of the base, and its ivf_data.bin and
    global_pq_codebook.bin are read back (formats.load_index, numpy only).
    Returns (index dict, seconds) or (None, reason)."""
    import shutil
    import subprocess
    import tempfile
    from fusiongpu_b200 import formats
    dim = base.shape[1]
    exe = os.path.join(ROOT, "oracle", "_ref", f"ref_build_global_{dim}_{pq_m}_{nlist}")
    if not os.path.exists(exe):
        return None, f"{os.path.relpath(exe, ROOT)} not built (reference sources absent when built)"
    tmp = tempfile.mkdtemp(prefix="fg_refbuild_")
    try:
        os.makedirs(os.path.join(tmp, "run"))
        os.makedirs(os.path.join(tmp, "res"))
        fv = os.path.join(tmp, "base.fvecs")
        formats.write_vecs(fv, np.ascontiguousarray(base, np.float32))
        t0 = time.time()
        r = subprocess.run([exe, fv], cwd=os.path.join(tmp, "run"), capture_output=True, text=True, timeout=1200)
        dt = time.time() - t0
        if r.returncode != 0:
            raise RuntimeError(f"reference build_global failed ({r.returncode}): {r.stderr[-500:]}")
        return formats.load_index(os.path.join(tmp, "res"), pq_m, dim), dt
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def main_reference(args):
    """CPU arm: the oracle restating the reference's search on the host cores,
    same workload, metric and sweep, each step a bounded query sample.  The
    index is the one the reference's own build_global writes for the same
    data (its k-means, rebalancing, PQ training and encoding; the CAGRA graph
    over centroids is not built, cuVS being absent), the ground truth an
    exact float64 k-NN in torch; nothing of this repository's library runs.
    Recall is over all 10,000 queries, like the GPU arm's."""
    import torch
    import oracle
    from fusiongpu_b200 import datasets as ds
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    spec, nlist = workload(args.quick)
    t0 = time.time()
    base, queries = ds.generate(spec)
    index, build_s = reference_build(base, nlist, CONFIG["pq_m"])
    if index is None:
        print(json.dumps({"impl": "reference", "unavailable": build_s}), flush=True)
        return
    gt = exact_gt(base, queries, 10, device)
    setup_s = time.time() - t0
    cores = os.cpu_count() or 1
    sample = 128
    nq = queries.shape[0]
    pts, sweep = [], []
    for nprobe in SWEEP:
        kw = dict(top_m=nprobe, p1_lists=CONFIG["p1_lists"], limit_k=CONFIG["limit_k"],
                  threshold_coeff=CONFIG["threshold_coeff"], prune_ratio=100.0, rerank_m=CONFIG["rerank_m"],
                  final_k=CONFIG["k"], mini_batch=CONFIG["mini_batch"], epsilon=CONFIG["epsilon"],
                  beta=CONFIG["beta"], ref_compat=False)
        ids, _ = oracle.search(index, base, queries, nthreads=cores, **kw)
        rec = recall10(ids, gt)
        for s in range(args.warmup):
            oracle.search(index, base, np.ascontiguousarray(queries[:sample]), nthreads=cores, **kw)
        tot = 0.0
        for s in range(args.steps):
            lo = (s * sample) % (nq - sample)
            qs = np.ascontiguousarray(queries[lo:lo + sample])
            t1 = time.perf_counter()
            oracle.search(index, base, qs, nthreads=cores, **kw)
            tot += time.perf_counter() - t1
        ms = tot / args.steps * 1e3
        sweep.append(dict(nprobe=nprobe, recall=rec, ms_per_step=ms, qps=sample / (ms / 1e3)))
        pts.append((nprobe, rec, sample / (ms / 1e3)))
    value, met = interp_at_recall(pts)
    op = next((s for s in sweep if s["recall"] >= RECALL_TARGET), max(sweep, key=lambda s: s["recall"]))
    out = {
        "impl": "reference",
        "metric": "QPS at recall@10=0.95 (C2 1M x 128 IVF-PQ)",
        "value": value,
        "unit": "queries/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": op["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture standing in for a dataset)",
        "config": dict(CONFIG, recall_target_met=met, operating_nprobe=op["nprobe"], quick=bool(args.quick),
                       parallelism="host CPU (OpenMP)", lists=int(index["centroids"].shape[0]),
                       index="written by the reference's build_global (oracle/_ref), CAGRA step not built",
                       recall_on=f"all {nq} queries (exact float64 ground truth)"),
        "sweep": sweep,
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": cores, "kind": "port",
                         "sample": f"{sample} queries per step; the reference ships no CPU search, so its C "
                                   "restatement (oracle/) runs on the reference-built index"},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_build_s": build_s,
        "setup_s": setup_s,
    }
    print(json.dumps(out), flush=True)


# ---- C3: 10M x 96 IVF-PQ, codes far beyond L2 ----------------------------------------

C3_CONFIG = dict(nlist=16384, pq_m=48, k=10, rerank_m=4096, nprobe=64, p1_lists=12, limit_k=50, threshold_coeff=1.0,
                 mini_batch=128, epsilon=0.1, beta=2, batches=[1, 100, 10000])


def main_c3(args):
    """C3: QPS and recall@10 at nprobe 64 with an exact rerank of the top 4096
    (intended mode) over 10M x 96 unit vectors; latency at batches of 1 and
    100.  The scan reads 480 MB of codes per pass (far beyond L2): its
    roofline is HBM."""
    import torch
    from fusiongpu_b200 import datasets as ds
    from fusiongpu_b200.index import IVFPQIndex, SearchParams, knn_exact, recall_at, run_gpu_batch_logic
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = dict(C3_CONFIG)
    # quick: 3M vectors, so that the 144 MB of codes still exceed the 126 MB L2
    spec = ds.scaled(ds.C3, 3_000_000, 2_000, n_centres=4096) if args.quick else ds.C3
    if args.quick:
        cfg["nlist"] = 4096
    t0 = time.time()
    base, queries = ds.generate(spec)
    print(f"[c3] generated {spec.n_base} x {spec.dim} in {time.time() - t0:.1f} s", file=sys.stderr, flush=True)
    t0 = time.time()
    xb = torch.from_numpy(base).to(device)
    idx = IVFPQIndex.build(xb, cfg["nlist"], cfg["pq_m"], kmeans_iters=20, pq_sample=50000, pq_iters=8, device=device)
    torch.cuda.synchronize(device)
    t_build = time.time() - t0
    print(f"[c3] index built in {t_build:.1f} s ({idx.nlist} lists)", file=sys.stderr, flush=True)
    qd = torch.from_numpy(queries).to(device)
    p = SearchParams(top_m=cfg["nprobe"], p1_lists=cfg["p1_lists"], limit_k=cfg["limit_k"],
                     threshold_coeff=cfg["threshold_coeff"], prune_ratio=100.0, rerank_m=cfg["rerank_m"],
                     final_k=cfg["k"], mini_batch=cfg["mini_batch"], epsilon=cfg["epsilon"], beta=cfg["beta"],
                     ref_compat=False)
    if args.profile in ("scan", "search", "rerank", "coarse"):
        # warmup+1 launches of one stage alone (the target of ncu -s <warmup> -c 1)
        pid, pdist = idx.coarse(qd, cfg["nprobe"])
        ti, td, tc, cc = run_gpu_batch_logic(idx, qd, pid, pdist, p)
        torch.cuda.synchronize(device)
        from fusiongpu_b200.index import run_gpu_rerank
        torch.cuda.profiler.start()  # ncu --profile-from-start off: skip the build's launches
        for _ in range(args.warmup + 1):
            if args.profile == "scan":
                run_gpu_batch_logic(idx, qd, pid, pdist, p)
            elif args.profile == "rerank":
                run_gpu_rerank(qd, ti, tc, idx.base, p, device)
            elif args.profile == "coarse":
                idx.coarse(qd, cfg["nprobe"])
            else:
                idx.search(qd, p)
        torch.cuda.synchronize(device)
        print(json.dumps({"profile": args.profile, "workload": spec.name, "nq": int(queries.shape[0])}))
        return
    gt, _ = knn_exact(xb, qd, 10, device=device)
    gt = gt.cpu().numpy()
    nq = queries.shape[0]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    ids = torch.empty((nq, cfg["k"]), dtype=torch.int32, device=device)
    dd = torch.empty((nq, cfg["k"]), dtype=torch.float32, device=device)

    def timed(fn, steps):
        tot = 0.0
        for _ in range(steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / steps

    clocks = ClockSampler(local)
    with clocks:
        for _ in range(args.warmup):
            idx.search(qd, p, out=(ids, dd))
        torch.cuda.synchronize(device)
        rec = recall_at(ids.cpu().numpy(), gt, 10)
        ms = timed(lambda: idx.search(qd, p, out=(ids, dd)), args.steps)
        lat, lat_graph = {}, {}
        for b in cfg["batches"]:
            b = min(b, nq)
            qb = qd[:b].contiguous()
            if b < nq:
                for _ in range(args.warmup):
                    idx.search(qb, p)
                lat[str(b)] = timed(lambda: idx.search(qb, p), args.steps)
            else:
                lat[str(b)] = ms
            g = idx.capture(b, p)  # the same search as one CUDA graph replay
            g.queries.copy_(qb)
            for _ in range(args.warmup):
                g.replay()
            lat_graph[str(b)] = timed(g.replay, args.steps)
            del g
        # roofline of the scan kernel alone
        pid, pdist = idx.coarse(qd, cfg["nprobe"])
        lens = (idx.offsets[1:] - idx.offsets[:-1]).to(torch.int64)
        code_bytes = int(lens[pid.long()].sum().item()) * idx.pq_m
        for _ in range(args.warmup):
            run_gpu_batch_logic(idx, qd, pid, pdist, p)
        scan_ms = timed(lambda: run_gpu_batch_logic(idx, qd, pid, pdist, p), args.steps)
        ti, td, tc, cc = run_gpu_batch_logic(idx, qd, pid, pdist, p)
        cand_bytes = 4 * int(cc.to(torch.int64).sum().item())
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    alg = code_bytes + cand_bytes
    achieved = alg / (scan_ms / 1e3) / 1e9
    # end to end: pinned host queries in, ids and distances out
    hq = torch.from_numpy(queries).pin_memory()
    hid = torch.empty((nq, cfg["k"]), dtype=torch.int32).pin_memory()
    hdd = torch.empty((nq, cfg["k"]), dtype=torch.float32).pin_memory()

    def one():
        # the public host-buffer call, replayed as one CUDA graph per step
        idx.search_host(hq, p, out=(hid, hdd), chunks=2, graph=True)

    one()
    e2e_ms = timed(one, args.steps)
    # parity on a query sample: the GPU search against the oracle, both modes
    parity = None
    if not args.no_cpu:
        import oracle
        sample = min(nq, 300)
        index_np = idx.to_numpy()
        parity = {"queries": sample, "index": "the GPU arm's index", "modes": {}}
        qs = np.ascontiguousarray(queries[:sample])
        for mode, rcm in (("intended", False), ("ref_compat", True)):
            pm = p.replace(ref_compat=rcm)
            t0 = time.perf_counter()
            oi, od = oracle.search(index_np, base, qs, nthreads=os.cpu_count() or 1, **oracle_kw(pm))
            dt = time.perf_counter() - t0
            gi, gd = idx.search(qd[:sample].contiguous(), pm)
            gi, gd = gi.cpu().numpy(), gd.cpu().numpy()
            mism, rel = compare_results(gi, gd, oi, od)
            parity["modes"][mode] = {"id_mismatches_beyond_1e-5_ties": mism, "max_rel_dist_err": rel,
                                     "bit_exact": bool(np.array_equal(gi, oi) and np.array_equal(gd, od)),
                                     "recall_gpu": recall_at(gi, gt[:sample], 10),
                                     "recall_oracle": recall_at(oi, gt[:sample], 10), "oracle_s": dt}
    out = {
        "metric": "QPS of the C3 IVF-PQ search (nprobe 64, exact rerank of the top 4096) with its recall@10",
        "value": nq / (ms / 1e3),
        "unit": "queries/s",
        "recall@10": rec,
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture: 16384 normalised centres, sigma 0.05, unit vectors)",
        "config": dict(cfg, workload=f"{spec.name}: {spec.n_base} x {spec.dim} fp32, {nq} queries, L2",
                       lists=idx.nlist, l2="flushed (256 MB write) between timed steps", quick=bool(args.quick),
                       mode="intended (full rerank_m gather)"),
        "latency_ms_by_batch": lat,
        "latency_ms_by_batch_cuda_graph": lat_graph,
        "e2e": {"value": nq / (e2e_ms / 1e3), "unit": "queries/s", "h2d_bytes_per_step": int(queries.nbytes),
                "d2h_bytes_per_step": int(nq * cfg["k"] * 8)},
        # per search: coarse stage 6, split scan 5 (pairs, two phases, select, fallback),
        # rerank 1; the timed step, batch latencies (3 batch sizes, eager and graph),
        # scan-only, e2e (2 pieces)
        "gpu_launches": 12 * args.steps * (1 + 6 + 2) + 5 * args.steps,
        "roofline": {"kernel": "scan (" + os.environ.get("FG_SCAN_KERNEL", "auto") + ")", "bound": "hbm",
                     "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": "measured" if "hbm_gbs" in peaks else "fallback", "traffic": None,
                     "algorithmic_bytes": alg, "ms_per_launch": scan_ms},
        "clocks": clocks.summary(),
        "build_s": t_build,
        "parity": parity,
    }
    print(json.dumps(out), flush=True)


# ---- C5: 100M x 128 uint8, inverted lists sharded across the GPUs ---------------

C5_CONFIG = dict(nlist=65536, pq_m=32, k=10, rerank_m=256, nprobe=64, p1_lists=12, limit_k=50, threshold_coeff=1.0,
                 mini_batch=128, epsilon=0.1, beta=2, kmeans_sample=2_000_000, kmeans_iters=20, gt_queries=1000)


def main_c5(args):
    """C5: QPS and recall@10 at nprobe 64 with an exact rerank of the top 256
    per shard, 10,000 queries broadcast to every GPU; the inverted lists (with
    their codes, ids and uint8 raw vectors) are dealt to the GPUs by list
    length.  Every rank builds the same deterministic index, keeps its shard,
    searches it, and the per-GPU top-k lists meet in one NCCL all-gather and
    the device merge (strong scaling).  k-means trains on 2M strided rows,
    then every row is assigned."""
    import torch
    import torch.distributed as dist
    from fusiongpu_b200 import datasets as ds
    from fusiongpu_b200.index import IVFPQIndex, SearchParams, knn_exact, recall_at
    from fusiongpu_b200.sharded import ShardedIndex
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=1800), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg = dict(C5_CONFIG)
    spec = ds.scaled(ds.C5, 10_000_000, 10_000, n_centres=8192) if args.quick else ds.C5
    if args.quick:
        cfg.update(nlist=8192, kmeans_sample=400_000)
    t0 = time.time()
    base, queries = ds.generate(spec)
    queries = queries.astype(np.float32)
    print(f"[c5] generated {spec.n_base} x {spec.dim} uint8 in {time.time() - t0:.1f} s", file=sys.stderr, flush=True)
    t0 = time.time()
    idx = IVFPQIndex.build(torch.from_numpy(base).to(device), cfg["nlist"], cfg["pq_m"],
                           kmeans_iters=cfg["kmeans_iters"], kmeans_sample=cfg["kmeans_sample"], device=device)
    torch.cuda.synchronize(device)
    t_build = max_over_ranks(time.time() - t0)
    print(f"[c5] index built in {t_build:.1f} s ({idx.nlist} lists)", file=sys.stderr, flush=True)
    p = SearchParams(top_m=cfg["nprobe"], p1_lists=cfg["p1_lists"], limit_k=cfg["limit_k"],
                     threshold_coeff=cfg["threshold_coeff"], prune_ratio=100.0, rerank_m=cfg["rerank_m"],
                     final_k=cfg["k"], mini_batch=cfg["mini_batch"], epsilon=cfg["epsilon"], beta=cfg["beta"],
                     ref_compat=False)
    qd = torch.from_numpy(queries).to(device)
    if args.profile in ("scan", "coarse", "rerank", "search") and world == 1:
        # warmup+1 launches of one stage alone (the target of ncu -s <warmup> -c 1)
        from fusiongpu_b200.index import run_gpu_batch_logic, run_gpu_rerank
        pid, pdist = idx.coarse(qd, cfg["nprobe"])
        ti, td, tc, cc = run_gpu_batch_logic(idx, qd, pid, pdist, p)
        torch.cuda.synchronize(device)
        torch.cuda.profiler.start()  # ncu --profile-from-start off: skip the build's launches
        for _ in range(args.warmup + 1):
            if args.profile == "scan":
                run_gpu_batch_logic(idx, qd, pid, pdist, p)
            elif args.profile == "coarse":
                idx.coarse(qd, cfg["nprobe"])
            elif args.profile == "rerank":
                run_gpu_rerank(qd, ti, tc, idx.base, p, device)
            else:
                idx.search(qd, p)
        torch.cuda.synchronize(device)
        print(json.dumps({"profile": args.profile, "workload": spec.name, "nq": int(queries.shape[0])}))
        return
    gt = None
    if rank == 0:
        ng = cfg["gt_queries"]
        gt, _ = knn_exact(idx.base, qd[:ng], 10, device=device)
        gt = gt.cpu().numpy()
    if world == 1:
        searcher = idx
    else:
        host = idx.to_numpy()
        del idx
        torch.cuda.empty_cache()
        searcher = ShardedIndex(host, base, rank, world, device=device)
    nq = queries.shape[0]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    clocks = ClockSampler(local)
    with clocks:
        for _ in range(args.warmup):
            ids, dd = searcher.search(qd, p)
        torch.cuda.synchronize(device)
        rec = recall_at(ids[:cfg["gt_queries"]].cpu().numpy(), gt, 10) if rank == 0 else None
        barrier()
        tot = 0.0
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            searcher.search(qd, p)
            e1.record(stream)
            e1.synchronize()
            tot += e0.elapsed_time(e1)
        barrier()
        ms = max_over_ranks(tot / args.steps)
    # one GPU: the oracle on a query sample of the same index (parity), and
    # recall against rerank depth (what bounds recall at this nprobe)
    parity, depth = None, None
    if world == 1 and rank == 0 and not args.no_cpu:
        parity, depth = c5_parity(idx, queries, qd, gt, p, cfg, args)
    # end to end: pinned host queries in, ids and distances out to pinned host
    # memory (one GPU: the public search_host call replayed as one CUDA graph;
    # N GPUs: upload, sharded search with its all-gather, download)
    hq = torch.from_numpy(queries).pin_memory()
    hid = torch.empty((nq, cfg["k"]), dtype=torch.int32).pin_memory()
    hdd = torch.empty((nq, cfg["k"]), dtype=torch.float32).pin_memory()
    qdev = torch.empty_like(qd)

    def one():
        if world == 1:
            searcher.search_host(hq, p, out=(hid, hdd), chunks=2, graph=True)
        else:
            qdev.copy_(hq, non_blocking=True)
            r_ids, r_d = searcher.search(qdev, p)
            hid.copy_(r_ids, non_blocking=True)
            hdd.copy_(r_d, non_blocking=True)

    barrier()
    tot = 0.0
    for i in range(1 + args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        one()
        e1.record(stream)
        e1.synchronize()
        if i:
            tot += e0.elapsed_time(e1)
    e2e = nq / (max_over_ranks(tot / args.steps) / 1e3)
    out = {
        "metric": "QPS of the C5 sharded IVF-PQ search (nprobe 64, rerank 256 per shard) with its recall@10",
        "value": nq / (ms / 1e3),
        "unit": "queries/s",
        "recall@10": rec,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32 (uint8 raw vectors)",
        "data": "synthetic (seeded Gaussian mixture: 65536 centres in [0,255], sigma 8, clamped, rounded, uint8)",
        "config": dict(cfg, workload=f"{spec.name}: {spec.n_base} x {spec.dim} uint8, {nq} queries, L2",
                       lists=int(host["centroids"].shape[0]) if world > 1 else idx.nlist,
                       parallelism=f"inverted lists dealt to {world} GPUs by length (NCCL all-gather, "
                                   "device merge)" if world > 1 else "one GPU",
                       recall_on=f"first {cfg['gt_queries']} queries (exact ground truth)",
                       l2="flushed (256 MB write) between timed steps", quick=bool(args.quick)),
        "e2e": {"value": e2e, "unit": "queries/s", "h2d_bytes_per_step": int(queries.nbytes),
                "d2h_bytes_per_step": int(nq * cfg["k"] * 8)},
        # per search: coarse stage 6, split scan 5 (pairs, two phases, select, fallback), rerank 1
        # (+ pack and merge on N GPUs); device and e2e
        "gpu_launches": (12 + (2 if world > 1 else 0)) * args.steps * 2,
        "clocks": clocks.summary(),
        "build_s": t_build,
        "parity": parity,
        "recall_by_knob": depth,
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


def c5_parity(idx, queries, qd, gt, p, cfg, args):
    """The GPU search of the first `sample` queries against the oracle on the
    same index: the oracle's candidate generation, then its rerank over a
    float copy of just the candidate rows (the oracle takes float vectors;
    ids are renumbered in increasing order, so every comparison and tie
    keeps its order) -- plus recall@10 at deeper reranks."""
    import torch
    import oracle
    from fusiongpu_b200.index import recall_at, run_gpu_batch_logic
    sample = 300
    qs = np.ascontiguousarray(queries[:sample])
    pid, pdist = idx.coarse(qd[:sample].contiguous(), p.top_m)
    eids, ed = oracle.coarse(idx.centroids.cpu().numpy(), qs, p.top_m)
    coarse_equal = bool(np.array_equal(pid.cpu().numpy().view(np.uint32), eids) and
                        np.array_equal(pdist.cpu().numpy(), ed))
    index_np = idx.to_numpy()
    kw = oracle_kw(p)
    t0 = time.perf_counter()
    oi, od, oc, st = oracle.batch_logic(index_np, qs, eids, ed, nthreads=os.cpu_count() or 1, **kw)
    rows = np.unique(oi[oi >= 0])
    sub = idx.base[torch.from_numpy(rows).to(idx.device).long()].float().cpu().numpy()
    remap = np.searchsorted(rows, np.where(oi >= 0, oi, 0)).astype(np.int32)
    ri, rd = oracle.rerank(qs, np.where(oi >= 0, remap, oi).astype(np.int32), oc, sub, **kw)
    ri = np.where(ri >= 0, rows[np.clip(ri, 0, rows.size - 1)], ri).astype(np.int32)
    dt = time.perf_counter() - t0
    gi, gd = idx.search(qd[:sample].contiguous(), p)
    gi, gd = gi.cpu().numpy(), gd.cpu().numpy()
    mism, rel = compare_results(gi, gd, ri, rd)
    parity = {"queries": sample, "coarse_equal": coarse_equal, "id_mismatches_beyond_1e-5_ties": mism,
              "max_rel_dist_err": rel, "bit_exact": bool(np.array_equal(gi, ri) and np.array_equal(gd, rd)),
              "recall_gpu": recall_at(gi, gt[:sample], 10), "recall_oracle": recall_at(ri, gt[:sample], 10),
              "oracle_s": dt, "mode": "intended"}
    # recall@10 on the ground-truth queries as the candidate-generation knobs
    # move: the rerank depth, the phase-1 per-list cap (limit_k) and the
    # phase-2 threshold coefficient
    depth = {}
    ng = gt.shape[0]
    for name, q in (("config", {}), ("rerank_m=1024", dict(rerank_m=1024)), ("rerank_m=4096", dict(rerank_m=4096)),
                    ("limit_k=200", dict(limit_k=200)), ("limit_k=200,rerank_m=1024", dict(limit_k=200, rerank_m=1024)),
                    ("threshold_coeff=1.5", dict(threshold_coeff=1.5)), ("p1_lists=64", dict(p1_lists=64)),
                    ("nprobe=128", dict(top_m=128))):
        ids, _ = idx.search(qd[:ng].contiguous(), p.replace(**q))
        depth[name] = recall_at(ids.cpu().numpy(), gt, 10)
    return parity, depth


# ---- C4: graph index ------------------------------------------------------------

# the IVF partition doubles as the entry index of the search: finer than the
# mixture's 2000 clusters, so that a list's medoid lies in the list's own cluster
C4_BUILD = dict(graph_degree=64, intermediate_degree=128, nlist=4096, probe_lists=8, kmeans_iters=10, seed=42,
                metric="ip")
C4_SEARCH = dict(itopk=128, search_width=4, max_iterations=0, k=10, seed=7, metric="ip", entry_probes=16)
C4_SWEEP = (32, 64, 128, 256)


def main_c4(args):
    """C4: QPS and recall@10 of the graph search (batch of 10,000 fp16
    queries, itopk 128, search width 4) on a degree-64 graph over 1M x 768
    fp16 unit vectors (inner product); itopk swept for the recall curve.  A
    step is one search of the whole batch.  Under torchrun the rows are
    partitioned across the GPUs (one graph per GPU, queries broadcast, one
    NCCL all-gather and a device merge per step; strong scaling)."""
    import torch
    import torch.distributed as dist
    from fusiongpu_b200 import datasets as ds
    from fusiongpu_b200.graph import GraphBuildParams, GraphIndex, GraphSearchParams, knn_ip
    from fusiongpu_b200.sharded import ShardedGraphIndex
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    spec = ds.scaled(ds.C4, 100_000, 2_000, n_centres=200) if args.quick else ds.C4
    t0 = time.time()
    base, queries = ds.generate(spec)
    t_gen = time.time() - t0
    print(f"[c4] generated {spec.n_base} x {spec.dim} in {t_gen:.1f} s", file=sys.stderr, flush=True)
    bp = dict(C4_BUILD, nlist=512 if args.quick else C4_BUILD["nlist"])
    # every shard keeps the full entry partition: its lists must stay finer than
    # the mixture's clusters, whose members every shard holds a share of
    torch.cuda.synchronize(device)
    t0 = time.time()
    if world == 1:
        xb = torch.from_numpy(base).to(device)
        gi = GraphIndex.build(xb, GraphBuildParams(**bp))
        searcher = gi
    else:
        xb = None
        gi = ShardedGraphIndex(base, rank, world, GraphBuildParams(**bp), device=device)
        searcher = gi
    torch.cuda.synchronize(device)
    t_build = max_over_ranks(time.time() - t0)
    print(f"[c4] graph built in {t_build:.1f} s", file=sys.stderr, flush=True)
    qd = torch.from_numpy(queries).to(device)
    if args.profile == "graph":
        # warmup+1 launches of the search alone: the target of
        # `ncu -k regex:graph_search -s <warmup> -c 1`
        sp = GraphSearchParams(**C4_SEARCH)
        torch.cuda.profiler.start()  # ncu --profile-from-start off: skip the build's launches
        for _ in range(args.warmup + 1):
            searcher.search(qd, sp)
        torch.cuda.synchronize(device)
        print(json.dumps({"profile": "graph", "nq": int(queries.shape[0]), "itopk": sp.itopk}))
        return
    gt = None
    if rank == 0:
        full = xb if xb is not None else torch.from_numpy(base).to(device)
        g, _ = knn_ip(full, qd, 10)
        gt = g.cpu().numpy()
        del full
    nq = queries.shape[0]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    local_graph = gi if world == 1 else gi.local
    sweep = []
    clocks = ClockSampler(local)
    with clocks:
        for itopk in C4_SWEEP:
            print(f"[c4] itopk {itopk}", file=sys.stderr, flush=True)
            sp = GraphSearchParams(**dict(C4_SEARCH, itopk=itopk))
            for _ in range(args.warmup):
                ids, dd = searcher.search(qd, sp)
            # device counters of this GPU's graph (a separate, untimed pass)
            _, _, cnt = local_graph.search(qd, sp, counters=True)
            torch.cuda.synchronize(device)
            evals, expanded, bad = (int(v) for v in cnt.cpu().numpy())
            if bad:
                raise RuntimeError(f"graph search skipped {bad} out-of-range accesses")
            rec = None
            if rank == 0:
                got = ids.cpu().numpy()
                rec = float(np.mean([len(set(got[i]) & set(gt[i])) / 10 for i in range(nq)]))
            barrier()
            torch.cuda.synchronize(device)
            tot = 0.0
            for _ in range(args.steps):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                searcher.search(qd, sp)
                e1.record(stream)
                e1.synchronize()
                tot += e0.elapsed_time(e1)
            barrier()
            ms = max_over_ranks(tot / args.steps)
            alg = evals * spec.dim * 2 + expanded * bp["graph_degree"] * 4
            sweep.append(dict(itopk=itopk, recall=rec, ms_per_step=ms, qps=nq / (ms / 1e3),
                              distance_evals_per_query=evals / nq, expanded_per_query=expanded / nq,
                              algorithmic_bytes_per_gpu=alg, achieved_gbs_per_gpu=alg / (ms / 1e3) / 1e9))
    op = next(s_ for s_ in sweep if s_["itopk"] == C4_SEARCH["itopk"])
    # end to end: pinned fp16 queries in, ids out
    sp = GraphSearchParams(**C4_SEARCH)
    hq = torch.from_numpy(queries).pin_memory()
    hid = torch.empty((nq, sp.k), dtype=torch.int32).pin_memory()
    qdev = torch.empty_like(qd)
    barrier()
    tot = 0.0
    for i in range(args.warmup + args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        qdev.copy_(hq, non_blocking=True)
        ids, _ = searcher.search(qdev, sp)
        hid.copy_(ids, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        if i >= args.warmup:
            tot += e0.elapsed_time(e1)
    e2e = nq / (max_over_ranks(tot / args.steps) / 1e3)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    out = {
        "metric": "QPS of the C4 graph search (itopk 128, search width 4) with its recall@10",
        "value": op["qps"],
        "unit": "queries/s",
        "recall@10": op["recall"],
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": op["ms_per_step"],
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded Gaussian mixture: 2000 N(0,I) centres, sigma 0.3, normalised, fp16)",
        "config": dict(workload=f"{spec.name}: {spec.n_base} x {spec.dim} fp16, {nq} queries, inner product",
                       build=bp, search=C4_SEARCH, itopk_sweep=list(C4_SWEEP),
                       parallelism=f"rows partitioned across {world} GPUs (graph per GPU, NCCL all-gather, "
                                   "device merge)" if world > 1 else "one GPU",
                       l2="flushed (256 MB write) between timed steps", quick=bool(args.quick)),
        "sweep": sweep,
        "e2e": {"value": e2e, "unit": "queries/s", "h2d_bytes_per_step": int(queries.nbytes),
                "d2h_bytes_per_step": int(nq * sp.k * 4)},
        "gpu_launches": args.steps * len(sweep),
        "roofline": {"kernel": "graph_search_kernel (+ entry selection)", "bound": "hbm",
                     "achieved": op["achieved_gbs_per_gpu"], "peak": peak, "unit": "GB/s",
                     "frac": op["achieved_gbs_per_gpu"] / peak,
                     "peak_source": "measured" if "hbm_gbs" in peaks else "fallback", "traffic": None,
                     "algorithmic_bytes": op["algorithmic_bytes_per_gpu"],
                     "bytes_rule": "distance evals x dim x 2 + expanded nodes x degree x 4 (device counters), "
                                   "per GPU, over the whole step"},
        "clocks": clocks.summary(),
        "build_s": t_build,
        "generate_s": t_gen,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        sample = 200 if not args.quick else 100
        g = gi.graph.cpu().numpy()
        qs = np.ascontiguousarray(queries[:sample])
        cores = os.cpu_count() or 1
        t0 = time.perf_counter()
        oracle.graph_search(base, g, qs, nthreads=cores, entry_centroids=gi.entry_centroids.cpu().numpy(),
                            entry_nodes=gi.entry_nodes.cpu().numpy(), **C4_SEARCH)
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": sample / dt, "unit": "queries/s", "cores": cores, "kind": "port",
                               "sample": f"first {sample} queries, same graph and parameters (oracle restatement)",
                               "seconds": dt}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
