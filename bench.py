#!/usr/bin/env python3
"""Benchmark of the exact learned-sparse scoring path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2]
                    [--impl ours|reference|cusparse|spare]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1: doc-range shards)

A step scores one batch of queries against the whole corpus and returns the exact top-k
(k = 1000) per query.  The corpus is a BASELINE config (default 2: 8.8M documents,
batch 1000) generated on each GPU from the seeded synthetic SPLADE-shaped law; with N
GPUs every rank builds the index of its own contiguous doc range, the ranks share a lower
bound of each query's k-th best key while they score (IPC-mapped boards), and the
per-shard top-k lists are exchanged by query blocks (one NCCL all-to-all), merged (each
rank its B/N queries) and all-gathered.  Work per step is fixed as N grows (strong
scaling).

Reported:
* value / ms_per_step / p50: device time (CUDA events, max over ranks) of K steps with
  queries and index resident in HBM (index >> L2, so no flush is needed between steps);
* e2e: the same steps through the public API with the query batch copied from pinned host
  memory and the top-k copied back every step;
* roofline: the scoring kernel's own launches timed with CUDA events on its stream;
  achieved = algorithmic bytes per launch / mean launch time, against the measured HBM
  copy bandwidth (MEASURED_PEAKS.json);
* cpu_baseline (rank 0, N = 1): the CPU oracle (a C restatement of the reference's
  scatter-add + top-k) on a bounded sample of the same workload, all host threads.

--impl reference times the reference's CPU path for this workload (the same C oracle
port, since the reference itself is Python/Triton and only its CPU restatement runs on
the GPU box): rank 0 only, the others exit immediately.

--impl cusparse is a context line only (one GPU, rank 0): the library route on the same
B200 -- cuSPARSE SpMM (torch.sparse.mm of the corpus CSR, in 2M-document chunks, with the
dense [V, B] query matrix) followed by torch.topk with a running top-k.  --impl spare is
another context line: the SPARe-style loop of the reference's baselines
(baselines/bench_spare_iterative.py:58-77) -- per query, one torch index_add_ per term into
a dense accumulator, then torch.topk -- on a bounded sample of the batch.
"""
from __future__ import annotations

import argparse
import json
import os
import resource
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "gpu-sparse_b200")]

METRIC = ("queries/sec & batch p50 latency at k=1000; scorer HBM GB/s vs peak "
          "(1/2/4/8 B200)")
V = 30522
CONFIGS = {
    0: dict(num_docs=100_000, batch=500, zipf_s=1.1, wdtype="fp32"),
    1: dict(num_docs=1_000_000, batch=1000, zipf_s=1.1, wdtype="fp32"),
    2: dict(num_docs=8_800_000, batch=1000, zipf_s=1.1, wdtype="fp32"),
    3: dict(num_docs=8_800_000, batch=1000, zipf_s=1.1, wdtype="u8"),
    4: dict(num_docs=50_000_000, batch=4096, zipf_s=1.2, wdtype="fp32"),
}
WBYTES = {"fp32": 4, "bf16": 2, "u8": 1}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "cusparse", "spare"], default="ours")
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--num-docs", type=int, default=None)
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--k", type=int, default=1000)
    ap.add_argument("--wdtype", choices=["fp32", "bf16", "u8"], default=None)
    ap.add_argument("--head-mode", choices=["auto", "cuda", "tc"], default="auto",
                    help="head terms: the library's choice, the CUDA cores (canonical order) or "
                         "the tensor cores (tcgen05, 3xTF32)")
    ap.add_argument("--phase-split", action="store_true",
                    help="also time each step's phases (score, exchange, merge, gather) with "
                         "CUDA events, max over ranks")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="target CPU work of the bounded CPU-baseline sample")
    return ap.parse_args()


def workload(args):
    c = dict(CONFIGS[args.config])
    if args.num_docs:
        c["num_docs"] = args.num_docs
    if args.batch:
        c["batch"] = args.batch
    if args.wdtype:
        c["wdtype"] = args.wdtype
    c["k"] = min(args.k, c["num_docs"])
    c["name"] = (f"config{args.config}: {c['num_docs']:,} docs, batch {c['batch']}, "
                 f"k={c['k']}, V={V}, zipf {c['zipf_s']}, {c['wdtype']} weights")
    return c


SCORER_SOURCES = ("common.cuh", "score.cu", "score_tc.cuh", "select.cu")


def source_tag():
    """Short hash of the sources the scoring launch is compiled from (csrc/common.cuh,
    score.cu, score_tc.cuh, select.cu): ties a committed ncu figure to the kernels it was
    measured on."""
    import hashlib
    d = os.path.join(ROOT, "gpu-sparse_b200", "csrc")
    h = hashlib.sha256()
    for f in SCORER_SOURCES:
        h.update(f.encode())
        h.update(open(os.path.join(d, f), "rb").read())
    return h.hexdigest()[:12]


def measured_traffic(config, world, num_docs_override):
    """DRAM bytes per scoring launch from the committed ncu summary
    (profiles/score_kernel_traffic_config<c>.md), used only when its source tag matches the
    sources being benchmarked; otherwise None and the reason."""
    import re
    tp = os.path.join(ROOT, "profiles", f"score_kernel_traffic_config{config}.md")
    if num_docs_override:
        return None, "no committed profile for a --num-docs override"
    if not os.path.exists(tp):
        return None, f"no committed profile for config {config}"
    txt = open(tp).read()
    m = re.search(rf"config{config}_gpus{world} dram_bytes_per_launch: (\d+) source: (\w+)", txt)
    if not m:
        return None, f"the committed profile has no figure for config {config} on {world} GPU(s)"
    if m.group(2) != source_tag():
        return None, f"the committed profile measured sources {m.group(2)}, these are {source_tag()}"
    return int(m.group(1)), f"ncu, sources {m.group(2)} ({os.path.relpath(tp, ROOT)})"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        j = json.load(open(p))
        return float(j["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return 6650.0, "fallback 6.65 TB/s"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self, gpus):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], [], set()
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        idxs = ([int(x) for x in vis.split(",") if x.strip().isdigit()] if vis else
                list(range(gpus)))[:gpus]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or not f[0].isdigit() or int(f[0]) not in idxs:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.f.name)
        if not sm:
            return None
        load = [x for x in sm if x > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def bytes_alg(index, qi, B, k, wdtype):
    """Algorithmic bytes of one scoring launch: the postings of the batch's unique terms
    (doc id + weight), one fp32 accumulator write + read per (query, document), and the
    top-k output."""
    import torch
    t = qi[(qi >= 0) & (qi < index.vocab_size)].long().unique()
    post = int(index.lengths[t].long().sum().item())
    b = post * (4 + WBYTES[wdtype]) + 2 * 4 * B * int(index.num_docs) + 8 * B * k
    if wdtype == "u8":
        b += 4 * int(t.numel())
    return b, post


def contributions(index, qi):
    """On-chip work of one scoring launch: one multiply-add per (query term, posting)."""
    import torch
    ok = (qi >= 0) & (qi < index.vocab_size)
    t = torch.where(ok, qi, torch.zeros_like(qi)).long()
    return int((index.lengths[t].long() * ok.long()).sum().item())


def cpu_sample(index, qi, qs, k, gpu_s, gpu_i, target_s):
    """The CPU oracle on a bounded sample of queries of the same workload (all host
    threads), plus a bit-exact parity check of those queries against the GPU result."""
    import numpy as np
    import torch
    from oracle import oracle as O
    import gpusparse
    nt = O.nthreads_default()
    oidx = O.Index(index.doc_ids.cpu().numpy(), None, index.offsets.cpu().numpy(),
                   index.lengths.cpu().numpy(), index.padded_lengths.cpu().numpy(), None,
                   int(index.num_docs), int(index.vocab_size))
    w = gpusparse.dequantized_weights(index).cpu().numpy()
    qi_h, qs_h = qi.cpu().numpy(), qs.cpu().numpy()
    head = index.head_ids.cpu().numpy()
    B = qi_h.shape[0]
    # calibrate on one query per thread, then size the timed sample to ~target_s
    nq = min(B, nt)
    t0 = time.perf_counter()
    O.score_topk(oidx, qi_h[:nq], qs_h[:nq], k, weights=w, nthreads=nt, head=head)
    dt = time.perf_counter() - t0
    reps = max(1, int(target_s / max(dt, 1e-3)))
    nq = min(B, nq * reps)
    r0 = resource.getrusage(resource.RUSAGE_SELF)
    t0 = time.perf_counter()
    s, i = O.score_topk(oidx, qi_h[:nq], qs_h[:nq], k, weights=w, nthreads=nt, head=head)
    wall = time.perf_counter() - t0
    r1 = resource.getrusage(resource.RUSAGE_SELF)
    cpu = (r1.ru_utime - r0.ru_utime) + (r1.ru_stime - r0.ru_stime)
    exact = bool(np.array_equal(s, gpu_s[:nq]) and np.array_equal(i, gpu_i[:nq]))
    # one core, on a smaller sample (a few seconds)
    n1 = max(1, min(nq, int(nq * max(target_s / 3.0, 1.0) / max(wall * nt, 1e-3))))
    t0 = time.perf_counter()
    O.score_topk(oidx, qi_h[:n1], qs_h[:n1], k, weights=w, nthreads=1, head=head)
    wall1 = time.perf_counter() - t0
    return {"value": nq / wall, "unit": "queries/s", "cores": nt, "kind": "port",
            "sample": f"{nq} of the {B} queries against all {int(index.num_docs):,} docs",
            "wall_s": round(wall, 3), "cpu_s": round(cpu, 3),
            "cpu_over_wall": round(cpu / wall, 2), "parity_bit_exact_vs_gpu": exact,
            "single_core": {"value": n1 / wall1, "unit": "queries/s", "sample": f"{n1} queries"}}


def physical_cores():
    """One logical CPU per physical core (lscpu), within this process's affinity mask; the
    reference notes that nproc can misreport (final_results/corrected_2026_08/README.md)."""
    allowed = sorted(os.sched_getaffinity(0))
    try:
        out = subprocess.run(["lscpu", "-p=CPU,CORE,SOCKET"], capture_output=True, text=True,
                             timeout=20).stdout
        first = {}
        for line in out.splitlines():
            if line.startswith("#"):
                continue
            cpu, core, sock = (int(x) for x in line.split(",")[:3])
            if cpu in allowed:
                first.setdefault((sock, core), cpu)
        cpus = sorted(first.values())
        return cpus or allowed, "lscpu"
    except Exception:
        return allowed, "affinity mask"


def reference_cpu_paths(wl, qi_h, qs_h, k, target_s):
    """The reference's own CPU scoring paths on a bounded sample, pinned with
    sched_setaffinity (the taskset of baselines/seismic_k_calibration.py:50-52) to all
    physical cores and to one core: the exhaustive dense fp32 path
    (src/remeasure_2026_09.py:238-258: densified document chunks, Q @ D^T, torch.topk
    merge) and cpu_sequential_score (src/gpu_scoring.py:221-259, pure Python).  Each
    covers a prefix of the corpus's documents and is scaled to whole-corpus queries/s
    (both cost time in proportion to the documents scored)."""
    import numpy as np
    import torch
    from oracle import oracle as O
    N = wl["num_docs"]
    dlaw = O.Law(zipf_s=wl["zipf_s"])
    cores, how = physical_cores()
    saved_mask, saved_threads = os.sched_getaffinity(0), torch.get_num_threads()
    res = {}
    try:
        # dense: a few chunks of documents, as many queries as make ~target_s of work
        nd = min(N, 4 * 16384)
        ip, ix, dt = O.synth_csr(nd, V, seed=0, law=dlaw)
        for label, cpu_set in (("all_cores", cores), ("one_core", cores[:1])):
            os.sched_setaffinity(0, cpu_set)
            torch.set_num_threads(len(cpu_set))
            nq = 8 if label == "one_core" else 32
            Q = O.dense_query_matrix(qi_h[:nq], qs_h[:nq], V)
            r0 = resource.getrusage(resource.RUSAGE_SELF)
            t0 = time.perf_counter()
            O.dense_reference_topk(ip, ix, dt, V, Q, k, doc_hi=nd)
            wall = time.perf_counter() - t0
            r1 = resource.getrusage(resource.RUSAGE_SELF)
            cpu = (r1.ru_utime - r0.ru_utime) + (r1.ru_stime - r0.ru_stime)
            res[f"dense_{label}"] = {
                "value": nq / (wall * N / nd), "unit": "queries/s", "cores": len(cpu_set),
                "pin": f"{how}: cpus {cpu_set[0]}..{cpu_set[-1]}" if len(cpu_set) > 1 else f"cpu {cpu_set[0]}",
                "sample": f"{nq} queries x the first {nd:,} docs, scaled to {N:,}",
                "wall_s": round(wall, 3), "cpu_s": round(cpu, 3), "cpu_over_wall": round(cpu / wall, 2)}
        del ip, ix, dt
        # sequential: pure Python, one core
        ns = min(N, 20000)
        ip, ix, dt = O.synth_csr(ns, V, seed=0, law=dlaw)
        os.sched_setaffinity(0, cores[:1])
        _, _, secs = O.sequential_score(ip, ix, dt, qi_h[:2], qs_h[:2], ns, k)
        res["sequential_one_core"] = {
            "value": 2 / (secs * N / ns), "unit": "queries/s", "cores": 1, "pin": f"cpu {cores[0]}",
            "sample": f"2 queries x the first {ns:,} docs (index build excluded), scaled to {N:,}",
            "wall_s": round(secs, 3)}
    finally:
        os.sched_setaffinity(0, saved_mask)
        torch.set_num_threads(saved_threads)
    res["physical_cores"] = len(cores)
    res["logical_cpus"] = len(saved_mask)
    return res


def run_ours(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import gpusparse
    from gpusparse import _lib as L
    from gpusparse import synth
    from gpusparse.distributed import ShardLayout, sharded_score_topk

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=180))
    wl = workload(args)
    N, B, k, wd = wl["num_docs"], wl["batch"], wl["k"], wl["wdtype"]
    lay = ShardLayout(N, world, rank)
    head_code = {"auto": L.HEAD_AUTO, "cuda": L.HEAD_CUDA_CORES, "tc": L.HEAD_TENSOR_CORES}[args.head_mode]
    L.check(L.lib().gsp_set_head_mode(head_code), "head mode")
    dlaw = synth.Law(zipf_s=wl["zipf_s"])
    qlaw = synth.Law(zipf_s=wl["zipf_s"], nnz_mean=30.0, nnz_sd=15.0, nnz_lo=5, nnz_hi=128,
                     min_nnz_item0=107)
    t0 = time.time()
    index = synth.synth_index(N, V, seed=0, law=dlaw, doc_range=(lay.lo, lay.hi), device=dev,
                              weight_dtype=wd, keep_fp32=(wd == "fp32"))
    if world > 1:
        from gpusparse.distributed import global_head
        from gpusparse.index import N_HEAD, ensure_head
        ensure_head(index, head_ids=global_head(index, N_HEAD))
    qi, qs = synth.synth_queries(B, V, seed=1, law=qlaw, device=dev)
    torch.cuda.synchronize()
    build_s = time.time() - t0

    def step(qi_d, qs_d, events=None):
        return sharded_score_topk(index, lay, qi_d, qs_d, k, events=events)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(args.warmup, 0)):
        out = step(qi, qs)
    torch.cuda.synchronize()
    barrier()

    # ---- device-timed steps (inputs resident)
    clocks = ClockSampler()
    if rank == 0:
        clocks.start()
        time.sleep(0.3)
    L.check(L.lib().gsp_profile_enable(1), "profile")
    K = args.steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)]
    barrier()
    torch.cuda.synchronize()
    ev[0].record()
    for s_ in range(K):
        out = step(qi, qs)
        ev[s_ + 1].record()
    torch.cuda.synchronize()
    barrier()
    per_step = [ev[j].elapsed_time(ev[j + 1]) for j in range(K)]
    phases = None
    if args.phase_split:
        # separate steps, so the timed ones above carry no extra events
        acc = {}
        for _ in range(K):
            e0_ = torch.cuda.Event(enable_timing=True)
            e0_.record()
            evs = []
            step(qi, qs, events=evs)
            torch.cuda.synchronize()
            prev = e0_
            for name, e in evs:
                acc[name] = acc.get(name, 0.0) + prev.elapsed_time(e)
                prev = e
        phases = {n: max_over_ranks(v / K) for n, v in acc.items()}
    total_ms = max_over_ranks(ev[0].elapsed_time(ev[K]))
    import ctypes
    tot, n = ctypes.c_double(0.0), ctypes.c_int64(0)
    L.check(L.lib().gsp_profile_collect(ctypes.byref(tot), ctypes.byref(n)), "profile")
    L.check(L.lib().gsp_profile_enable(0), "profile")
    kern_ms = max_over_ranks(tot.value / max(n.value, 1))
    p50 = statistics.median(per_step)
    p90 = sorted(per_step)[min(K - 1, int(0.9 * K))]
    p50 = max_over_ranks(p50)
    p90 = max_over_ranks(p90)
    clk = clocks.stop(world) if rank == 0 else None

    # ---- end to end through the public API (pinned host buffers both ways)
    qi_h = qi.cpu().pin_memory()
    qs_h = qs.cpu().pin_memory()
    qi_d = torch.empty_like(qi)
    qs_d = torch.empty_like(qs)
    s0, i0 = out
    s_h = torch.empty(s0.shape, dtype=s0.dtype).pin_memory()
    i_h = torch.empty(i0.shape, dtype=i0.dtype).pin_memory()

    def e2e_step():
        qi_d.copy_(qi_h, non_blocking=True)
        qs_d.copy_(qs_h, non_blocking=True)
        s, i = step(qi_d, qs_d)
        if rank == 0:
            s_h.copy_(s, non_blocking=True)
            i_h.copy_(i, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return s_h, i_h

    for _ in range(max(args.warmup, 1)):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    h2d = qi.numel() * qi.element_size() + qs.numel() * qs.element_size()
    d2h = s0.numel() * s0.element_size() + i0.numel() * i0.element_size()

    # ---- one query alone (after the timed region; small-batch latency, device time, p50)
    lat1 = None
    if world == 1:
        q1, s1 = qi[1:2].contiguous(), qs[1:2].contiguous()   # query 0 is the forced 107+-term one
        for _ in range(3):
            step(q1, s1)
        t1 = []
        for _ in range(9):
            a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a_.record()
            step(q1, s1)
            b_.record()
            torch.cuda.synchronize()
            t1.append(a_.elapsed_time(b_))
        lat1 = statistics.median(t1)

    # ---- roofline of the scoring kernel (this rank's shard)
    from gpusparse.index import index_memory_stats
    index_bytes = int(index_memory_stats(index)["total_MB"] * 1e6)
    balg, post = bytes_alg(index, qi, B, min(k, index.num_docs), wd)
    balg = max_over_ranks(balg)
    mads = max_over_ranks(contributions(index, qi))
    peak, peak_src = peaks()
    achieved = balg / (kern_ms * 1e-3) / 1e9
    traffic, traffic_src = measured_traffic(args.config, world, args.num_docs)
    if args.head_mode == "tc":
        traffic, traffic_src = None, "the committed profile covers the CUDA-core scorer"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gs, gi = (x.cpu().numpy() for x in out)
        cpu = cpu_sample(index, qi, qs, k, gs, gi, args.cpu_seconds)
        cpu["reference_paths"] = reference_cpu_paths(wl, qi.cpu().numpy(), qs.cpu().numpy(), k,
                                                     args.cpu_seconds)

    sharing = None
    if world > 1:
        from gpusparse.distributed import _BOARDS, release_threshold_boards, shared_thresholds_enabled
        mapped = sum(len(b.peers[0]) for b in _BOARDS.values())
        sharing = (f"on: union bound over {world} shards, {mapped} peer boards mapped"
                   if shared_thresholds_enabled() else "off")
        release_threshold_boards()
        dist.destroy_process_group()
    if rank != 0:
        return
    # plan, score, candidate counts, shard merge (+ global merge); the tensor-core mode adds
    # the query head-weight kernel
    launches_per_step = (4 if world == 1 else 5) + (1 if args.head_mode == "tc" else 0)
    line = {
        "metric": METRIC,
        "value": B * K / (total_ms * 1e-3),
        "unit": "queries/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": total_ms / K,
        "p50_ms": p50,
        "p90_ms": p90,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded SPLADE-shaped law of BASELINE.json; generated on device)",
        "config": {"workload": wl["name"], "num_docs": N, "batch": B, "k": k, "vocab": V,
                   "weights": wd, "parallelism": f"doc-range shards x{world}" +
                   (" + NCCL all-to-all of query blocks, merge, all-gather" if world > 1 else ""),
                   "l2": "inputs larger than L2 (index >> 126 MB); no flush",
                   "index_build_s": round(build_s, 2),
                   "index_device_bytes": index_bytes,
                   **({"exchange": __import__("gpusparse.distributed", fromlist=["x"]).exchange_mode()}
                      if world > 1 else {}),
                   "head_terms": {"auto": "library choice (CUDA cores)", "cuda": "CUDA cores",
                                  "tc": "tensor cores (tcgen05, 3xTF32)"}[args.head_mode],
                   **({"threshold_sharing": sharing} if sharing else {})},
        "gpu_launches": launches_per_step * K,
        **({"phases_ms": phases} if phases else {}),
        **({"single_query_latency": {"batch": 1, "k": k, "p50_ms": lat1,
                                     "note": "query 1 of the batch alone, device time"}}
           if lat1 is not None else {}),
        "e2e": {"value": B * K / (e2e_ms * 1e-3), "unit": "queries/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_src,
                     "source_tag": source_tag(), "peak_source": peak_src,
                     "kernel": "score_kernel", "kernel_ms": kern_ms,
                     "bytes_alg_per_launch": balg, "postings_per_launch": post,
                     "multiply_adds_per_launch": mads},
        "cpu_baseline": cpu,
        "clocks": clk,
    }
    emit(line)


def run_reference(args):
    """The reference's CPU scoring path for the same workload (C oracle port)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle as O
    wl = workload(args)
    N, B, k, wd = wl["num_docs"], wl["batch"], wl["k"], wl["wdtype"]
    nt = O.nthreads_default()
    dlaw = O.Law(zipf_s=wl["zipf_s"])
    qlaw = O.Law(zipf_s=wl["zipf_s"], nnz_mean=30.0, nnz_sd=15.0, nnz_lo=5, nnz_hi=128,
                 min_nnz_item0=107)
    t0 = time.time()
    ip, ix, dt = O.synth_csr(N, V, seed=0, law=dlaw, nthreads=nt)
    idx = O.build_index(ip, ix, dt, V)
    del ip, ix, dt
    w = None
    if wd == "u8":
        q, sc = O.quantize_u8(idx)
        w = O.dequantize_u8(q, sc, idx.offsets, idx.lengths, idx.padded_lengths)
    elif wd == "bf16":
        import torch
        w = torch.from_numpy(idx.scores).bfloat16().float().numpy()
    qi, qs = O.synth_queries(B, V, seed=1, law=qlaw)
    build_s = time.time() - t0
    # one step = a bounded sample of the batch sized to ~cpu-seconds, all host threads
    t0 = time.perf_counter()
    O.score_topk(idx, qi[:nt], qs[:nt], k, weights=w, nthreads=nt)
    one = time.perf_counter() - t0
    nq = int(min(B, max(nt, nt * int(max(1.0, args.cpu_seconds / 4) / max(one, 1e-3)))))
    times, cpu = [], 0.0
    for s_ in range(args.warmup + args.steps):
        lo = (s_ * nq) % B
        sel = np.arange(lo, lo + nq) % B
        r0 = resource.getrusage(resource.RUSAGE_SELF)
        t0 = time.perf_counter()
        O.score_topk(idx, qi[sel], qs[sel], k, weights=w, nthreads=nt)
        t1 = time.perf_counter()
        r1 = resource.getrusage(resource.RUSAGE_SELF)
        if s_ >= args.warmup:
            times.append(t1 - t0)
            cpu += (r1.ru_utime - r0.ru_utime) + (r1.ru_stime - r0.ru_stime)
    wall = sum(times)
    value = nq * len(times) / wall
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "queries/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * wall / len(times), "p50_ms": 1e3 * statistics.median(times),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded SPLADE-shaped law of BASELINE.json; generated on host)",
        "config": {"workload": wl["name"], "num_docs": N, "batch": B, "k": k, "vocab": V,
                   "weights": wd, "step_sample_queries": nq,
                   "index_build_s": round(build_s, 1)},
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": nt, "kind": "port",
                         "sample": f"{nq} queries per step against all {N:,} docs",
                         "cpu_over_wall": round(cpu / max(wall, 1e-9), 2),
                         "threads": nt, "affinity": f"{len(os.sched_getaffinity(0))} logical CPUs",
                         "physical_cores": len(physical_cores()[0])},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


def run_cusparse(args):
    """Context line, not the reference arm: the same workload through cuSPARSE SpMM and
    torch.topk on one GPU.  Its fp32 sums run in another order than the canonical one, so
    it is compared with this build's result by score within the 1e-5 relative tolerance."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    import gpusparse
    from gpusparse import synth
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = workload(args)
    N, B, k = wl["num_docs"], wl["batch"], wl["k"]
    dlaw = synth.Law(zipf_s=wl["zipf_s"])
    qlaw = synth.Law(zipf_s=wl["zipf_s"], nnz_mean=30.0, nnz_sd=15.0, nnz_lo=5, nnz_hi=128,
                     min_nnz_item0=107)
    ch = 1 << 21
    chunks = []
    for lo in range(0, N, ch):
        n = min(ch, N - lo)
        ip, ix, dt = synth.synth_csr(n, V, seed=0, first=lo, law=dlaw, device=dev)
        chunks.append((lo, torch.sparse_csr_tensor(ip.to(torch.int32), ix, dt, size=(n, V))))
    qi, qs = synth.synth_queries(B, V, seed=1, law=qlaw, device=dev)
    Q = torch.zeros((V, B), dtype=torch.float32, device=dev)
    ok = qi >= 0
    cols = torch.arange(B, device=dev).unsqueeze(1).expand_as(qi)
    Q.index_put_((qi[ok].long(), cols[ok]), qs[ok], accumulate=True)

    def step():
        bs = bi = None
        for lo, A in chunks:
            S = torch.sparse.mm(A, Q)
            s, i = torch.topk(S, min(k, S.shape[0]), dim=0)
            i = i + lo
            if bs is None:
                bs, bi = s, i
            else:
                cs, ci = torch.cat([bs, s]), torch.cat([bi, i])
                bs, j = torch.topk(cs, k, dim=0)
                bi = torch.gather(ci, 0, j)
        return bs.t(), bi.t()

    for _ in range(max(args.warmup, 1)):
        out = step()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    ev[0].record()
    for j in range(args.steps):
        out = step()
        ev[j + 1].record()
    torch.cuda.synchronize()
    per = [ev[j].elapsed_time(ev[j + 1]) for j in range(args.steps)]
    total = ev[0].elapsed_time(ev[args.steps])
    s_lib = out[0].contiguous()
    del chunks, out
    torch.cuda.empty_cache()
    index = synth.synth_index(N, V, seed=0, law=dlaw, device=dev)
    s_ours, _ = gpusparse.triton_fused_score(index, qi, qs, top_k=k)
    rel = float(((s_lib - s_ours).abs() / s_ours.abs().clamp_min(1e-30)).max().item())
    line = {
        "impl": "cusparse", "metric": METRIC, "value": B * args.steps / (total * 1e-3),
        "unit": "queries/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total / args.steps, "p50_ms": statistics.median(per),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded SPLADE-shaped law of BASELINE.json; generated on device)",
        "config": {"workload": wl["name"], "num_docs": N, "batch": B, "k": k, "vocab": V,
                   "route": "torch.sparse.mm (cuSPARSE SpMM) per 2M-document chunk + torch.topk",
                   "max_rel_score_diff_vs_ours": rel},
    }
    emit(line)


def run_spare(args):
    """Context line: the SPARe-style iterative loop (one index_add_ per query term over the
    term-major posting arrays, then torch.topk per query) on one GPU, timed on a bounded
    sample of the batch's queries."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    from gpusparse import synth
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    wl = workload(args)
    N, B, k = wl["num_docs"], wl["batch"], wl["k"]
    dlaw = synth.Law(zipf_s=wl["zipf_s"])
    qlaw = synth.Law(zipf_s=wl["zipf_s"], nnz_mean=30.0, nnz_sd=15.0, nnz_lo=5, nnz_hi=128,
                     min_nnz_item0=107)
    index = synth.synth_index(N, V, seed=0, law=dlaw, device=dev)
    qi, qs = synth.synth_queries(B, V, seed=1, law=qlaw, device=dev)
    off = index.offsets.cpu().tolist()
    ln = index.lengths.cpu().tolist()
    qi_h, qs_h = qi.cpu().tolist(), qs.cpu()
    doc_ids, wts = index.doc_ids, index.scores

    def one(b):
        acc = torch.zeros(N, dtype=torch.float32, device=dev)
        for j, t in enumerate(qi_h[b]):
            if 0 <= t < V and ln[t] > 0:
                s0, s1 = off[t], off[t] + ln[t]
                acc.index_add_(0, doc_ids[s0:s1].long(), wts[s0:s1] * float(qs_h[b, j]))
        return torch.topk(acc, k)

    one(0)
    torch.cuda.synchronize()
    # size the sample to a few seconds per step
    t0 = time.perf_counter()
    one(1 % B)
    torch.cuda.synchronize()
    per_q = max(time.perf_counter() - t0, 1e-4)
    nq = int(max(1, min(B, 3.0 / per_q)))
    times = []
    for s_ in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for b in range(nq):
            one((s_ * nq + b) % B)
        torch.cuda.synchronize()
        if s_ >= args.warmup:
            times.append(time.perf_counter() - t0)
    wall = sum(times)
    line = {
        "impl": "spare", "metric": METRIC, "value": nq * len(times) / wall, "unit": "queries/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * wall / len(times), "p50_ms": 1e3 * statistics.median(times),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded SPLADE-shaped law of BASELINE.json; generated on device)",
        "config": {"workload": wl["name"], "num_docs": N, "batch": B, "k": k, "vocab": V,
                   "route": "per query: torch index_add_ per term + torch.topk (host-timed)",
                   "step_sample_queries": nq},
    }
    emit(line)


_JSON_FD = None


def emit(line: dict) -> None:
    """Write the one JSON result line to the process's original stdout."""
    os.write(_JSON_FD if _JSON_FD is not None else 1, (json.dumps(line) + "\n").encode())


def main():
    global _JSON_FD
    # Libraries (NCCL's version banner, for one) may print to stdout; everything but the
    # result line goes to stderr so that stdout holds exactly one JSON line.
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "cusparse":
        run_cusparse(args)
    elif args.impl == "spare":
        run_spare(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
