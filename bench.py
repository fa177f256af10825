#!/usr/bin/env python
"""Benchmark of the exact flat scan + top-k (MetalANNS search hot path).

Workload: n = 1,000,000 x d = 384 fp32 rows, i.i.d.
N(0,1) then L2-normalised, cosine, top-10, synthetic (numpy default_rng(0):
database first, then the queries from the same generator).  One step = one
batch of --nq queries searched exactly.  With --gpus N > 1 (launched by
torch.distributed.run) the rows are sharded contiguously over the ranks, each
rank scans its shard, the per-shard top-k blocks are all-gathered over NCCL
and merged on the device by (distance, id).

`value` is device-timed with inputs resident in HBM; `e2e` goes through the
public C ABI with pinned host buffers (query upload and result download inside
the timed region).  `--impl reference` times the reference CPU exact path
(ParallelFlatScan restated in oracle/, inner loop = the reference's own dots.c
when it was built) on the host cores instead.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC_NAMES = {"cosine": 0, "l2": 1, "ip": 2}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--n", type=int, default=1_000_000)
    ap.add_argument("--dim", type=int, default=384)
    ap.add_argument("--nq", type=int, default=1)
    ap.add_argument("--k", type=int, default=10)
    ap.add_argument("--metric", default="cosine", choices=list(METRIC_NAMES))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--tc-min-batch", type=int, default=16,
                    help="batches of at least this many queries use the tensor-core path")
    ap.add_argument("--no-also", action="store_true",
                    help="skip the extra measurements reported under `also`")
    ap.add_argument("--no-index", action="store_true",
                    help="skip the IVF-flat / IVF-PQ lines of the default flat run")
    ap.add_argument("--also-nq", default="32,1024",
                    help="comma-separated batch sizes of the extra flat measurements")
    ap.add_argument("--workload", default="flat", choices=["flat", "ivf", "ivfpq"],
                    help="flat: exact scan (configs[1]); ivf: IVF-flat (configs[2]); "
                         "ivfpq: IVF-PQ ADC (configs[3])")
    ap.add_argument("--nlist", type=int, default=None)
    ap.add_argument("--nprobe", type=int, default=None)
    ap.add_argument("--components", type=int, default=None)
    ap.add_argument("--pq-m", type=int, default=16)
    ap.add_argument("--pq-shard", default="list", choices=["list", "row"],
                    help="IVF-PQ over N > 1 GPUs: whole inverted lists per rank (each rank "
                         "builds tables only for the probed lists it holds) or row ranges")
    ap.add_argument("--ivf-layout", default="replica", choices=["replica", "shard"],
                    help="IVF-flat at N > 1: a full replica of the index per GPU, each GPU "
                         "serving its own queries (default; the 1M-row index fits one GPU), "
                         "or row shards with a merge of every query's per-shard blocks")
    ap.add_argument("--transport", default="p2p", choices=["p2p", "nccl"],
                    help="how row shards exchange their top-k blocks (N > 1)")
    a = ap.parse_args()
    # per-workload defaults (BASELINE.json configs[2] and [3])
    if a.workload == "ivf":
        a.nlist = a.nlist or 1024
        a.nprobe = a.nprobe or 8
        a.components = a.components or 1024
    elif a.workload == "ivfpq":
        a.nlist = a.nlist or 4096
        a.nprobe = a.nprobe or 32
        a.components = a.components or 4096
        if "--n" not in sys.argv:
            a.n = 10_000_000
        if "--dim" not in sys.argv:
            a.dim = 128
        if "--metric" not in sys.argv:
            a.metric = "l2"
        if "--nq" not in sys.argv:
            a.nq = 1024
    return a


def make_data(n, dim, nq, seed=0):
    rng = np.random.default_rng(seed)
    v = rng.standard_normal((n, dim), dtype=np.float32)
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    q = rng.standard_normal((nq, dim), dtype=np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    return v, q


# Draws of at least this many elements use torch's CUDA generator when a GPU
# is present: numpy's single-stream generator takes minutes for 10M x 128.
_DEVICE_DRAW_ELEMENTS = 1 << 26


def make_mixture(n, dim, components, nq, sigma=0.3, seed=0):
    """BASELINE.json configs[2..3] generator: centres = normalise(N(0,1)),
    x = centre[assign] + sigma * N(0,1), renormalised; queries drawn from the
    same mixture after the database.  The noise is drawn in row chunks, which
    yields the same values as one draw and bounds the temporaries.  Below
    2^26 elements (or without a GPU) the draws come from numpy
    default_rng(seed); above, from torch's CUDA Philox generator seeded with
    `seed` (same distribution, same values on every GPU of a run)."""
    if n * dim >= _DEVICE_DRAW_ELEMENTS:
        try:
            import torch
            if torch.cuda.is_available():
                return _mixture_on_device(n, dim, components, nq, sigma, seed)
        except ImportError:
            pass
    rng = np.random.default_rng(seed)
    centres = rng.standard_normal((components, dim), dtype=np.float32)
    centres /= np.linalg.norm(centres, axis=1, keepdims=True)

    def draw(m):
        a = rng.integers(0, components, m)
        x = np.empty((m, dim), np.float32)
        for c0 in range(0, m, 1 << 20):
            c1 = min(m, c0 + (1 << 20))
            x[c0:c1] = centres[a[c0:c1]] + np.float32(sigma) * rng.standard_normal(
                (c1 - c0, dim), dtype=np.float32)
            x[c0:c1] /= np.linalg.norm(x[c0:c1], axis=1, keepdims=True)
        return x

    return draw(n), draw(nq)


def _mixture_on_device(n, dim, components, nq, sigma, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    centres = torch.randn((components, dim), generator=g, device="cuda", dtype=torch.float32)
    centres /= centres.norm(dim=1, keepdim=True)

    def draw(m):
        out = np.empty((m, dim), np.float32)
        for c0 in range(0, m, 1 << 21):
            c1 = min(m, c0 + (1 << 21))
            a = torch.randint(0, components, (c1 - c0,), generator=g, device="cuda")
            x = centres[a] + sigma * torch.randn((c1 - c0, dim), generator=g, device="cuda",
                                                 dtype=torch.float32)
            x /= x.norm(dim=1, keepdim=True)
            out[c0:c1] = x.cpu().numpy()
        return out

    v = draw(n)
    q = draw(nq)
    return v, q


def train_centroids(v, nlist, iters=4, seed=42, device=None):
    """Coarse centroids: Lloyd iterations on a strided sample of
    min(n, max(L, min(4096, 16L))) rows, the sample size of
    IVFFlatSearch.buildPartition (IVFFlatSearch.swift:529-551), with torch
    matmuls (the reference's KMeans is seeded by Swift's generator, which
    cannot be reproduced here)."""
    import torch
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    n = v.shape[0]
    sample = min(n, max(nlist, min(4096, 16 * nlist)))
    stride = max(1, n // sample)
    x = torch.from_numpy(v[::stride][:sample]).to(dev)
    g = torch.Generator(device="cpu").manual_seed(seed)
    cent = x[torch.randperm(x.shape[0], generator=g)[:nlist].to(dev)].clone()
    for _ in range(iters):
        a = torch.argmax(x @ cent.T - 0.5 * (cent * cent).sum(1), dim=1)
        s = torch.zeros_like(cent).index_add_(0, a, x)
        c = torch.bincount(a, minlength=nlist).unsqueeze(1).to(s.dtype)
        cent = torch.where(c > 0, s / c.clamp(min=1), cent)
    return cent.cpu().numpy().astype(np.float32)


def train_pq_codebooks(v, coarse, m, iters=4, seed=43, device=None):
    """Per-subspace 256-centroid codebooks on the residuals of a 65,536-row
    sample (torch; codebook training is outside the search path)."""
    import torch
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    n, dim = v.shape
    sub = dim // m
    g = torch.Generator(device="cpu").manual_seed(seed)
    samp = torch.randperm(n, generator=g)[:min(n, 65536)].numpy()
    x = torch.from_numpy(v[samp]).to(dev)
    ct = torch.from_numpy(coarse).to(dev)
    near = torch.argmin(torch.cdist(x, ct), dim=1)
    x = x - ct[near]
    books = []
    for s in range(m):
        xs = x[:, s * sub:(s + 1) * sub]
        cb = xs[torch.randperm(xs.shape[0], generator=g)[:256].to(dev)].clone()
        for _ in range(iters):
            a = torch.argmin(torch.cdist(xs, cb), dim=1)
            acc = torch.zeros_like(cb).index_add_(0, a, xs)
            c = torch.bincount(a, minlength=256).unsqueeze(1).to(acc.dtype)
            cb = torch.where(c > 0, acc / c.clamp(min=1), cb)
        books.append(cb)
    return torch.stack(books).cpu().numpy().astype(np.float32)


def train_partition(v, nlist, metric, iters=4, seed=42, device=None):
    """Coarse centroids + row assignment for an IVF partition (build-time step,
    outside the search path): Lloyd iterations on a strided sample, as
    IVFFlatSearch.buildPartition samples min(n, max(L, min(4096, 16L))) rows
    (IVFFlatSearch.swift:529-551), computed with torch matmuls.  Returns
    (centroids, assignment) with assignment = argmin of the metric key."""
    import torch
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    n = v.shape[0]
    cent = torch.from_numpy(train_centroids(v, nlist, iters=iters, seed=seed, device=dev)).to(dev)
    full = torch.from_numpy(v).to(dev)
    cn = (cent * cent).sum(1)
    assign = torch.empty(n, dtype=torch.int64, device=dev)
    for a0 in range(0, n, 65536):
        xb = full[a0:a0 + 65536]
        dots = xb @ cent.T
        if metric == 2:
            key = -dots
        elif metric == 1:
            key = cn - 2 * dots
        else:
            key = -dots / cn.clamp(min=1e-20).sqrt()
        assign[a0:a0 + 65536] = torch.argmin(key, dim=1)
    return cent.cpu().numpy().astype(np.float32), assign.cpu().numpy()


def train_ivfpq(v, nlist, m, metric=1, iters=4, seed=42, device=None):
    """Trained IVF-PQ artefacts for synthetic data (a build-time step outside
    the search path): coarse centroids by Lloyd iterations, per-subspace
    256-centroid codebooks on residuals of a sample, codes by nearest
    codebook entry and inverted lists in insertion (row) order.  Torch
    matmuls; the search kernels take these as inputs."""
    import torch
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    n, dim = v.shape
    sub = dim // m
    cent, assign = train_partition(v, nlist, metric, iters=iters, seed=seed, device=dev)
    g = torch.Generator(device="cpu").manual_seed(seed + 1)
    samp = torch.randperm(n, generator=g)[:min(n, 65536)]
    x = torch.from_numpy(v[samp.numpy()]).to(dev) - torch.from_numpy(cent[assign[samp.numpy()]]).to(dev)
    books = []
    for s in range(m):
        xs = x[:, s * sub:(s + 1) * sub]
        cb = xs[torch.randperm(xs.shape[0], generator=g)[:256].to(dev)].clone()
        for _ in range(iters):
            a = torch.argmin(torch.cdist(xs, cb), dim=1)
            acc = torch.zeros_like(cb).index_add_(0, a, xs)
            c = torch.bincount(a, minlength=256).unsqueeze(1).to(acc.dtype)
            cb = torch.where(c > 0, acc / c.clamp(min=1), cb)
        books.append(cb)
    codebooks = torch.stack(books)  # m x 256 x sub
    codes = torch.empty((n, m), dtype=torch.uint8, device=dev)
    ct = torch.from_numpy(cent).to(dev)
    at = torch.from_numpy(assign).to(dev)
    for a0 in range(0, n, 262144):
        r = torch.from_numpy(v[a0:a0 + 262144]).to(dev) - ct[at[a0:a0 + 262144]]
        for s in range(m):
            d = torch.cdist(r[:, s * sub:(s + 1) * sub], codebooks[s])
            codes[a0:a0 + 262144, s] = torch.argmin(d, dim=1).to(torch.uint8)
    order = np.argsort(assign, kind="stable").astype(np.uint32)
    offsets = np.concatenate([[0], np.cumsum(np.bincount(assign, minlength=nlist))]).astype(np.int64)
    return (cent, codebooks.cpu().numpy().astype(np.float32), codes.cpu().numpy(),
            offsets, order)


def p50(xs):
    s = sorted(xs)
    return s[max(0, math.ceil(0.5 * len(s)) - 1)]  # nearest rank (LatencyDistribution.swift:154-160)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic(workload, kernel="scan"):
    """Per-launch DRAM bytes (read + write) of the dominant kernel from the
    committed ncu summaries, keyed "<workload>/<kernel>"."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        d = json.load(f)
    return d.get(f"{workload}/{kernel}")


def cpu_reference_qps(v, q, k, metric, seconds, max_queries=None, cores=None):
    """ParallelFlatScan (the reference CPU exact path) on the host cores
    (all of them unless `cores` is given)."""
    import oracle as O
    cores = cores or os.cpu_count() or 1
    used = min(cores, 32, max(1, v.shape[0] // 2048))  # ParallelFlatScan.sliceCount
    norms = O.row_norms(v) if metric in (0, 1) else None
    use_ref = O.ref_lib() is not None
    O.parallel_flat_scan(v, q[0], k, metric, cores, norms=norms, use_reference_dots=use_ref)
    t0 = time.perf_counter()
    done = 0
    while True:
        O.parallel_flat_scan(v, q[done % len(q)], k, metric, cores, norms=norms,
                             use_reference_dots=use_ref)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds or (max_queries and done >= max_queries):
            break
    return done / el, used, done, use_ref


def cpu_batch_qps(v, q, k, metric, seconds):
    """The reference CPU route for query batches at n >= 16384
    (FlatGPUSearch.parallelHostBatchSearch -> BoundedExactScan per query,
    queries in parallel on the host cores): int8 prefilter + fp32 rescore.
    The int8 planes are built once outside the timing (the reference caches
    them per corpus).  Rounds of `threads` queries until `seconds` pass."""
    import oracle as O
    cores = os.cpu_count() or 1
    planes = O.int8_planes(v)
    norms = O.row_norms(v) if metric in (0, 1) else None
    use_ref = O.ref_lib() is not None
    threads = cores
    O.bounded_exact_batch(v, planes, q[:threads], k, metric, threads, norms=norms,
                          use_reference_dots=use_ref)
    t0 = time.perf_counter()
    done = 0
    while True:
        idx = [(done + i) % len(q) for i in range(threads)]
        O.bounded_exact_batch(v, planes, q[idx], k, metric, threads, norms=norms,
                              use_reference_dots=use_ref)
        done += threads
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return done / el, threads, done, use_ref


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload != "flat":
        run_reference_index(args)
        return
    metric = METRIC_NAMES[args.metric]
    v, q = make_data(args.n, args.dim, max(args.nq, 1))
    import oracle as O
    cores = os.cpu_count() or 1
    used = min(cores, 32, max(1, v.shape[0] // 2048))
    norms = O.row_norms(v) if metric in (0, 1) else None
    use_ref = O.ref_lib() is not None
    batch = args.nq > 1 and v.shape[0] >= 16384
    # Each step is a bounded sample of the batch: queries are independent on
    # the CPU routes, so per-query throughput does not depend on the batch
    # size, and a full 1024-query batch would take seconds per step.
    per_step = min(args.nq, 2 * cores) if batch else min(args.nq, 8)
    if batch:
        # FlatGPUSearch.batchSearch on the host tier: BoundedExactScan per
        # query, queries in parallel (the int8 planes are cached per corpus)
        planes = O.int8_planes(v)
        used = cores

        def one_step():
            O.bounded_exact_batch(v, planes, q[:per_step], args.k, metric, cores, norms=norms,
                                  use_reference_dots=use_ref)
    else:
        def one_step():
            for j in range(per_step):
                O.parallel_flat_scan(v, q[j], args.k, metric, cores, norms=norms,
                                     use_reference_dots=use_ref)
    for i in range(args.warmup):
        one_step()
    times = []
    for i in range(args.steps):
        t = time.perf_counter()
        one_step()
        times.append(time.perf_counter() - t)
    total = sum(times)
    value = per_step * args.steps / total
    line = {
        "impl": "reference", "metric": "queries_per_sec", "value": value, "unit": "queries/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "p50_us": 1e6 * p50(times),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(args),
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": used,
                         "kind": "port",
                         "sample": (f"{per_step} of the batch's {args.nq} queries per step "
                                    f"through the batch route (BoundedExactScan restated: "
                                    f"int8 prefilter + fp32 rescore, queries in parallel)"
                                    if batch else
                                    f"{per_step} of {args.nq} quer{'y' if args.nq == 1 else 'ies'} "
                                    f"per step, full {args.n}x{args.dim} scan; ParallelFlatScan "
                                    f"restated")
                                   + f", inner loops {'reference dots.c' if use_ref else 'restated dots.c'}"},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_index(args):
    """Reference arm of the IVF workloads: the restated single-threaded
    reference search per query (index artefacts trained as in our arm)."""
    v, q, art = build_index_data(args, max(args.nq, 1))
    qs = q[:max(args.nq, 1)]
    one = index_searcher(args, v, art)
    for i in range(args.warmup):
        one(qs[i % len(qs)])
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        for j in range(args.nq):
            one(qs[j])
        times.append(time.perf_counter() - t)
    total = sum(times)
    value = args.nq * args.steps / total
    print(json.dumps({
        "impl": "reference", "metric": "queries_per_sec", "value": value, "unit": "queries/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "p50_us": 1e6 * p50(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": index_workload_config(args),
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": 1, "kind": "port",
                         "sample": f"{args.nq} queries per step, one thread"},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


def workload_config(args, nq=None):
    nq = args.nq if nq is None else nq
    return {"workload": f"exact_flat_{args.n}x{args.dim}_{args.metric}_top{args.k}_nq{nq}",
            "n": args.n, "dim": args.dim, "nq": nq, "k": args.k, "metric": args.metric,
            "parallelism": f"rowshard{args.gpus}",
            "l2": l2_note(args.n * args.dim * 4)}


def l2_note(corpus_bytes, l2_bytes=126 << 20):
    """How the timed steps relate to the 126 MB L2: the rule is inputs larger
    than L2 or a flush between steps."""
    if corpus_bytes > l2_bytes:
        return (f"inputs larger than L2 (corpus {corpus_bytes / 1e9:.2f} GB streamed "
                f"per step)")
    return (f"corpus ({corpus_bytes / 1e6:.1f} MB) fits in L2: steps after the first read "
            f"it from L2")


def measured_bf16_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


class Runner:
    """Runs search steps of one batch size on this rank's row shard."""

    def __init__(self, args, torch, mb, lib, ctx, buf, ws, world, rank, dist, metric):
        self.a, self.torch, self.mb, self.lib = args, torch, mb, lib
        self.ctx, self.buf, self.ws = ctx, buf, ws
        self.world, self.rank, self.dist, self.metric = world, rank, dist, metric
        self.stream = torch.cuda.current_stream()
        self.sp = self.stream.cuda_stream

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def _sharded(self, nq, kout):
        sharded = self.mb.ShardedFlatSearch(self.ctx, self.buf, self.world, self.dist,
                                            transport=self.a.transport, rank=self.rank)
        return sharded, sharded.buffers(nq, kout)

    def _host_search(self, hq_ptr, nq, h_out, kout):
        rc = self.lib.mans_flat_search(self.ctx.handle, self.buf.handle, C.c_void_p(hq_ptr), nq,
                                       self.a.dim, self.a.k, self.metric,
                                       C.c_void_p(h_out.data_ptr()),
                                       C.c_void_p(h_out[nq * kout:].data_ptr()),
                                       C.c_void_p(h_out[2 * nq * kout:].data_ptr()))
        self.mb.check(rc)

    def measure(self, q, steps, warmup, with_clocks):
        """`q` is (P, nq, dim): step i searches batch i % P (P distinct
        single queries for the nq = 1 line, one batch otherwise)."""
        torch, mb, a = self.torch, self.mb, self.a
        pool, nq = q.shape[0], q.shape[1]
        kout = min(a.k, mb.MAX_TOP_K)
        dq = torch.from_numpy(np.ascontiguousarray(q)).cuda()
        P = mb.shard.packed_words(nq, kout)  # packed [dist | ids | counts] per rank
        ws, sp = self.ws, self.sp
        sharded, bufs = self._sharded(nq, kout)
        out = bufs[2]

        def step(src):
            return sharded.search_device(ws, src.data_ptr(), nq, a.k, self.metric, bufs, sp)

        for i in range(max(3, warmup)):
            step(dq[i % pool])
        ws.check(sp)
        ws.stats()
        ws.set_timing(True)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        clocks = ClockSampler(torch.cuda.current_device()) if with_clocks else None
        if clocks:
            clocks.start()
            time.sleep(0.3)
        self.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(self.stream)
        for i in range(steps):
            ev[i][0].record(self.stream)
            step(dq[i % pool])
            ev[i][1].record(self.stream)
        t1.record(self.stream)
        self.barrier()
        clock_info = clocks.stop() if clocks else None
        ws.check(sp)
        kern_ms, kern_launches, total_launches = ws.stats()
        ws.set_timing(False)
        path = ws.last_path()
        fallbacks = ws.fallbacks()
        total_ms = t0.elapsed_time(t1)
        step_ms = [x.elapsed_time(y) for x, y in ev]
        device_out = out.clone()

        # end to end through the C ABI with pinned host buffers
        hq = torch.from_numpy(np.ascontiguousarray(q)).pin_memory()
        h_out = torch.empty((P,), dtype=torch.int32).pin_memory()
        dq2 = torch.empty_like(dq[0])

        def e2e_step(i):
            if self.world == 1:
                self._host_search(hq[i % pool].data_ptr(), nq, h_out, kout)
            else:
                dq2.copy_(hq[i % pool], non_blocking=True)
                r = step(dq2)
                h_out.copy_(r, non_blocking=True)
                torch.cuda.current_stream().synchronize()

        # per-stage breakdown (CUDA events around every kernel of a step,
        # outside the timed region above; max over ranks per stage)
        n_st = min(steps, 20)
        ws.set_timing(False, stages=True)
        self.barrier()
        for i in range(n_st):
            step(dq[i % pool])
        self.barrier()
        st = ws.stage_times()
        ws.set_timing(False)
        stage_t = torch.tensor([st[name][0] for name in ws.STAGES], dtype=torch.float64,
                               device="cuda")
        stage_n = [st[name][1] for name in ws.STAGES]

        for i in range(max(3, warmup)):
            e2e_step(i)
        self.barrier()
        e2e_times = []
        for i in range(steps):
            t = time.perf_counter()
            e2e_step(i)
            e2e_times.append(time.perf_counter() - t)
        self.barrier()
        ok = bool(torch.equal(device_out.cpu(), h_out))

        stats = torch.tensor([total_ms, sum(e2e_times) * 1e3, kern_ms / max(kern_launches, 1)],
                             dtype=torch.float64, device="cuda")
        steps_t = torch.tensor(step_ms, dtype=torch.float64, device="cuda")
        e2e_t = torch.tensor(e2e_times, dtype=torch.float64, device="cuda")
        if self.world > 1:
            self.dist.all_reduce(stats, op=self.dist.ReduceOp.MAX)
            self.dist.all_reduce(steps_t, op=self.dist.ReduceOp.MAX)
            self.dist.all_reduce(e2e_t, op=self.dist.ReduceOp.MAX)
            self.dist.all_reduce(stage_t, op=self.dist.ReduceOp.MAX)
        total_ms, e2e_ms, kern_avg_ms = stats.tolist()
        stages_us = {name: round(1e3 * ms / n_st, 2)
                     for name, ms, c in zip(ws.STAGES, stage_t.tolist(), stage_n) if c > 0}
        # every rank is done with the peers' buffers before any is released
        self.barrier()
        sharded.close()
        return {"nq": nq, "steps": steps, "total_ms": total_ms, "e2e_ms": e2e_ms,
                "kern_avg_ms": kern_avg_ms, "kern_launches": kern_launches,
                "launches": total_launches, "p50_ms": p50(steps_t.tolist()),
                "e2e_p50_s": p50(e2e_t.tolist()), "clocks": clock_info, "ok": ok, "kout": kout,
                "path": path, "fallbacks_last_step": fallbacks,
                "distinct_batches": min(pool, steps), "stages_us": stages_us}

    def latency(self, qs):
        """Single-query latency over len(qs) distinct queries, each timed on
        its own (the reference's protocol: >= 200 queries timed individually,
        p50 by nearest rank, LatencyDistribution.swift:154-160).  Device time
        per query (CUDA events on the launching stream, queries not
        overlapped; max over ranks) and end-to-end time through the host C
        ABI; exact re-scans of the tensor-core path are counted."""
        torch, mb, a = self.torch, self.mb, self.a
        kout = min(a.k, mb.MAX_TOP_K)
        count = qs.shape[0]
        dq = torch.from_numpy(np.ascontiguousarray(qs)).cuda()
        ws, sp = self.ws, self.sp
        sharded, bufs = self._sharded(1, kout)
        for i in range(5):
            sharded.search_device(ws, dq[i % count].data_ptr(), 1, a.k, self.metric, bufs, sp)
        ws.check(sp)
        dev_ms, fallbacks = [], 0
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        self.barrier()
        for i in range(count):
            e0.record(self.stream)
            sharded.search_device(ws, dq[i].data_ptr(), 1, a.k, self.metric, bufs, sp)
            e1.record(self.stream)
            e1.synchronize()
            dev_ms.append(e0.elapsed_time(e1))
            fallbacks += ws.fallbacks()
            if self.world > 1:
                self.dist.barrier()
        ws.check(sp)
        e2e_s = []
        if self.world == 1:
            hq = torch.from_numpy(np.ascontiguousarray(qs)).pin_memory()
            h_out = torch.empty((self.mb.shard.packed_words(1, kout),),
                                dtype=torch.int32).pin_memory()
            for i in range(count):
                t = time.perf_counter()
                self._host_search(hq[i].data_ptr(), 1, h_out, kout)
                e2e_s.append(time.perf_counter() - t)
        d = torch.tensor(dev_ms, dtype=torch.float64, device="cuda")
        if self.world > 1:
            self.dist.all_reduce(d, op=self.dist.ReduceOp.MAX)
        self.barrier()
        sharded.close()
        dev = sorted(d.tolist())

        def rank_at(xs, f):
            return xs[max(0, math.ceil(f * len(xs)) - 1)]

        out = {"queries": count, "distinct": True, "p50_us": 1e3 * rank_at(dev, 0.5),
               "p90_us": 1e3 * rank_at(dev, 0.9), "p99_us": 1e3 * rank_at(dev, 0.99),
               "mean_us": 1e3 * sum(dev) / len(dev), "exact_fallbacks": int(fallbacks),
               "timing": "device (CUDA events per query, one query in flight)"}
        if e2e_s:
            e2 = sorted(e2e_s)
            out["e2e_p50_us"] = 1e6 * rank_at(e2, 0.5)
            out["e2e_p99_us"] = 1e6 * rank_at(e2, 0.99)
        return out


def roofline(args, res, shard_rows, metric, tc_min_batch, workload):
    """Roofline of the dominant kernel of the path that ran (reported by the
    workspace): the exact scan is HBM bound on the fp32 rows; the tensor-core
    pass is bound by the slower of its operand stream (the bf16 / int8 copy,
    plus |r|^2 for L2) and its MMA work, whichever takes longer at peak."""
    nq = res["nq"]
    kern_s = res["kern_avg_ms"] * 1e-3
    hbm_peak, hbm_kind = measured_peaks()
    label = {0: "scan", 1: "tc_bf16", 2: "tc_int8"}[res.get("path", 0)]
    traffic = committed_traffic(workload, label)
    if traffic is not None:
        traffic = traffic * shard_rows / args.n  # committed capture is of the unsharded launch
    if res.get("path", 0) in (1, 2):
        esize = 2 if res["path"] == 1 else 1
        ld = -(-args.dim // 64) * 64 if esize == 2 else -(-args.dim // 128) * 128
        bytes_ = shard_rows * ld * esize + (shard_rows * 4 if metric == 1 else 0)
        flops = 2.0 * shard_rows * args.dim * nq
        tc_peak, tc_kind = measured_bf16_peak()
        if res["path"] == 2:
            tc_peak, tc_kind = 2 * tc_peak, tc_kind + " x2 (int8 MMA rate)"
        kname = "tc_scan_kernel (filtered full pass, %s)" % ("bf16" if esize == 2 else "int8")
        if flops / (tc_peak * 1e12) >= bytes_ / (hbm_peak * 1e9):
            achieved = flops / kern_s / 1e12
            return {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
                    "frac": achieved / tc_peak, "traffic": traffic, "kernel": kname,
                    "kernel_avg_us": res["kern_avg_ms"] * 1e3,
                    "algorithmic_flops_per_launch": flops,
                    "peak_source": f"{tc_kind} bf16_tflops (dense, burst)"}
        achieved = bytes_ / kern_s / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "traffic": traffic, "kernel": kname,
                "kernel_avg_us": res["kern_avg_ms"] * 1e3, "algorithmic_bytes_per_launch": bytes_,
                "note": "bytes of the low-precision row copy the pass streams; the exact "
                        "re-score reads the fp32 rows of the certified candidates only",
                "peak_source": f"{hbm_kind} hbm_gbs"}
    groups = math.ceil(nq / 8) if nq > 8 else 1
    row_bytes = args.dim * 4 + (4 if metric in (0, 1) else 0)
    alg = shard_rows * row_bytes * groups + nq * args.dim * 4
    achieved = alg / kern_s / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
            "frac": achieved / hbm_peak, "traffic": traffic, "kernel": "scan_topk_kernel",
            "kernel_avg_us": res["kern_avg_ms"] * 1e3, "algorithmic_bytes_per_launch": alg,
            "peak_source": f"{hbm_kind} hbm_gbs"}


# ---------------------------------------------------------------------------
# IVF-flat and IVF-PQ workloads
# ---------------------------------------------------------------------------

def index_workload_config(args, nq=None, nprobe=None):
    nq = args.nq if nq is None else nq
    nprobe = args.nprobe if nprobe is None else nprobe
    base = f"{args.n}x{args.dim}_mix{args.components}_nlist{args.nlist}"
    if args.workload == "ivf":
        name = f"ivf_flat_{base}_nprobe{nprobe}_{args.metric}_top{args.k}_nq{nq}"
    else:
        name = f"ivfpq_{base}_m{args.pq_m}_nprobe{nprobe}_{args.metric}_top{args.k}_nq{nq}"
    cfg = {"workload": name, "n": args.n, "dim": args.dim, "nq": nq, "k": args.k,
           "metric": args.metric, "nlist": args.nlist, "nprobe": nprobe,
           "components": args.components,
           "parallelism": (f"listshard{args.gpus}" if args.workload == "ivfpq" and args.gpus > 1
                           and args.pq_shard == "list" else
                           f"replica{args.gpus}" if index_replicas(args, args.gpus) else
                           f"rowshard{args.gpus}"),
           "l2": "probed lists differ per query; each step streams its lists once "
                 "(no flush; lists of one batch may hit L2)"}
    if args.workload == "ivfpq":
        cfg["pq_m"] = args.pq_m
        cfg["pq_ks"] = 256
    return cfg


def build_index_data(args, nq_max, device=None, mb=None, ctx=None, shard=None, dist=None):
    """Synthetic mixture data and the index artefacts (build-time steps
    outside the timed search path).  With the library (`mb`, `ctx`) the
    partition layout / the PQ codes are built on the device by
    mans_ivf_build / mans_pq_encode (timed as `build_gpu_s`); otherwise
    (the reference arm) with torch."""
    metric = METRIC_NAMES[args.metric]
    v, q = make_mixture(args.n, args.dim, args.components, nq_max)
    if mb is not None and args.workload == "ivf":
        import torch
        cent = train_centroids(v, args.nlist)
        if dist is not None:  # one set of centroids for every shard
            ct = torch.from_numpy(cent).cuda()
            dist.broadcast(ct, 0)
            cent = ct.cpu().numpy()
        r0, r1 = shard if shard else (0, v.shape[0])
        buf = mb.VectorBuffer(ctx, v[r0:r1], id_offset=r0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        part = mb.Partition.build(ctx, buf, cent, mb.Metric(metric))
        gpu_s = time.perf_counter() - t0
        off, ids = part.layout()
        return v, q, {"centroids": cent, "offsets": off, "ids": ids, "partition": part,
                      "corpus": buf, "build_gpu_s": gpu_s,
                      "build_gpu": "mans_ivf_build: assignRows + layout + packed rows"}
    if mb is not None:
        coarse = train_centroids(v, args.nlist, seed=42)
        cb = train_pq_codebooks(v, coarse, args.pq_m)
        if dist is not None:  # one coarse quantiser and codebook set for every shard
            import torch
            ct, bt = torch.from_numpy(coarse).cuda(), torch.from_numpy(cb).cuda()
            dist.broadcast(ct, 0)
            dist.broadcast(bt, 0)
            coarse, cb = ct.cpu().numpy(), bt.cpu().numpy()
        if shard is not None and args.pq_shard == "list":
            # whole lists per rank: every rank learns every row's list from one
            # all-gather of the ranks' coarse assignments, the lists are spread
            # by size (pq.list_owners) and each rank encodes the rows of its own
            import torch
            from meltan_b200 import pq as mpq
            world, rank = dist.get_world_size(), dist.get_rank()
            bounds = [mb.row_shard(v.shape[0], world, r) for r in range(world)]
            r0, r1 = shard
            t0 = time.perf_counter()
            _, sassign = mb.pq_encode(ctx, v[r0:r1], coarse, cb, mb.Metric(metric))
            width = max(b - a for a, b in bounds)
            mine = torch.full((width,), -1, dtype=torch.int32, device="cuda")
            mine[: r1 - r0] = torch.from_numpy(sassign.astype(np.int32)).cuda()
            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine)
            assign = np.concatenate([pt.cpu().numpy()[: b - a] for pt, (a, b) in zip(parts, bounds)])
            off = np.concatenate([[0], np.cumsum(np.bincount(assign, minlength=args.nlist))])
            flat = np.argsort(assign, kind="stable").astype(np.uint32)
            owner = mpq.list_owners(np.diff(off), world)
            soff, sflat, spos = mb.IVFPQIndex.shard_lists_by_list(off, flat, owner == rank)
            mcodes, massign = mb.pq_encode(ctx, v[sflat], coarse, cb, mb.Metric(metric))
            gpu_s = time.perf_counter() - t0
            if not np.array_equal(massign, assign[sflat]):
                raise RuntimeError("list shard: the re-encoded rows changed lists")
            codes = np.zeros((v.shape[0], args.pq_m), np.uint8)
            codes[sflat] = mcodes
            return v, q, {"coarse": coarse, "codebooks": cb, "codes": codes,
                          "offsets": soff, "lists": sflat, "positions": spos,
                          "build_gpu_s": gpu_s,
                          "build_gpu": "mans_pq_encode: every rank's rows (assignment), then "
                                       "the rows of this rank's lists (codes)"}
        if shard is not None:
            # this rank's rows; list entries carry their positions in the
            # global lists (earlier shards' entries of a list come first)
            import torch
            r0, r1 = shard
            t0 = time.perf_counter()
            scodes, sassign = mb.pq_encode(ctx, v[r0:r1], coarse, cb, mb.Metric(metric))
            gpu_s = time.perf_counter() - t0
            cnt = torch.from_numpy(np.bincount(sassign, minlength=args.nlist)).cuda()
            allc = [torch.empty_like(cnt) for _ in range(dist.get_world_size())]
            dist.all_gather(allc, cnt)
            before = sum(c.cpu().numpy() for c in allc[:dist.get_rank()]) if dist.get_rank() else \
                np.zeros(args.nlist, np.int64)
            order = np.argsort(sassign, kind="stable")
            soff = np.concatenate([[0], np.cumsum(np.bincount(sassign, minlength=args.nlist))])
            lists_of = np.repeat(np.arange(args.nlist), np.diff(soff))
            spos = (before[lists_of] + np.arange(len(order)) - soff[lists_of]).astype(np.uint32)
            codes = np.zeros((v.shape[0], args.pq_m), np.uint8)
            codes[r0:r1] = scodes
            return v, q, {"coarse": coarse, "codebooks": cb, "codes": codes,
                          "offsets": soff.astype(np.int64), "lists": (order + r0).astype(np.uint32),
                          "positions": spos, "build_gpu_s": gpu_s,
                          "build_gpu": "mans_pq_encode of this rank's rows"}
        t0 = time.perf_counter()
        codes, assign = mb.pq_encode(ctx, v, coarse, cb, mb.Metric(metric))
        gpu_s = time.perf_counter() - t0
        flat = np.argsort(assign, kind="stable").astype(np.uint32)
        off = np.concatenate([[0], np.cumsum(np.bincount(assign, minlength=args.nlist))])
        return v, q, {"coarse": coarse, "codebooks": cb, "codes": codes,
                      "offsets": off.astype(np.int64), "lists": flat, "build_gpu_s": gpu_s,
                      "build_gpu": "mans_pq_encode: nearestCoarseCentroid + residual codes"}
    if args.workload == "ivf":
        cent, assign = train_partition(v, args.nlist, metric, device=device)
        order = np.argsort(assign, kind="stable").astype(np.uint32)
        off = np.concatenate([[0], np.cumsum(np.bincount(assign, minlength=args.nlist))])
        return v, q, {"centroids": cent, "offsets": off.astype(np.int64), "ids": order}
    coarse, cb, codes, off, flat = train_ivfpq(v, args.nlist, args.pq_m, metric=metric,
                                               device=device)
    return v, q, {"coarse": coarse, "codebooks": cb, "codes": codes, "offsets": off,
                  "lists": flat}


def probed_list_rows(args, art, q, distinct=False):
    """Rows of the lists each query probes (the per-query unit of the
    roofline), or with `distinct` the rows of the union of the batch's probed
    lists (what a batch that reads each probed list once must read):
    top-nprobe centroids by the search's own key, with torch."""
    import torch
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    qt = torch.from_numpy(q).to(dev)
    if args.workload == "ivf":
        c = torch.from_numpy(art["centroids"]).to(dev)
        off = torch.from_numpy(art["offsets"]).to(dev)
        sizes = off[1:] - off[:-1]
        dots = qt @ c.T
        cn = (c * c).sum(1)
        metric = METRIC_NAMES[args.metric]
        key = -dots if metric == 2 else (cn - 2 * dots if metric == 1 else
                                         -dots / cn.clamp(min=1e-20).sqrt())
    else:
        c = torch.from_numpy(art["coarse"]).to(dev)
        off = torch.from_numpy(art["offsets"]).to(dev)
        sizes = off[1:] - off[:-1]
        key = torch.cdist(qt, c)
    top = torch.topk(key, min(args.nprobe, key.shape[1]), dim=1, largest=False).indices
    if distinct:
        return int(sizes[torch.unique(top)].sum().item())
    return sizes[top].sum(1).cpu().numpy().astype(np.int64)


def index_searcher(args, v, art):
    """One query through the restated reference search (single-threaded, as
    IVFFlatSearch.scanProbedLists / _IVFPQIndex.search run)."""
    import oracle as O
    metric = METRIC_NAMES[args.metric]
    if args.workload == "ivf":
        order = art["ids"]
        off = art["offsets"]
        packed = v[order]
        pn = O.row_norms(packed)

        def one(x):
            O.ivf_search(art["centroids"], packed, pn, order, off, x, args.k, args.nprobe, metric)
    else:
        def one(x):
            O.ivfpq_search(art["coarse"], art["codebooks"], art["codes"], art["offsets"],
                           art["lists"], x, args.k, args.nprobe, metric)
    return one


def cpu_index_qps(args, v, q, art, seconds):
    """The restated reference search on a bounded sample of queries."""
    one = index_searcher(args, v, art)
    one(q[0])
    t0 = time.perf_counter()
    done = 0
    while True:
        one(q[done % len(q)])
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return done / el, done


def measure_index(torch, ws, search_dev, search_host, q, kout, steps, warmup, with_clocks,
                  barrier=None):
    """Device-timed steps (inputs resident) and end-to-end steps through the
    host C ABI (pinned buffers), as Runner.measure does for the flat scan.
    Row shards (``search_host`` None): ``search_dev`` returns the merged
    packed block and the end-to-end step copies the queries in and the block
    out around it; ``barrier`` lines the ranks up around the timed loops."""
    if q.ndim == 2:
        q = q[None]
    pool, nq = q.shape[0], q.shape[1]
    dq_pool = torch.from_numpy(np.ascontiguousarray(q)).cuda()
    dq = dq_pool[0]
    sync = barrier or torch.cuda.synchronize
    od = torch.empty((nq, kout), dtype=torch.float32, device="cuda")
    oi = torch.empty((nq, kout), dtype=torch.int32, device="cuda")
    oc = torch.empty((nq,), dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def step(src=dq):
        return search_dev(src.data_ptr(), nq, od.data_ptr(), oi.data_ptr(), oc.data_ptr(), sp)

    for _ in range(max(3, warmup)):
        last = step()
    ws.check(sp)
    ws.stats()
    ws.set_timing(True)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    clocks = ClockSampler(torch.cuda.current_device()) if with_clocks else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    sync()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        ev[i][0].record(stream)
        last = step(dq_pool[i % pool])
        ev[i][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    sync()
    clock_info = clocks.stop() if clocks else None
    ws.check(sp)
    kern_ms, kern_launches, total_launches = ws.stats()
    ws.set_timing(False)
    total_ms = t0.elapsed_time(t1)
    step_ms = [x.elapsed_time(y) for x, y in ev]
    # the device outputs above are those of batch (steps - 1) % pool, which
    # the last end-to-end step searches too
    hq_pool = torch.from_numpy(np.ascontiguousarray(q)).pin_memory()
    hd = torch.empty((nq, kout), dtype=torch.float32).pin_memory()
    hi = torch.empty((nq, kout), dtype=torch.int32).pin_memory()
    hc = torch.empty((nq,), dtype=torch.int32).pin_memory()
    if search_host is None:
        from meltan_b200 import shard as _shard
        d, i, c = _shard.block_views(last, nq, kout)
        dev_out = (d.cpu().numpy(), i.cpu().numpy(), c.cpu().numpy())
        dq2 = torch.empty_like(dq)
        hblk = torch.empty_like(last, device="cpu").pin_memory()

        def e2e(j):
            dq2.copy_(hq_pool[j % pool], non_blocking=True)
            r = step(dq2)
            hblk.copy_(r, non_blocking=True)
            stream.synchronize()
            bd, bi, bc = _shard.block_views(hblk, nq, kout)
            hd.copy_(bd)
            hi.copy_(bi)
            hc.copy_(bc)
    else:
        dev_out = (od.cpu().numpy(), oi.cpu().numpy(), oc.cpu().numpy())

        def e2e(j):
            search_host(hq_pool[j % pool].data_ptr(), nq, hd.data_ptr(), hi.data_ptr(),
                        hc.data_ptr())

    for j in range(max(3, warmup)):
        e2e(j)
    sync()
    e2e_times = []
    for j in range(steps):
        t = time.perf_counter()
        e2e(j)
        e2e_times.append(time.perf_counter() - t)
    ok = bool(np.array_equal(dev_out[2], hc.numpy()) and np.array_equal(dev_out[1], hi.numpy())
              and np.array_equal(dev_out[0], hd.numpy()))
    return {"nq": nq, "steps": steps, "pool": pool, "total_ms": total_ms,
            "e2e_ms": 1e3 * sum(e2e_times),
            "kern_avg_ms": kern_ms / max(kern_launches, 1), "kern_launches": kern_launches,
            "launches": total_launches, "p50_ms": p50(step_ms), "e2e_p50_s": p50(e2e_times),
            "clocks": clock_info, "ok": ok, "kout": kout}


def index_roofline(args, res, list_rows, distinct_rows=None):
    """HBM roofline of the timed kernel: the list scan (IVF-flat) or the ADC
    scoring kernel (IVF-PQ), with the bytes of the probed lists: IVF-flat
    rows (d*4) + norm (4) + id (4); IVF-PQ code (m) + id (4).  The IVF-flat
    batch scan reads every probed list once for all the queries that probe
    it, so its bytes are those of the distinct probed lists; the other
    kernels count each query's lists."""
    peak, src = measured_peaks()
    per_row = args.dim * 4 + 8 if args.workload == "ivf" else args.pq_m + 4
    alg = float(list_rows.sum()) * per_row
    batch_scan = args.workload == "ivf" and distinct_rows is not None and \
        res["launches"] != res["steps"]
    if batch_scan:
        alg = float(distinct_rows) * per_row
    # One library launch per step: the one-launch IVF-flat search, whose
    # timed kernel also scores the centroids (rows + norms, once per launch).
    one_launch = args.workload == "ivf" and res["launches"] == res["steps"]
    if one_launch:
        alg += float(args.nlist) * (args.dim * 4 + 4)
        kernel = "ivf_probe_kernel (centroid scan + top-nprobe + probed lists, one launch)"
    else:
        kernel = ("ivf_seg_scan_kernel (distinct probed lists, read once per batch)"
                  if batch_scan and args.k <= 32 else
                  "scan_topk_kernel (probed lists)" if args.workload == "ivf" else "pq_adc_kernel")
    kern_s = res["kern_avg_ms"] * 1e-3
    achieved = alg / kern_s / 1e9 if kern_s > 0 else 0.0
    wl = index_workload_config(args, res["nq"])["workload"]
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": committed_traffic(wl, "probe" if one_launch else
                                         "list_scan" if args.workload == "ivf" else "adc"),
            "kernel": kernel, "kernel_avg_us": 1e3 * res["kern_avg_ms"],
            "algorithmic_bytes_per_launch": alg,
            "per_query_bytes_per_launch": float(list_rows.sum()) * per_row,
            "peak_source": f"{src} hbm_gbs (STREAM copy)"}


def index_args(base, workload):
    """The IVF-flat or IVF-PQ workload with its
    BASELINE defaults, for the extra lines of the default run."""
    import copy
    a = copy.copy(base)
    a.workload = workload
    a.k = 10
    if workload == "ivf":
        a.n, a.dim, a.metric, a.nq = 1_000_000, 384, "cosine", 1
        a.nlist, a.nprobe, a.components = 1024, 8, 1024
    else:
        a.n, a.dim, a.metric, a.nq = 10_000_000, 128, "l2", 1024
        a.nlist, a.nprobe, a.components, a.pq_m = 4096, 32, 4096, 16
    return a


def index_session(args, torch, mb, lib, world, rank, dist, cases):
    """Builds the index of args.workload on this rank (its shard for N > 1)
    and measures each case (nq, nprobe, steps, warmup, with_clocks).  Returns
    (results, build seconds, host data for the CPU baselines); the device
    objects are released before returning."""
    metric = METRIC_NAMES[args.metric]
    t_build = time.perf_counter()
    ctx = mb.Context(torch.cuda.current_device())
    # N > 1: IVF-PQ shards its rows or lists over the ranks (shared centroids
    # and codebooks, list positions, per-rank blocks gathered and resolved into
    # the unsharded result); IVF-flat does the same with --ivf-layout shard,
    # and by default keeps a full replica per rank, each rank searching its
    # own queries.
    replicas = index_replicas(args, world)
    ivf_sharded = world > 1 and not replicas
    # each case cycles through a pool of distinct query batches (per rank for
    # replicas); queries are drawn after the database, so their number leaves
    # the database unchanged
    q_need = max(c[0] * query_pool(c[0]) * (world if replicas else 1) for c in cases)
    shard = mb.row_shard(args.n, world, rank) if ivf_sharded else None
    v, q_all, art = build_index_data(args, q_need, mb=mb, ctx=ctx, shard=shard,
                                     dist=dist if ivf_sharded else None)
    ws = mb.Workspace(ctx)
    L = lib
    kout = min(args.k, mb.MAX_TOP_K)
    barrier = None
    sharded = None
    if ivf_sharded and args.workload == "ivfpq":
        ix = mb.IVFPQIndex(ctx, art["coarse"], art["codebooks"], art["codes"],
                           (art["offsets"], art["lists"]), metric=mb.Metric(metric),
                           list_positions=art["positions"])
        index = ix
        sharded = mb.ShardedIVFPQSearch(ctx, ix, world, dist)
        bufs_by_nq = {}

        def dev_fn(nprobe):
            def f(qp, nq, d, i, c, s):
                b = bufs_by_nq.setdefault(nq, sharded.buffers(nq, args.k))
                return sharded.search_device(ws, qp, nq, args.k, nprobe, b, s)
            return f

        def host_fn(nprobe):
            return None

        def barrier():
            dist.barrier()
            torch.cuda.synchronize()
    elif ivf_sharded:
        part = art["partition"]
        index = part
        sharded = mb.ShardedIVFSearch(ctx, part, world, dist, transport=args.transport, rank=rank)
        bufs_by_nq = {}

        def dev_fn(nprobe):
            def f(qp, nq, d, i, c, s):
                b = bufs_by_nq.setdefault(nq, sharded.buffers(nq, kout))
                return sharded.search_device(ws, qp, nq, args.k, nprobe, metric, b, s)
            return f

        def host_fn(nprobe):
            return None

        def barrier():
            dist.barrier()
            torch.cuda.synchronize()
    elif args.workload == "ivf":
        part = art["partition"]
        index = part

        def dev_fn(nprobe):
            return lambda qp, nq, d, i, c, s: mb.IVFFlatSearch.search_device(
                ctx, part, ws, qp, nq, args.k, nprobe, metric, d, i, c, s)

        def host_fn(nprobe):
            return lambda qp, nq, d, i, c: mb.check(L.mans_ivf_search(
                ctx.handle, part.handle, C.c_void_p(qp), nq, args.dim, args.k, nprobe, metric,
                C.c_void_p(d), C.c_void_p(i), C.c_void_p(c)))
    else:
        ix = mb.IVFPQIndex(ctx, art["coarse"], art["codebooks"], art["codes"],
                           (art["offsets"], art["lists"]), metric=mb.Metric(metric))
        index = ix

        def dev_fn(nprobe):
            return lambda qp, nq, d, i, c, s: ix.search_device(ws, qp, nq, args.k, nprobe, d, i,
                                                               c, s)

        def host_fn(nprobe):
            return lambda qp, nq, d, i, c: mb.check(L.mans_ivfpq_search(
                ctx.handle, ix.handle, C.c_void_p(qp), nq, args.dim, args.k, nprobe,
                C.c_void_p(d), C.c_void_p(i), C.c_void_p(c)))
    build_s = time.perf_counter() - t_build

    results = []
    for nq, nprobe, steps, warmup, with_clocks in cases:
        saved = args.nprobe
        args.nprobe = nprobe
        try:
            pool = query_pool(nq)
            off = rank * nq * pool if replicas else 0
            q = q_all[off:off + nq * pool].reshape(pool, nq, args.dim)
            r = measure_index(torch, ws, dev_fn(nprobe), host_fn(nprobe), q, kout, steps, warmup,
                              with_clocks, barrier=barrier if not replicas else
                              (lambda: (dist.barrier(), torch.cuda.synchronize())))
            if world > 1:
                t = torch.tensor([r["total_ms"], r["e2e_ms"]], dtype=torch.float64,
                                 device="cuda")
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                r["total_ms"], r["e2e_ms"] = t.tolist()
            r["nprobe"] = nprobe
            # bytes per launch: the mean over the pool's batches
            rows = np.float64(np.mean([np.sum(probed_list_rows(args, art, qb)) for qb in q]))
            drows = (np.float64(np.mean([np.sum(probed_list_rows(args, art, qb, distinct=True))
                                         for qb in q]))
                     if args.workload == "ivf" else None)
            r["roofline"] = index_roofline(args, r, rows, drows)
            r["workload"] = index_workload_config(args, nq, nprobe)["workload"]
            r["config"] = index_workload_config(args, nq, nprobe)
            results.append(r)
        finally:
            args.nprobe = saved
    if sharded is not None:
        barrier()  # every rank is done with the peers' buffers
        if hasattr(sharded, "close"):
            sharded.close()
    ws.close()
    index.close()
    if "corpus" in art:
        art["corpus"].close()
    ctx.close()
    torch.cuda.synchronize()
    host = {"v": v, "q": q_all, "art": {kk: vv for kk, vv in art.items()
                                        if kk not in ("partition", "corpus")},
            "build_gpu_s": art.get("build_gpu_s"), "build_gpu": art.get("build_gpu")}
    return results, build_s, host


def index_replicas(args, world):
    """IVF-flat at N > 1 runs as replicas unless --ivf-layout shard."""
    return world > 1 and args.workload == "ivf" and args.ivf_layout == "replica"


def query_pool(nq):
    """Distinct query batches a timed case cycles through: 64 single queries,
    4 batches up to 256 queries, 2 larger batches."""
    return 64 if nq == 1 else (4 if nq <= 256 else 2)


def index_entry(args, r, world, ivf_sharded):
    """One measured case as a JSON object (the main line's keys)."""
    return {"workload": r["workload"], "nq": r["nq"], "nprobe": r["nprobe"],
            "steps": r["steps"], "metric": "queries_per_sec",
            "value": (1 if ivf_sharded else world) * r["nq"] * r["steps"] / (r["total_ms"] * 1e-3),
            "unit": "queries/s", "ms_per_step": r["total_ms"] / r["steps"],
            "p50_us": 1e3 * r["p50_ms"],
            "e2e": {"value": (1 if ivf_sharded else world) * r["nq"] * r["steps"] /
                             (r["e2e_ms"] * 1e-3), "unit": "queries/s",
                    "p50_us": 1e6 * r["e2e_p50_s"],
                    "h2d_bytes_per_step": r["nq"] * args.dim * 4,
                    "d2h_bytes_per_step": r["nq"] * r["kout"] * 8 + r["nq"] * 4},
            "gpu_launches": int(r["launches"]), "roofline": r["roofline"],
            "scaling": "strong" if ivf_sharded or world == 1 else "weak",
            "distinct_batches_timed": r["pool"],
            "config": r["config"], "e2e_matches_device_path": r["ok"],
            "dtype": "f32" if args.workload == "ivf" else "f32 (u8 codes)"}


def index_cpu_baseline(args, host, seconds, threads):
    """The restated reference search on a bounded sample of queries: one
    thread per query as the reference runs it; with threads > 1 the queries
    are spread over that many host threads (the ctypes calls release the
    GIL)."""
    one = index_searcher(args, host["v"], host["art"])
    q = host["q"]
    one(q[0])
    if threads <= 1:
        qps, done = cpu_index_qps(args, host["v"], q, host["art"], seconds)
        kind = ("IVFFlatSearch.scanProbedLists restated" if args.workload == "ivf"
                else "_IVFPQIndex.search restated (coarse BoundedSortedList, sequential ADC, "
                     "newest-first merge)")
        return {"value": qps, "unit": "queries/s", "cores": 1, "kind": "port",
                "sample": f"{done} single-query searches (~{seconds:.0f} s), nprobe "
                          f"{args.nprobe}, one thread; {kind}"}
    from concurrent.futures import ThreadPoolExecutor
    done = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        while True:
            idx = [(done + i) % len(q) for i in range(threads)]
            list(ex.map(lambda j: one(q[j]), idx))
            done += threads
            el = time.perf_counter() - t0
            if el >= seconds:
                break
    return {"value": done / el, "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{done} queries (~{seconds:.0f} s), nprobe {args.nprobe}, queries spread "
                      f"over {threads} host threads, each query single-threaded as the "
                      f"reference runs it; "
                      + ("IVFFlatSearch.scanProbedLists restated" if args.workload == "ivf"
                         else "_IVFPQIndex.search restated")}


def index_cases(args):
    """(nq, nprobe, steps, warmup, clocks) of the main line and its extras."""
    main = (args.nq, args.nprobe, args.steps, args.warmup, True)
    if args.no_also:
        return [main]
    if args.workload == "ivf":
        extra = [(1, p) for p in (4, 32) if p != args.nprobe] + [(256, args.nprobe)]
    else:
        extra = [(256, args.nprobe)]
    return [main] + [(nq2, p2, max(20, min(args.steps, int(20000 / nq2))), 5, False)
                     for nq2, p2 in extra]


def run_index(args, torch, mb, lib, world, rank, dist):
    ivf_sharded = world > 1 and not index_replicas(args, world)
    results, build_s, host = index_session(args, torch, mb, lib, world, rank, dist,
                                           index_cases(args))
    if rank == 0:
        res = results[0]
        line = {
            "metric": "queries_per_sec",
            "value": (1 if ivf_sharded else world) * args.nq * args.steps / (res["total_ms"] * 1e-3),
            "unit": "queries/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["total_ms"] / args.steps, "p50_us": 1e3 * res["p50_ms"],
            "higher_is_better": True,
            "scaling": "strong" if ivf_sharded or world == 1 else "weak",
            "vs_baseline": None,
            "distinct_batches_timed": res["pool"],
            "dtype": "f32" if args.workload == "ivf" else "f32 (u8 codes)",
            "data": index_data_note(args, build_s),
            "config": index_workload_config(args),
            "roofline": res["roofline"],
            "e2e": {"value": (1 if ivf_sharded else world) * args.nq * args.steps /
                             (res["e2e_ms"] * 1e-3), "unit": "queries/s",
                    "p50_us": 1e6 * res["e2e_p50_s"],
                    "h2d_bytes_per_step": args.nq * args.dim * 4,
                    "d2h_bytes_per_step": args.nq * res["kout"] * 8 + args.nq * 4},
            "gpu_launches": int(res["launches"]),
            "clocks": res["clocks"],
            "e2e_matches_device_path": res["ok"],
            "build": {"device_s": host["build_gpu_s"], "what": host["build_gpu"],
                      "rows": args.n},
            "also": [index_entry(args, r, world, ivf_sharded) for r in results[1:]],
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = index_cpu_baseline(args, host, args.cpu_seconds, 1)
            if args.workload == "ivfpq":
                line["cpu_baseline_all_cores"] = index_cpu_baseline(
                    args, host, args.cpu_seconds, os.cpu_count() or 1)
        print(json.dumps(line), flush=True)


def index_data_note(args, build_s):
    return (f"synthetic {args.components}-component Gaussian mixture (sigma 0.3, "
            f"L2-normalised; numpy default_rng(0) below 2^26 elements, torch CUDA Philox "
            f"seed 0 above); index trained with torch (build {build_s:.0f} s, outside the "
            f"timed region)")


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", local))

    import meltan_b200 as mb
    from meltan_b200._lib import lib

    if args.workload != "flat":
        run_index(args, torch, mb, lib(), world, rank, dist)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    metric = METRIC_NAMES[args.metric]
    also_nq = [] if args.no_also else [
        x for x in (int(t) for t in args.also_nq.split(",") if t.strip()) if x != args.nq]
    # the nq = 1 line times distinct queries: step i searches query i % pool
    pool = max(LATENCY_QUERIES, args.steps) if args.nq == 1 else 1
    v, q_all = make_data(args.n, args.dim, max([args.nq * pool, LATENCY_QUERIES] + also_nq))
    r0, r1 = mb.row_shard(args.n, world, rank)
    ctx = mb.Context(local)
    tc_min = args.tc_min_batch
    ctx.set_tensor_core_batch(tc_min)
    buf = mb.VectorBuffer(ctx, v[r0:r1], id_offset=r0)
    ws = mb.Workspace(ctx)
    R = Runner(args, torch, mb, lib(), ctx, buf, ws, world, rank, dist, metric)
    main_res = R.measure(q_all[:args.nq * pool].reshape(pool, args.nq, args.dim), args.steps,
                         args.warmup, with_clocks=True)
    latency = R.latency(q_all[:LATENCY_QUERIES]) if args.nq == 1 else None
    also = []
    for nq2 in also_nq:
        st = max(20, min(args.steps, int(20000 / nq2)))
        also.append(R.measure(q_all[:nq2][None], st, 5, with_clocks=False))
    fp32 = None
    if not args.no_also and args.nq == 1:
        # the exact fp32 CUDA-core scan alone (tensor-core path off): the
        # single-query scan of the fp32 rows the north star's HBM target names
        ctx.set_tensor_core_batch(0)
        st = max(20, min(args.steps, 200))
        fp32 = R.measure(q_all[:st].reshape(st, 1, args.dim), st, 5, with_clocks=False)
        fp32["latency"] = R.latency(q_all[:LATENCY_QUERIES])
        ctx.set_tensor_core_batch(tc_min)
    ws.close()
    buf.close()
    ctx.close()

    index_results = []
    if not args.no_also and not args.no_index and args.n == 1_000_000 and args.dim == 384:
        # BASELINE.json configs[2] (IVF-flat) and configs[3] (IVF-PQ) on the
        # same run, each with its own roofline and CPU baseline
        for wl in ("ivf", "ivfpq"):
            ia = index_args(args, wl)
            if wl == "ivf":
                cases = [(1, 8, max(20, min(args.steps, 200)), 5, False),
                         (1, 4, max(20, min(args.steps, 200)), 5, False),
                         (1, 32, max(20, min(args.steps, 200)), 5, False),
                         (256, 8, max(20, min(args.steps, 80)), 5, False)]
            else:
                cases = [(1024, 32, max(20, min(args.steps, 20)), 5, False)]
            res, build_s, host = index_session(ia, torch, mb, lib(), world, rank, dist, cases)
            index_results.append((ia, res, build_s, host))

    if rank == 0:
        workload = workload_config(args)["workload"]
        res = main_res
        line = {
            "metric": "queries_per_sec",
            "value": args.nq * args.steps / (res["total_ms"] * 1e-3),
            "unit": "queries/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": res["total_ms"] / args.steps,
            "p50_us": 1e3 * (latency["p50_us"] / 1e3 if latency else res["p50_ms"]),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (numpy default_rng(0) Gaussian rows, L2-normalised)",
            "config": workload_config(args),
            "roofline": roofline(args, res, r1 - r0, metric, tc_min, workload),
            "e2e": {"value": args.nq * args.steps / (res["e2e_ms"] * 1e-3), "unit": "queries/s",
                    "p50_us": 1e6 * res["e2e_p50_s"],
                    "h2d_bytes_per_step": args.nq * args.dim * 4,
                    "d2h_bytes_per_step": args.nq * res["kout"] * 8 + args.nq * 4},
            "gpu_launches": int(res["launches"]),
            "clocks": res["clocks"],
            "e2e_matches_device_path": res["ok"],
            "distinct_queries_timed": res["distinct_batches"] * args.nq,
            "exact_fallbacks_last_step": res["fallbacks_last_step"],
            "stages_us": dict(res["stages_us"], note=STAGES_NOTE),
        }
        if latency:
            line["p50_steps_us"] = 1e3 * res["p50_ms"]
            line["latency"] = latency
        line["also"] = []
        for r in also:
            wl = workload_config(args, r["nq"])["workload"]
            line["also"].append(flat_entry(args, r, r1 - r0, metric, tc_min, wl))
        if fp32 is not None:
            entry = flat_entry(args, fp32, r1 - r0, metric, 0,
                               workload_config(args, 1)["workload"] + "_fp32scan")
            entry["path"] = "exact fp32 CUDA-core scan (tensor-core path off)"
            entry["latency"] = fp32["latency"]
            entry["p50_us"] = fp32["latency"]["p50_us"]
            line["also"].append(entry)
        for ia, results, build_s, host in index_results:
            for i, r in enumerate(results):
                e = index_entry(ia, r, world, world > 1 and not index_replicas(ia, world))
                e["data"] = index_data_note(ia, build_s)
                if i == 0:
                    e["build"] = {"device_s": host["build_gpu_s"], "what": host["build_gpu"],
                                  "rows": ia.n}
                line["also"].append(e)
        if world == 1 and not args.no_cpu_baseline:
            add_cpu_baselines(args, line, also, fp32, index_results, v, q_all, metric)
        print(json.dumps(line), flush=True)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


LATENCY_QUERIES = 200
STAGES_NOTE = ("per step, device time of each stage (CUDA events around its kernels on the "
               "launching stream, 20 extra steps outside the timed region, max over ranks); "
               "merge = slot merge, or shard exchange + merge")


def flat_entry(args, r, shard_rows, metric, tc_min, wl):
    return {"workload": wl, "nq": r["nq"], "steps": r["steps"],
            "metric": "queries_per_sec",
            "value": r["nq"] * r["steps"] / (r["total_ms"] * 1e-3), "unit": "queries/s",
            "ms_per_step": r["total_ms"] / r["steps"], "p50_us": 1e3 * r["p50_ms"],
            "e2e_value": r["nq"] * r["steps"] / (r["e2e_ms"] * 1e-3),
            "e2e_p50_us": 1e6 * r["e2e_p50_s"], "gpu_launches": int(r["launches"]),
            "roofline": roofline(args, r, shard_rows, metric, tc_min, wl),
            "e2e_matches_device_path": r["ok"],
            "distinct_queries_timed": r["distinct_batches"] * r["nq"],
            "exact_fallbacks_last_step": r["fallbacks_last_step"],
            "stages_us": r["stages_us"],
            "config": workload_config(args, r["nq"])}


def add_cpu_baselines(args, line, also, fp32, index_results, v, q_all, metric):
    """The reference's CPU routes, timed on bounded samples on this host:
    ParallelFlatScan for single queries (all cores, and one core), the
    BoundedExactScan batch route for batches, scanProbedLists (one thread per
    query, as the reference runs it) for IVF-flat, _IVFPQIndex.search for
    IVF-PQ (one thread, and queries spread over all cores)."""
    batch_base = None
    if args.n >= 16384 and (args.nq > 1 or any(r["nq"] > 1 for r in also)):
        # the reference's CPU route for batches (BoundedExactScan per query)
        bq, bused, bdone, buse_ref = cpu_batch_qps(v, q_all, args.k, metric, args.cpu_seconds)
        batch_base = {
            "value": bq, "unit": "queries/s", "cores": bused, "kind": "port",
            "sample": f"{bdone} queries (~{args.cpu_seconds:.0f} s) through the batch "
                      f"route: BoundedExactScan restated (int8 prefilter, provable "
                      f"lower bounds, fp32 rescore) per query, queries in parallel over "
                      f"{bused} threads; inner loops "
                      f"{'reference dots.c' if buse_ref else 'restated dots.c'}"}
        for entry, r in zip(line["also"], also):
            if r["nq"] > 1:
                entry["cpu_baseline"] = batch_base
    if args.nq > 1 and batch_base is not None:
        line["cpu_baseline"] = batch_base
        return_single = False
    else:
        return_single = True
    if return_single or fp32 is not None:
        qps, used, done, use_ref = cpu_reference_qps(v, q_all, args.k, metric, args.cpu_seconds)
        single = {
            "value": qps, "unit": "queries/s", "cores": used, "kind": "port",
            "sample": f"{done} single-query scans of the full {args.n}x{args.dim} corpus "
                      f"(~{args.cpu_seconds:.0f} s), {used} threads; ParallelFlatScan restated, "
                      f"inner loop {'reference dots.c' if use_ref else 'restated dots.c'}"}
        qps1, _, done1, _ = cpu_reference_qps(v, q_all, args.k, metric, args.cpu_seconds / 2,
                                              cores=1)
        one_core = {
            "value": qps1, "unit": "queries/s", "cores": 1, "kind": "port",
            "sample": f"{done1} single-query scans (~{args.cpu_seconds / 2:.0f} s) on one core "
                      f"(ParallelFlatScan with one slice)"}
        if return_single:
            line["cpu_baseline"] = single
            line["cpu_baseline_1core"] = one_core
        for entry in line["also"]:
            if entry["workload"].endswith("_fp32scan"):
                entry["cpu_baseline"] = single
                entry["cpu_baseline_1core"] = one_core
    for ia, results, build_s, host in index_results:
        for entry, r in zip([e for e in line["also"] if e["workload"] in
                             {x["workload"] for x in results}], results):
            saved = ia.nprobe
            ia.nprobe = r["nprobe"]
            try:
                secs = args.cpu_seconds if r["nprobe"] in (8, 32) else args.cpu_seconds / 2
                entry["cpu_baseline"] = index_cpu_baseline(ia, host, secs, 1)
                if ia.workload == "ivfpq":
                    entry["cpu_baseline_all_cores"] = index_cpu_baseline(
                        ia, host, secs, os.cpu_count() or 1)
            finally:
                ia.nprobe = saved


if __name__ == "__main__":
    main()
