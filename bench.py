"""Benchmark of the exact-kNN hot path on B200 (one process per GPU).

Default workload (north star target, BASELINE.json config 4 at k=10):
  exact inner-product kNN, base 10,000,000 x 768 fp32 unit-norm N(0,1) rows,
  10,000 unit-norm queries, k = 10; the base is row-sharded over the ranks
  (strong scaling: the same 10M rows at every GPU count) and the per-rank
  top-k lists are merged by one NCCL all-gather plus an on-device merge.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1)

Reported on one JSON line (rank 0):
  value       QPS with queries resident in HBM (device-timed, max over ranks)
  e2e         QPS through the public API with host queries/results, i.e.
              H2D of the queries and D2H of ids+distances inside the timing
  roofline    the dominant kernel's achieved TFLOP/s (2*nq*n*d per launch over
              its CUDA-event time) against the tensor-core rate of the pass
              it runs, derived from the measured bf16 peak in
              MEASURED_PEAKS.json
  cpu_baseline the CPU oracle (C++ restatement of the reference's
              FlatIndex::search_batch, all host threads) on a query sample
--impl reference times only that CPU implementation (rank 0; other ranks exit).
Data are synthetic (seeded torch generators); the base (30.7 GB) is larger
than L2, so no flush is needed between steps.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (metric, n, dim, nq, k, generator)
    "c4k10": ("ip", 10_000_000, 768, 10_000, 10, "unit"),
    "c4k100": ("ip", 10_000_000, 768, 10_000, 100, "unit"),
    "c1": ("ip", 100_000, 384, 1_000, 10, "unit"),
    "c2": ("l2", 1_000_000, 128, 1_000, 10, "sift"),
    "c2q64": ("l2", 1_000_000, 128, 64, 10, "sift"),
    "c2q1": ("l2", 1_000_000, 128, 1, 10, "sift"),
    "c5": ("l2", 100_000_000, 96, 10_000, 10, "mixture"),
    # config 5's distribution on a tenth of the rows (quick comparisons, ncu)
    "c5s": ("l2", 10_000_000, 96, 10_000, 10, "mixture"),
    # profiling case for ncu: config 4's distribution and rows per split on 1/38 of the rows
    "prof": ("ip", 262_144, 768, 18_944, 10, "unit"),
    # config 4's 40 query groups on the profiling case's rows (short splits)
    "prof40": ("ip", 262_144, 768, 10_000, 10, "unit"),
    # profiling case for ncu: config 5's distribution on 2M rows (2.8 GB on the device)
    "prof5": ("l2", 2_000_000, 96, 10_000, 10, "mixture"),
    # the same rows with 74 query groups over 2 splits: lists as long as config 5's
    "prof5l": ("l2", 2_000_000, 96, 18_944, 10, "mixture"),
    # PQ ADC scan (config 3): m=16 x 256 centroids trained on a 100k sample
    "c3": ("pq-l2", 1_000_000, 128, 1_000, 10, "sift"),
}
WORKLOAD_TEXT = {
    "c4k10": "exact IP kNN, base 10,000,000x768 unit-norm N(0,1), 10,000 queries, k=10 (config 4 at k=10)",
    "c4k100": "exact IP kNN, base 10,000,000x768 unit-norm N(0,1), 10,000 queries, k=100 (config 4)",
    "c1": "exact IP kNN, base 100,000x384 unit-norm N(0,1), 1,000 queries, k=10 (config 1)",
    "c2": "exact L2 kNN, base 1,000,000x128 SIFT-like integer mixture, 1,000 queries, k=10 (config 2)",
    "c2q64": "exact L2 kNN, base 1,000,000x128 SIFT-like, 64 queries, k=10 (config 2)",
    "c2q1": "exact L2 kNN, base 1,000,000x128 SIFT-like, 1 query, k=10 (config 2)",
    "c5": "exact L2 kNN, base 100,000,000x96 Gaussian mixture, one 10,000-query batch, k=10 (config 5)",
    "c5s": ("config 5's distribution on a tenth of the rows: exact L2 kNN, base 10,000,000x96 Gaussian "
            "mixture, 10,000 queries, k=10"),
    "prof": ("profiling case: exact IP kNN, base 262,144x768 unit-norm N(0,1), 18,944 queries, k=10 "
             "(2.8 GB on the device; 131k rows per split, as config 4 has 270k)"),
    "prof40": ("profiling case: exact IP kNN, base 262,144x768 unit-norm N(0,1), 10,000 queries (config 4's "
               "40 query groups, 37 splits of 28 tiles), k=10 (2.8 GB on the device)"),
    "prof5": ("profiling case: exact L2 kNN, config 5's Gaussian mixture on 2,000,000x96 rows, 10,000 "
              "queries, k=10 (2.8 GB on the device)"),
    "prof5l": ("profiling case: exact L2 kNN, config 5's Gaussian mixture on 2,000,000x96 rows, 18,944 "
               "queries (74 query groups over 2 splits, 250k rows per list), k=10 (2.9 GB on the device)"),
    "c3": "PQ ADC scan, L2, m=16 x 256 centroids (k-means on a 100,000-row sample), 1,000,000 codes, "
          "1,000 queries, k=10 (config 3)",
}
BLOCK = 1 << 18  # rows generated per seeded block


# ---------------------------------------------------------------- data ------

def _gen_block(kind, b, rows, dim, seed, device):
    """Rows [b*BLOCK, b*BLOCK+rows) of a seeded synthetic set (identical for
    any world size: each block has its own generator)."""
    import torch
    g = torch.Generator(device=device)
    if kind == "unit":
        g.manual_seed(seed * 1_000_003 + b)
        x = torch.randn((rows, dim), generator=g, device=device, dtype=torch.float32)
        return x / torch.linalg.vector_norm(x, dim=1, keepdim=True)
    if kind == "sift":
        gc = torch.Generator(device=device)
        gc.manual_seed(seed)
        centres = torch.rand((1000, dim), generator=gc, device=device) * 128
        g.manual_seed(seed * 1_000_003 + b + 1)
        lab = torch.randint(0, 1000, (rows,), generator=g, device=device)
        x = centres[lab] + torch.randn((rows, dim), generator=g, device=device) * 20
        return torch.clamp(x, 0, 255).round()
    if kind == "mixture":
        gc = torch.Generator(device=device)
        gc.manual_seed(seed)
        centres = torch.randn((10_000, dim), generator=gc, device=device) * 4
        g.manual_seed(seed * 1_000_003 + b + 1)
        lab = torch.randint(0, 10_000, (rows,), generator=g, device=device)
        return centres[lab] + torch.randn((rows, dim), generator=g, device=device)
    raise ValueError(kind)


def gen_rows(kind, begin, end, dim, seed, device, sink):
    """Calls sink(tensor) for consecutive pieces of rows [begin, end)."""
    b0, b1 = begin // BLOCK, (end - 1) // BLOCK
    for b in range(b0, b1 + 1):
        lo, hi = b * BLOCK, (b + 1) * BLOCK
        x = _gen_block(kind, b, BLOCK, dim, seed, device)
        s, e = max(lo, begin) - lo, min(hi, end) - lo
        sink(x[s:e].contiguous())
        del x


def gen_queries(kind, nq, dim, seed, device):
    # Queries come from the same distribution with an independent seed
    # (held out: no query is a base row).
    return _gen_block(kind, 10_000_000 + 7, nq, dim, seed + 1, device).contiguous()


# ---------------------------------------------------------------- clocks ----

class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during a region."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.reasons = 0
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            self._stop.wait(0.05)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------- helpers ---

def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"bf16_tflops": p["bf16_tflops"], "bf16_tflops_sustained": p["bf16_tflops_sustained"],
                "hbm_gbs": p["hbm_gbs"], "source": "measured"}
    except Exception:
        return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0,
                "source": "fallback"}


def ncu_traffic(config, kernel):
    """Per-launch DRAM bytes of `kernel` on `config` from the committed ncu
    summary (profiles/traffic.txt), or None if that pair was not captured."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) == 4 and not line.startswith("#") and parts[0] == config and parts[1] == kernel:
                    return int(parts[2]) + int(parts[3])
    except OSError:
        pass
    return None


def host_cores():
    """Host threads the CPU baseline may use (torchrun sets OMP_NUM_THREADS=1
    for its workers, so the count is passed to the oracle explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_threads():
    return host_cores()


def cpu_sample_qps(base_host, metric, queries_host, k, sample, threads=None):
    """Times the oracle (reference CPU path restated) on `sample` queries."""
    import oracle as O
    m = O.L2 if metric == "l2" else O.IP
    q = np.ascontiguousarray(queries_host[:sample])
    t = time.perf_counter()
    ids, d = O.flat_search_batch(base_host, m, q, k, num_threads=threads or host_cores())
    dt = time.perf_counter() - t
    return sample / dt, dt, ids, d


def host_copy(kind, n, dim, seed, device):
    """The whole base in host memory (for the CPU baseline and parity)."""
    out = np.empty((n, dim), dtype=np.float32)
    pos = [0]

    def sink(x):
        c = x.shape[0]
        out[pos[0]:pos[0] + c] = x.cpu().numpy()
        pos[0] += c
    gen_rows(kind, 0, n, dim, seed, device, sink)
    return out


# ---------------------------------------------------------------- arms ------

def run_reference(args, cfg, rank, world):
    """--impl reference: the reference CPU implementation (restated) only."""
    metric, n, dim, nq, k, kind = cfg
    if rank != 0:
        return 0
    import torch
    device = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    base = host_copy(kind, n, dim, args.seed, device)
    queries = gen_queries(kind, nq, dim, args.seed, device).cpu().numpy()
    if metric.startswith("pq"):
        return run_reference_pq(args, cfg, world, base, queries)
    sample = args.ref_sample
    for _ in range(args.warmup):
        cpu_sample_qps(base, metric, queries[:max(1, sample // 4)], k, max(1, sample // 4))
    times = []
    for s in range(args.steps):
        off = (s * sample) % max(1, nq - sample)
        _, dt, _, _ = cpu_sample_qps(base, metric, queries[off:off + sample], k, sample)
        times.append(dt)
    value = sample * args.steps / sum(times)
    line = {
        "metric": f"exact kNN QPS (k={k})", "value": value, "unit": "queries/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD_TEXT[args.config], "n_base": n, "dim": dim, "nq": nq, "k": k,
                   "metric": metric},
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": cpu_threads(), "kind": "port",
                         "sample": f"{sample} queries per step against the full {n}x{dim} base; "
                                   "C++ restatement of FlatIndex::search_batch (flat.rs:150-191), "
                                   "all host threads (the Rust crate cannot be built here)"},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference_pq(args, cfg, world, base, queries):
    """--impl reference for config 3: codebooks and codes from the oracle's
    restatement of ProductQuantizer::train / encode_into with the parameters
    the GPU arm uses (so both scan the same codes), then the oracle's
    PqIndex::search_batch over all queries each step."""
    import oracle as O
    metric, n, dim, nq, k, kind = cfg
    books = O.pq_train(base, 16, nbits=8, train_iters=25, train_sample=100_000, seed=args.seed)
    codes = O.pq_encode(books, base)
    for _ in range(args.warmup):
        O.pq_search_batch(books, O.L2, codes, queries[:max(1, nq // 8)], k, num_threads=host_cores())
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        O.pq_search_batch(books, O.L2, codes, queries, k, num_threads=host_cores())
        times.append(time.perf_counter() - t)
    value = nq * args.steps / sum(times)
    line = {
        "metric": f"PQ ADC QPS (k={k})", "value": value, "unit": "queries/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 (u8 codes)",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD_TEXT[args.config], "n_codes": n, "dim": dim, "m": 16, "nq": nq, "k": k},
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": cpu_threads(), "kind": "port",
                         "sample": f"all {nq} queries per step against all {n} codes; C++ restatement of "
                                   "PqIndex::search_batch (pq.rs:349-396), all host threads"},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_pq(args, cfg, rank, world, local_rank):
    """Config 3: the PQ ADC scan through PqIndex (host buffers, one GPU)."""
    import torch
    import proxima_b200 as px
    from proxima_b200 import _lib

    metric, n, dim, nq, k, kind = cfg
    if world > 1:
        if rank == 0:
            print(json.dumps({"metric": f"PQ ADC QPS (k={k})", "unavailable": "PQ bench runs on one GPU"}))
        return 0
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(local_rank)
    base = host_copy(kind, n, dim, args.seed, device)
    queries = gen_queries(kind, nq, dim, args.seed, device).cpu().numpy()
    t0 = time.time()
    pq = px.PqIndex(dim, px.Metric.L2, m=16, nbits=8, train_iters=25, train_sample=100_000, seed=args.seed,
                    devices=[local_rank])
    pq.train(base)
    pq.add(base)
    build_s = time.time() - t0
    lib = _lib.load()
    d_q = torch.from_numpy(queries).to(device)
    d_ids = torch.empty((nq, k), dtype=torch.int64, device=device)
    d_d = torch.empty((nq, k), dtype=torch.float32, device=device)
    sp = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)

    def step_device():
        _lib.check(lib.px_pq_search_device(pq.handle, ctypes.c_void_p(d_q.data_ptr()), nq, k, 0,
                                           ctypes.c_void_p(d_ids.data_ptr()), ctypes.c_void_p(d_d.data_ptr()), sp))

    for _ in range(args.warmup):
        step_device()
        pq.search_batch(queries, k=k)
    torch.cuda.synchronize()
    # ---- device-resident timing (queries and results in HBM) -------------
    _lib.set_profiling(True)
    launches0 = _lib.launch_count()
    kernel_ms = []
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        start.record()
        for _ in range(args.steps):
            step_device()
            kernel_ms.append(pq.last_search_profile()["main_kernel_ms"])
        stop.record()
        torch.cuda.synchronize()
    _lib.set_profiling(False)
    launches = _lib.launch_count() - launches0
    dev_step_s = start.elapsed_time(stop) / 1e3 / args.steps
    kern_s = statistics.mean(kernel_ms) / 1e3
    # ---- end to end through PqIndex.search_batch (host buffers) ----------
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        ids, d = pq.search_batch(queries, k=k)
        times.append(time.perf_counter() - t)
    step_s = statistics.mean(times)
    m = 16
    gathers = float(nq) * n * m
    byts = n * m + nq * (dim * 4 + m * 256 * 4)
    pk = peaks()
    clock = clocks.summary()
    sm_ghz = (clock.get("sm_mhz") or 1965.0) / 1e3
    smem_peak = 148 * 32 * sm_ghz  # conflict-free 32-bit gathers per ns
    cpu = parity = None
    if not args.no_cpu_baseline:
        import oracle as O
        from tests import _parity
        books = pq.codebooks
        codes = pq.encode(base)
        sample = min(args.cpu_sample * 4, nq)
        t = time.perf_counter()
        ref_ids, ref_d = O.pq_search_batch(books, O.L2, codes, queries[:sample], k, num_threads=host_cores())
        dt = time.perf_counter() - t
        s1 = max(1, sample // cpu_threads())
        t1 = time.perf_counter()
        O.pq_search_batch(books, O.L2, codes, queries[:s1], k, num_threads=1)
        dt1 = time.perf_counter() - t1
        cpu = {"value": sample / dt, "unit": "queries/s", "cores": cpu_threads(), "kind": "port",
               "sample": f"first {sample} of the {nq} queries against all {n} codes ({dt:.2f} s); "
                         "C++ restatement of PqIndex::search_batch, all host threads",
               "single_thread": {"value": s1 / dt1, "unit": "queries/s", "cores": 1,
                                 "sample": f"first {s1} queries, one thread ({dt1:.2f} s)"}}
        try:
            ties = _parity.check(ids[:sample], d[:sample], ref_ids, ref_d,
                                 _parity.pq_natural(books, O.L2, codes, queries[:sample]))
            parity = {"queries": sample, "ok": True, "tie_positions": int(ties)}
        except AssertionError as e:
            parity = {"queries": sample, "ok": False, "error": str(e)[:200]}
    line = {
        "metric": f"PQ ADC QPS (k={k})", "value": nq / dev_step_s, "unit": "queries/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dev_step_s, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32 (u8 codes)", "data": "synthetic",
        "config": {"workload": WORKLOAD_TEXT[args.config], "n_codes": n, "dim": dim, "m": m, "nq": nq, "k": k,
                   "build_s": round(build_s, 2),
                   "timing": "value: px_pq_search_device, queries and results in HBM (CUDA events); "
                             "e2e: host-to-host PqIndex.search_batch",
                   "l2_flush": "none: the 16 MB of codes stay in L2 by design (the scan is bound by "
                               "on-chip LUT gathers, not HBM)"},
        # Config 3 at nq = 1,000 is bound by the shared-memory LUT gathers (16
        # per code per query), not by HBM: the codes are 16 MB per pass.
        "roofline": {"bound": "smem", "achieved": gathers / kern_s / 1e9, "peak": smem_peak,
                     "unit": "LUT gathers/ns", "frac": gathers / kern_s / 1e9 / smem_peak,
                     "traffic": ncu_traffic(args.config, "pq_scan_kernel"),
                     "kernel": "pq_scan_kernel", "kernel_ms": 1e3 * kern_s,
                     "algorithmic_gathers_per_launch": gathers,
                     "peak_basis": "148 SMs x 32 four-byte shared-memory words per clock x the median SM clock "
                                   "sampled during the run (no measured shared-memory peak exists)",
                     "hbm_view": {"achieved_gbs": byts / kern_s / 1e9, "peak_gbs": pk["hbm_gbs"],
                                  "frac": byts / kern_s / 1e9 / pk["hbm_gbs"],
                                  "algorithmic_bytes_per_launch": byts}},
        "cpu_baseline": cpu, "parity_sample": parity,
        "e2e": {"value": nq / step_s, "unit": "queries/s", "h2d_bytes_per_step": int(queries.nbytes),
                "d2h_bytes_per_step": int(nq * k * 12), "api": "PqIndex.search_batch (px_pq_search)"},
        "clocks": clock, "gpu_launches": int(launches),
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, cfg, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import proxima_b200 as px
    from proxima_b200 import _lib
    from proxima_b200.distributed import ShardedFlatIndex, shard_range

    metric, n, dim, nq, k, kind = cfg
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    m = px.Metric.L2 if metric == "l2" else px.Metric.InnerProduct
    index = ShardedFlatIndex(dim, m, device=local_rank)
    begin, end = shard_range(n, world, rank)
    index.set_offset(begin)
    index.local.set_search_path(args.path)
    index.reserve_local(end - begin)
    t0 = time.time()
    gen_rows(kind, begin, end, dim, args.seed, device, index.add_local_device)
    build_s = time.time() - t0
    queries = gen_queries(kind, nq, dim, args.seed, device)
    q_host = torch.empty(queries.shape, dtype=torch.float32, pin_memory=True)
    q_host.copy_(queries)
    ids_host = torch.empty((nq, k), dtype=torch.int64, pin_memory=True)
    d_host = torch.empty((nq, k), dtype=torch.float32, pin_memory=True)
    lib = _lib.load()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def step_device():
        return index.search_device(queries, k)

    # Warm-up (also sizes every workspace: no allocation in the timed region).
    for _ in range(args.warmup):
        step_device()
    barrier()

    # ---- device-resident timing with kernel profiling -------------------
    _lib.set_profiling(True)
    index.local.profile_totals(reset=True)
    launches0 = _lib.launch_count()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        start.record()
        for _ in range(args.steps):
            step_device()
        stop.record()
        barrier()
    launches = _lib.launch_count() - launches0
    # The library sums the dominant kernel's event times over the timed
    # searches, so the loop above reads nothing back between steps.
    tot = index.local.profile_totals()
    kernel_ms = [tot["main_kernel_ms"] / tot["profiled_searches"]] if tot["profiled_searches"] else []
    fallbacks, refined = tot["fallback_queries"], tot["refined_queries"]
    _lib.set_profiling(False)
    dev_ms = start.elapsed_time(stop)
    t = torch.tensor([dev_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms = float(t.item())
    ms_per_step = dev_ms / args.steps
    value = nq / (ms_per_step / 1e3)
    path = index.local.last_search_profile()["path"]

    # ---- end-to-end through the public API (host buffers) -----------------
    def step_e2e():
        if world == 1:
            st = lib.px_flat_search(index.local.handle, ctypes.cast(q_host.data_ptr(), _lib._f32p), nq, k,
                                    ctypes.cast(ids_host.data_ptr(), _lib._i64p),
                                    ctypes.cast(d_host.data_ptr(), _lib._f32p))
            _lib.check(st)
        else:
            dq = torch.empty_like(queries)
            dq.copy_(q_host, non_blocking=True)
            ids, d = index.search_device(dq, k)
            ids_host.copy_(ids, non_blocking=True)
            d_host.copy_(d, non_blocking=True)
            torch.cuda.current_stream().synchronize()

    for _ in range(max(1, args.warmup // 2)):
        step_e2e()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step_e2e()
    barrier()
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_s = float(t.item())
    e2e = {"value": nq * args.steps / e2e_s, "unit": "queries/s",
           "h2d_bytes_per_step": int(q_host.numel() * 4),
           "d2h_bytes_per_step": int(ids_host.numel() * 8 + d_host.numel() * 4) if rank == 0 else 0,
           "api": "px_flat_search (C ABI, pinned host buffers)" if world == 1 else
                  "ShardedFlatIndex.search_device + pinned H2D/D2H"}

    # ---- roofline of the dominant kernel ----------------------------------
    pk = peaks()
    n_local = end - begin
    roofline = None
    if kernel_ms:
        avg_s = statistics.mean(kernel_ms) / 1e3
        if path == "tensor":
            flops = 2.0 * nq * n_local * dim
            achieved = flops / avg_s / 1e12
            first = index.local.last_search_profile()["first_pass"]
            sample_tiles = index.local.last_search_profile()["sample_tiles"]
            # bf16 MMAs issue at the measured bf16 rate, tf32 at half of it,
            # and the 3xTF32 sum takes three tf32 MMAs per product.
            peak = pk["bf16_tflops_sustained"] / {"bf16": 1.0, "tf32": 2.0, "3xtf32": 6.0}[first]
            fp32_peak = pk["bf16_tflops_sustained"] / 6.0
            traffic = ncu_traffic(args.config, "gemm_topk_kernel") if world == 1 else None
            roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                        "frac": achieved / peak, "traffic": traffic,
                        "traffic_note": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch; "
                                        f"the bf16 base is {2 * n_local * dim / 1e9:.2f} GB" if traffic else None,
                        "kernel": {"bf16": "gemm_topk_pair_kernel (tcgen05 cta_group::2 kind::f16, bf16 operands)",
                                   "tf32": "gemm_topk_kernel (tcgen05 kind::tf32, hi values)",
                                   "3xtf32": "gemm_topk_kernel (tcgen05 kind::tf32, 3xTF32 sum)"}[first],
                        "kernel_ms": statistics.mean(kernel_ms),
                        # The timed span starts before the sample pass (that
                        # many single base tiles per query group) and its merge.
                        "sample_pass_tiles": sample_tiles,
                        "peak_basis": {"bf16": "bf16 rate = bf16_tflops_sustained",
                                       "tf32": "TF32 rate = bf16_tflops_sustained / 2",
                                       "3xtf32": "3xTF32 rate = bf16_tflops_sustained / 2 / 3"}[first]
                                      + f" ({pk['bf16_tflops_sustained']}), " + pk["source"],
                        "frac_of_bf16_peak": achieved / pk["bf16_tflops_sustained"],
                        # Exact kNN throughput against the fp32-accurate (3xTF32)
                        # tensor roofline: the results are exact on every path.
                        "vs_fp32_accurate_roofline": {"achieved_tflops": achieved, "peak_tflops": fp32_peak,
                                                      "frac": achieved / fp32_peak,
                                                      "basis": "3xTF32 rate = bf16_tflops_sustained / 2 / 3"},
                        "algorithmic_flops_per_launch": flops}
            # A few queries against many rows (config 2 at 64 queries) cannot
            # keep the MMAs busy: the pass must still read its operand plane
            # once (2 bytes per element for bf16, 4 for tf32 values), and when
            # that takes longer at the measured HBM rate than the MMAs at
            # theirs, HBM is the bound the fraction is reported against.
            plane = (2.0 if first == "bf16" else 4.0) * n_local * dim
            if plane / (pk["hbm_gbs"] * 1e9) > flops / (peak * 1e12):
                tensor_view = {k2: roofline[k2] for k2 in ("achieved", "peak", "unit", "frac")}
                achieved_b = plane / avg_s / 1e9
                roofline.update({"bound": "hbm", "achieved": achieved_b, "peak": pk["hbm_gbs"], "unit": "GB/s",
                                 "frac": achieved_b / pk["hbm_gbs"], "algorithmic_bytes_per_launch": plane,
                                 "tensor_view": tensor_view,
                                 "peak_basis": f"hbm_gbs ({pk['hbm_gbs']}), " + pk["source"]})
        else:
            byts = 4.0 * n_local * dim
            achieved = byts / avg_s / 1e9
            roofline = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                        "frac": achieved / pk["hbm_gbs"], "traffic": None,
                        "kernel": "exact_scan_kernel", "kernel_ms": statistics.mean(kernel_ms),
                        "algorithmic_bytes_per_launch": byts}

    # ---- CPU baseline + parity sample (rank 0, N=1) -----------------------
    cpu = None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base_host = host_copy(kind, n, dim, args.seed, device)
        qh = queries.cpu().numpy()
        sample = args.cpu_sample
        qps, dt, ref_ids, ref_d = cpu_sample_qps(base_host, metric, qh, k, sample)
        # The same path on one thread, on a proportionally smaller sample.
        s1 = max(1, sample // cpu_threads())
        qps1, dt1, _, _ = cpu_sample_qps(base_host, metric, qh, k, s1, threads=1)
        cpu = {"value": qps, "unit": "queries/s", "cores": cpu_threads(), "kind": "port",
               "sample": f"first {sample} of the {nq} queries against the full {n}x{dim} base "
                         f"({dt:.1f} s); C++ restatement of FlatIndex::search_batch, all host threads",
               "single_thread": {"value": qps1, "unit": "queries/s", "cores": 1,
                                 "sample": f"first {s1} queries, one thread ({dt1:.1f} s)"}}
        import oracle as O
        from tests import _parity
        ids, d = index.search_device(queries[:sample].contiguous(), k)
        try:
            ties = _parity.check(ids.cpu().numpy(), d.cpu().numpy(), ref_ids, ref_d,
                                 _parity.flat_natural(base_host, O.L2 if metric == "l2" else O.IP, qh[:sample]))
            parity = {"queries": sample, "ok": True, "tie_positions": int(ties)}
        except AssertionError as e:
            parity = {"queries": sample, "ok": False, "error": str(e)[:200]}
        del base_host

    if rank == 0:
        line = {
            "metric": f"exact kNN QPS (k={k})", "value": value, "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded torch generators)",
            "config": {"workload": WORKLOAD_TEXT[args.config], "n_base": n, "dim": dim, "nq": nq, "k": k,
                       "metric": metric, "sharding": f"rows over {world} GPU(s)",
                       "l2_flush": "none needed: inputs larger than L2 (base "
                                   f"{n * dim * 4 / 1e9:.1f} GB)",
                       "path": path, "build_s": round(build_s, 2)},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks.summary(),
            "gpu_launches": int(launches), "certificate_fallback_queries": fallbacks,
            "three_pass_refined_queries": refined,
            "parity_sample": parity,
        }
        print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c4k10")
    ap.add_argument("--seed", type=int, default=2024)
    ap.add_argument("--cpu-sample", type=int, default=112,
                    help="queries timed on the CPU baseline; also the parity sample")
    ap.add_argument("--ref-sample", type=int, default=16, help="queries per step of --impl reference")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--path", choices=["auto", "exact", "tensor", "tensor_3xtf32"], default="auto",
                    help="flat-search kernel path (auto is the library default)")
    args = ap.parse_args(argv)
    if args.warmup < 3 and args.impl == "ours":
        print("note: --warmup raised to 3 (timing rule)", file=sys.stderr)
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference(args, cfg, rank, world)

    import torch.distributed as dist
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        import torch
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if cfg[0].startswith("pq"):
            return run_pq(args, cfg, rank, world, local_rank)
        return run_ours(args, cfg, rank, world, local_rank)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
