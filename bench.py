"""Benchmark: exact L2 k-NN QPS on the headline configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one search batch of Q queries against the whole dataset (row-
sharded over the N GPUs, one process per GPU under torchrun).  The default
workload is BASELINE.json's headline: N = 1,000,000 rows, D = 1024, Q = 100,
K = 10, unit-norm Gaussian mixture (10,000 centres, sigma 0.3).

Printed on rank 0, one JSON line:
  value        QPS with queries and results resident in HBM (device timing,
               CUDA events on the launching stream, max over ranks)
  e2e          QPS through the public API with pinned HOST queries/results,
               H2D + D2H inside the timed region
  roofline     the scan kernel's achieved HBM GB/s (algorithmic bytes
               N_shard * D * 2 per launch / its CUDA-event duration) against
               MEASURED_PEAKS.json's copy bandwidth
  cpu_baseline the reference's own CPU exact search (oracle/_ref, compiled
               from its src/cagra.cpp) on a bounded sample of queries, all
               host threads; plus an OpenBLAS expanded-form port
  latency      per-batch latency percentiles (nearest rank, as the
               reference's cuvs_silicon/benchmark.py:573-578): end to end
               through the blocking call with host buffers (host clock, as
               tests/test_cohere_wiki_validation.cpp:165-185 times it) and
               device-resident (CUDA events per search); max over ranks
  parity       the merged result of the last end-to-end search (rank 0,
               every GPU count) against the reference's own search on the
               fp16-rounded rows, for a sample of the queries (acceptance
               rule oracle.check_parity: indices equal or float64 distances
               within rel 1e-3, recall 1, sorted, padding)
  clocks       SM clock samples (NVML) during the timed region

--impl reference times the reference's CPU implementation alone (rank 0).
--sweep c5 runs BASELINE config 5 (Q in {1, 16} x K in {10, 256}) on one
index and prints one line per combination.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "cuvs-silicon_b200")



METRIC = "QPS at N=1M D=1024 K=10 Q=100 (1/2/4/8 B200) and % of HBM/tensor roofline"
UNIT = "queries/s"
PUBLISHED_QPS = 1012.0  # the reference README.md:23-27: Apple M3 Max, 1M x 1024, batch of 100
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    # --rows is the same option: under torch.distributed.run "--n" is an
    # ambiguous prefix of the launcher's own options
    ap.add_argument("--n", "--rows", dest="n", type=int, default=1_000_000)
    ap.add_argument("--dim", type=int, default=1024)
    ap.add_argument("--q", type=int, default=100)
    ap.add_argument("--k", type=int, default=10)
    ap.add_argument("--centres", type=int, default=10_000)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--metric", default="l2", choices=["l2", "ip"],
                    help="l2: squared L2 (the headline); ip: inner product")
    ap.add_argument("--rerank", action="store_true",
                    help="exact fp32 re-ranking of the fp16 scan's candidates")
    ap.add_argument("--no-graphs", action="store_true",
                    help="launch every search directly instead of replaying CUDA graphs")
    ap.add_argument("--sweep", default=None, choices=["c5"],
                    help="c5: BASELINE config 5 (Q in {1, 16} x K in {10, 256}) on one index, "
                         "one JSON line per combination (the default run prints one line)")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    return a


def workload_name(a):
    head = (a.n, a.dim, a.q, a.k) == (1_000_000, 1024, 100, 10)
    name = ("headline " if head else "") + f"N={a.n} D={a.dim} Q={a.q} K={a.k}"
    if a.metric == "ip":
        name += " InnerProduct"
    if a.rerank:
        name += " exact-fp32-rerank"
    return name


def peaks():
    """(HBM GB/s, dense bf16 TFLOP/s sustained, burst, kind): the measured
    figures of MEASURED_PEAKS.json, else the pool's earlier fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), float(p["bf16_tflops_sustained"]),
                float(p["bf16_tflops"]), "measured")
    except Exception:
        return 6650.0, 1400.0, 1590.0, "fallback"


def roofline(n_shard, dim, nq, kernel_ms):
    """The scan's roofline (the slower of streaming N_shard * D * 2 bytes at
    the HBM peak and 2 * Q * N_shard * D flops at the dense fp16 tensor peak,
    which equals bf16 on B200): the bound, what the kernel achieved against
    it, and both algorithmic amounts per launch.  The tensor peak is the
    sustained one (the scan is timed inside a loop of back-to-back searches);
    the burst figure is reported beside it."""
    hbm, tf_sus, tf_burst, kind = peaks()
    nbytes = n_shard * dim * 2
    flops = 2.0 * nq * n_shard * dim
    t_hbm = nbytes / (hbm * 1e9)
    t_tensor = flops / (tf_sus * 1e12)
    secs = kernel_ms / 1000.0
    if t_tensor > t_hbm:
        achieved = flops / secs / 1e12
        return {"bound": "tensor", "achieved": achieved, "peak": tf_sus, "unit": "TFLOP/s",
                "frac": achieved / tf_sus, "frac_of_burst": achieved / tf_burst,
                "peak_kind": f"{kind} (sustained; burst {tf_burst})",
                "algorithmic_flops_per_launch": flops, "algorithmic_bytes_per_launch": nbytes}
    achieved = nbytes / secs / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm, "peak_kind": kind,
            "algorithmic_bytes_per_launch": nbytes, "algorithmic_flops_per_launch": flops}


def profile_traffic(a, n_shard):
    """dram bytes per scan launch from the committed ncu figures
    (profiles/knn_scan_traffic.json: dram__bytes_read.sum +
    dram__bytes_write.sum of one captured launch per configuration), scaled
    to this shard's rows when captured on a different row count (the scan's
    traffic grows in proportion to the rows it reads).  Uses the capture of
    the same dim and k whose query count is within a factor of two of this
    run's; None when there is none."""
    path = os.path.join(ROOT, "profiles", "knn_scan_traffic.json")
    try:
        with open(path) as f:
            v = json.load(f)
        for c in v["captures"]:
            if int(c["captured_dim"]) != a.dim or int(c["captured_k"]) != a.k:
                continue
            cq = int(c["captured_queries"])
            if a.q // 2 <= cq <= 2 * a.q:
                return float(c["traffic_bytes_per_launch"]) * n_shard / float(c["captured_rows"])
        return None
    except Exception:
        return None


def nearest_rank(values, pct):
    """Nearest-rank percentile (the reference's cuvs_silicon/benchmark.py:573-578)."""
    import math

    v = sorted(values)
    i = math.ceil(pct / 100.0 * len(v)) - 1
    return v[max(0, min(i, len(v) - 1))]


class ClockSampler:
    """Samples the SM clock and throttle reasons through NVML (read only)."""

    def __init__(self, device_index: int):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None
        self.names = {}
        if self.nv:
            for n in ("GpuIdle", "ApplicationsClocksSetting", "SwPowerCap", "HwSlowdown",
                      "SyncBoost", "SwThermalSlowdown", "HwThermalSlowdown",
                      "HwPowerBrakeSlowdown", "DisplayClockSetting"):
                v = getattr(self.nv, "nvmlClocksEventReason" + n, None)
                if v is None:
                    v = getattr(self.nv, "nvmlClocksThrottleReason" + n, None)
                if v is not None:
                    self.names[v] = n

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                try:
                    r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except Exception:
                    r = self.nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                for bit, name in self.names.items():
                    if r & bit and name != "GpuIdle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.nv:
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def gen_mixture_device(torch, n_total, begin, end, dim, centres, seed, device, sigma=0.3):
    """Rows [begin, end) of the unit-norm mixture, generated on the GPU in
    65,536-row chunks; chunk c uses generator seed (seed, c), so every rank
    reproduces its own row shard without materialising the others."""
    chunk = 65536
    out = torch.empty((end - begin, dim), dtype=torch.float32, device=device)
    c0, c1 = begin // chunk, (end - 1) // chunk if end > begin else -1
    for c in range(c0, c1 + 1):
        lo, hi = c * chunk, min(n_total, (c + 1) * chunk)
        g = torch.Generator(device=device)
        g.manual_seed(seed * 1_000_003 + c)
        u = torch.randint(0, centres.shape[0], (hi - lo,), generator=g, device=device)
        x = torch.randn((hi - lo, dim), generator=g, device=device)
        x.mul_(sigma).add_(centres[u])
        x.div_(x.norm(dim=1, keepdim=True))
        a, b = max(lo, begin), min(hi, end)
        out[a - begin:b - begin] = x[a - lo:b - lo]
    return out


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_reference_qps(base16_host, q16_host, k, sample_q, threads):
    """The reference's own exact CPU search (oracle/_ref) on sample_q queries
    against every row; returns (qps, seconds, idx)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    q = q16_host[:sample_q]
    # the reference's build copies the dataset into its index on every call
    # (one call per thread): past 96 GB of copies the C restatement, which
    # reads the rows in place, stands in (same results, pinned bit for bit)
    use_ref = oracle.ref_available() and \
        base16_host.nbytes * min(threads, sample_q) <= 96 * 10 ** 9
    t0 = time.perf_counter()
    if use_ref:
        idx, dist = oracle.ref_knn(base16_host, q, k, threads=threads)
    else:
        idx, dist = oracle.port_knn(base16_host, q, k, threads=threads)
    dt = time.perf_counter() - t0
    return sample_q / dt, dt, idx, dist, ("reference" if use_ref else "port")


# ---------------------------------------------------------------- reference arm
def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np

    import oracle

    threads = host_threads()
    centres = oracle.gen_centres(a.centres, a.dim)
    base = oracle.round_fp16(oracle.gen_mixture(a.n, a.dim, a.centres, oracle.SEED_BASE,
                                                centres=centres, threads=threads))
    queries = oracle.round_fp16(oracle.gen_mixture(a.q, a.dim, a.centres,
                                                   oracle.SEED_QUERIES, centres=centres))
    kind = "reference" if oracle.ref_available() else "port"
    fn = oracle.ref_knn if kind == "reference" else oracle.port_knn
    # one step = a bounded sample of the batch: one query per host thread
    sample = max(1, min(a.q, threads))
    times = []
    for s in range(a.warmup + a.steps):
        lo = (s * sample) % a.q
        q = np.roll(queries, -lo, axis=0)[:sample]
        t0 = time.perf_counter()
        fn(base, q, a.k, threads=threads)
        dt = time.perf_counter() - t0
        if s >= a.warmup:
            times.append(dt)
    total = sum(times)
    qps = sample * len(times) / total
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": UNIT,
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": 1000.0 * total / len(times), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": qps / PUBLISHED_QPS, "dtype": "f32",
        "data": "synthetic: unit-norm Gaussian mixture (numpy PCG64, seeds 11/12/13), "
                "fp16-rounded, fp32 on host",
        "config": {"workload": workload_name(a), "n_rows": a.n, "dim": a.dim,
                   "n_queries": a.q, "k": a.k, "metric": "L2Expanded",
                   "exact_fp32_rerank": False,
                   "sample": f"{sample} queries per step x all {a.n} rows"},
        "cpu_baseline": {"value": qps, "unit": UNIT, "cores": min(threads, sample),
                         "kind": kind,
                         "sample": f"{sample} of {a.q} queries per step against all rows"},
        "e2e": {"value": qps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


# ---------------------------------------------------------------- engine arm
def full_dataset_fp16_host(torch, a, centres, dev):
    """The whole dataset, generated again on this GPU chunk by chunk with the
    same per-chunk seeds every rank used for its shard, rounded to fp16 on
    the device and returned as fp32 host rows (the values the engine
    searches)."""
    import numpy as np

    out = np.empty((a.n, a.dim), dtype=np.float32)
    step = 65536 * 4
    for lo in range(0, a.n, step):
        hi = min(a.n, lo + step)
        x = gen_mixture_device(torch, a.n, lo, hi, a.dim, centres, 12, dev)
        out[lo:hi] = x.half().float().cpu().numpy()
        del x
    return out


C5_SWEEP = [(1, 10), (1, 256), (16, 10), (16, 256)]  # Q x K


def run_engine(a):
    import numpy as np
    import torch
    import torch.distributed as dist

    sys.path.insert(0, PKG)
    import cuvs_b200 as E

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=dev)

    combos = C5_SWEEP if a.sweep == "c5" else [(a.q, a.k)]
    max_q = max(q for q, _ in combos)
    max_k = max(k for _, k in combos)

    # ---- data (synthetic, on device)
    cg = torch.Generator(device=dev)
    cg.manual_seed(11)
    centres = torch.randn((a.centres, a.dim), generator=cg, device=dev)
    lo, hi = E.shard_range(a.n, world, rank)
    shard = gen_mixture_device(torch, a.n, lo, hi, a.dim, centres, 12, dev)
    all_queries = gen_mixture_device(torch, max_q, 0, max_q, a.dim, centres, 13, dev)

    # all engine work and every timing event on one explicit stream (the
    # legacy default stream's handle is 0, which the engine reads as "use
    # the index's own stream")
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    idx = E.Index(local)
    idx.set_stream(stream.cuda_stream)
    if a.no_graphs:
        idx.set_graphs(False)
    if a.rerank:
        idx.set_rerank(True)
    metric = E.METRIC_INNER_PRODUCT if a.metric == "ip" else E.METRIC_L2_EXPANDED
    idx.build(shard, metric=metric, row_offset=lo, total_rows=a.n)
    torch.cuda.synchronize()
    host_base = None
    check = rank == 0 and not a.no_cpu_baseline and a.metric == "l2"
    if check and world == 1:
        # the rows the engine's results are exact for: fp16-rounded, or the
        # fp32 rows themselves with re-ranking
        host_base = (shard if a.rerank else shard.half().float()).cpu().numpy()
    del shard
    if world > 1:
        obj = [E.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        idx.attach_comm(obj[0], world, rank)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor(x if isinstance(x, list) else [x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        v = t.cpu().tolist()
        return v if isinstance(x, list) else v[0]

    def measure(nq, k):
        """Throughput, kernel split, latency and end-to-end QPS of Q = nq, K = k."""
        queries = all_queries[:nq].contiguous()
        out_i = torch.empty((nq, k), dtype=torch.int32, device=dev)
        out_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
        # ---- warm-up
        for _ in range(a.warmup):
            idx.search_async(queries, k, out_i, out_d)
        idx.sync()
        r = {}
        # ---- device-resident timing (value)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        idx.reset_kernel_stats()
        barrier()
        ev0.record(stream)
        for _ in range(a.steps):
            idx.search_async(queries, k, out_i, out_d)
        ev1.record(stream)
        idx.sync()
        torch.cuda.synchronize()
        r["dev_ms"] = max_over_ranks(ev0.elapsed_time(ev1))
        launches = idx.kernel_stats()["kernel_launches"]
        r["launches_total"] = int(max_over_ranks(float(launches)) * world)
        r["value"] = nq * a.steps / (r["dev_ms"] / 1000.0)
        # ---- kernel timing for the roofline (events around the scan kernel)
        idx.set_profiling(True)
        idx.reset_kernel_stats()
        barrier()
        for _ in range(a.steps):
            idx.search_async(queries, k, out_i, out_d)
        idx.sync()
        st = idx.kernel_stats()
        idx.set_profiling(False)
        r["scan_ms"] = max_over_ranks(st["scan_ms"] / max(1, st["scan_launches"]))
        r["merge_ms"] = max_over_ranks(st["merge_ms"] / max(1, st["scan_launches"]))
        # ---- device-resident latency: one search at a time, events around each
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(a.steps)]
        barrier()
        for e0, e1 in evs:
            e0.record(stream)
            idx.search_async(queries, k, out_i, out_d)
            e1.record(stream)
            idx.sync()
        torch.cuda.synchronize()
        r["lat_dev"] = max_over_ranks([e0.elapsed_time(e1) for e0, e1 in evs])
        # ---- end-to-end through the public API with pinned host buffers
        q_host = queries.cpu().pin_memory()
        i_host = torch.empty((nq, k), dtype=torch.int32).pin_memory()
        d_host = torch.empty((nq, k), dtype=torch.float32).pin_memory()
        for _ in range(3):
            idx.search(q_host, k, neighbors=i_host, distances=d_host)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.steps):
            idx.search(q_host, k, neighbors=i_host, distances=d_host)
        e1.record(stream)
        torch.cuda.synchronize()
        r["e2e"] = nq * a.steps / (max_over_ranks(e0.elapsed_time(e1)) / 1000.0)
        # per-batch wall-clock latency of the blocking call (the reference's
        # benchmark times each cagra::search call with a host clock)
        lat = []
        barrier()
        for _ in range(a.steps):
            t0 = time.perf_counter()
            idx.search(q_host, k, neighbors=i_host, distances=d_host)
            lat.append(1000.0 * (time.perf_counter() - t0))
        r["lat_e2e"] = max_over_ranks(lat)
        r["nbrs"] = i_host.numpy().view("uint32").copy()
        r["dists"] = d_host.numpy().copy()
        # every rank holds the merged global result: do they agree?
        r["ranks_agree"] = True
        if world > 1:
            mine = torch.from_numpy(np.concatenate([r["nbrs"].view(np.int32).ravel(),
                                                    r["dists"].view(np.int32).ravel()])).to(dev)
            allr = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(allr, mine)
            r["ranks_agree"] = all(bool(torch.equal(allr[0], t)) for t in allr)
        return r

    clk = ClockSampler(local)
    clk.__enter__()
    results = [measure(q, k) for q, k in combos]
    clk.__exit__(None, None, None)

    # ---- CPU baselines (rank 0, N = 1 only; bounded samples) and parity
    # (rank 0, every N): one run of the reference at the largest k, sliced
    # for the smaller ones (its top-k is a prefix of its top-K)
    cpu = None
    extra = {}
    oracle_out = None
    if check:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle

        threads = host_threads()
        q16 = (all_queries if a.rerank else all_queries.half().float()).cpu().numpy()
        if world == 1:
            sample = max(1, min(max_q, 2 * threads))
            qps, secs, ref_i, ref_d, kind = cpu_reference_qps(host_base, q16, max_k, sample,
                                                              threads)
            if a.sweep is None:
                cpu = {"value": qps, "unit": UNIT, "cores": min(threads, sample), "kind": kind,
                       "sample": f"{sample} of {max_q} queries against all {a.n} rows "
                                 f"({secs:.1f} s, "
                                 + ("reference cagra::search" if kind == "reference" else
                                    "C restatement of the reference's search")
                                 + ", one query slice per thread)"}
                try:
                    t0 = time.perf_counter()
                    oracle.blas_knn(host_base, q16, a.k)
                    bt = time.perf_counter() - t0
                    extra["cpu_blas_expanded_form"] = {
                        "value": a.q / bt, "unit": UNIT, "cores": threads, "kind": "port",
                        "sample": f"all {a.q} queries, numpy float32 matmul "
                                  f"(OpenBLAS sgemm, {oracle.blas_threads()}), {bt:.1f} s"}
                except Exception as e:  # informational only
                    extra["cpu_blas_expanded_form"] = {"error": str(e)[:200]}
        else:
            # the merged multi-rank result against the whole dataset, which
            # no rank holds: regenerate it here
            host_base = full_dataset_fp16_host(torch, a, centres, dev)
            sample = max(1, min(max_q, 16))
            _, secs, ref_i, ref_d, kind = cpu_reference_qps(host_base, q16, max_k, sample,
                                                            threads)
        oracle_out = (host_base, q16, sample, ref_i, ref_d, kind, oracle)

    def parity_of(r, nq, k):
        if oracle_out is None:
            return None
        base, q16, sample, ref_i, ref_d, kind, oracle = oracle_out
        m = min(sample, nq)
        oi, od = ref_i[:m, :k], ref_d[:m, :k]
        par = (oracle.check_parity(base, q16[:m], r["nbrs"][:m], r["dists"][:m], oi, od, 1e-3)
               if not a.rerank else None)
        exact = (bool(np.array_equal(r["nbrs"][:m], oi) and np.array_equal(r["dists"][:m], od))
                 if a.rerank else None)
        return {
            "ok": bool(par.ok if par is not None else exact) and r["ranks_agree"],
            "queries_checked": m, "of": nq,
            "oracle": ("reference cagra::search (oracle/_ref, the reference's "
                       "src/cagra.cpp compiled unmodified)" if kind == "reference"
                       else "C restatement of src/cagra.cpp:211-252 (oracle/knn_oracle.c)"),
            "rule": ("byte-identical to the reference's fp32 search" if a.rerank else
                     "oracle.check_parity on fp16-rounded rows: index equal or float64 "
                     "distances within rel 1e-3; recall@k 1.0; sorted; padding"),
            "detail": par.detail if par is not None else f"identical={exact}",
            "ranks_agree": r["ranks_agree"],
            "result_of": f"the last end-to-end search, merged over {world} rank(s)",
        }

    n_shard = hi - lo
    shard_mb = n_shard * a.dim * 2 / 2 ** 20
    if rank == 0:
        for (nq, k), r in zip(combos, results):
            aa = argparse.Namespace(**vars(a))
            aa.q, aa.k = nq, k
            line = {
                "metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": r["dev_ms"] / a.steps,
                "higher_is_better": True, "scaling": "strong",
                "vs_baseline": r["value"] / PUBLISHED_QPS, "dtype": "f16",
                "data": "synthetic: unit-norm Gaussian mixture (10,000 centres, sigma 0.3), "
                        "generated on device with torch (seeds 11/12/13)",
                "config": {"workload": workload_name(aa), "n_rows": a.n, "dim": a.dim,
                           "n_queries": nq, "k": k,
                           "metric": "InnerProduct" if a.metric == "ip" else "L2Expanded",
                           "exact_fp32_rerank": bool(a.rerank),
                           "parallelism": f"row-shard x{world}" + (
                               " + NVLink peer exchange of the per-rank top-k lists"
                               if world > 1 else ""),
                           "l2": f"inputs larger than L2 (dataset shard {shard_mb:.0f} MiB "
                                 f"> 126 MiB), no flush" if shard_mb > 126 else
                                 f"dataset shard {shard_mb:.0f} MiB fits in the 126 MiB L2 "
                                 f"(no flush): not an HBM measurement"},
                "roofline": dict(roofline(n_shard, a.dim, nq, r["scan_ms"]),
                                 traffic=profile_traffic(aa, n_shard),
                                 kernel="knn_scan_kernel", kernel_ms=r["scan_ms"],
                                 merge_ms=r["merge_ms"]),
                "cpu_baseline": cpu,
                "e2e": {"value": r["e2e"], "unit": UNIT, "h2d_bytes_per_step": nq * a.dim * 4,
                        "d2h_bytes_per_step": nq * k * 8},
                "latency": {
                    "e2e_p50_ms": nearest_rank(r["lat_e2e"], 50),
                    "e2e_p99_ms": nearest_rank(r["lat_e2e"], 99),
                    "device_p50_ms": nearest_rank(r["lat_dev"], 50),
                    "device_p99_ms": nearest_rank(r["lat_dev"], 99),
                    "samples": a.steps,
                    "how": "one batch at a time; e2e = host clock around the blocking search "
                           "with pinned host buffers; device = CUDA events around one "
                           "device-resident search; max over ranks per sample; nearest rank"},
                "parity": parity_of(r, nq, k),
                "gpu_launches": r["launches_total"],
                "clocks": clk.summary(),
            }
            if a.sweep:
                line["sweep"] = a.sweep
            line.update(extra)
            emit(line)
    idx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    a = parse()
    # rank 0's stdout must carry exactly one JSON line: native libraries
    # (NCCL's version banner, for one) write to file descriptor 1, so it
    # points at stderr until the line is printed
    sys.stdout.flush()
    real_stdout = os.dup(1)
    os.dup2(2, 1)
    global _emit_fd
    _emit_fd = real_stdout
    if a.impl == "reference":
        return run_reference(a)
    return run_engine(a)


_emit_fd = None


def emit(line: dict) -> None:
    """Writes the result line to the real standard output."""
    data = (json.dumps(line) + "\n").encode()
    if _emit_fd is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_emit_fd, data)


if __name__ == "__main__":
    sys.exit(main())
