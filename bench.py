"""Exact top-k search benchmark on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload mixed-100m] [--rows R] [--no-extra]

Workload (default): the 100M x 384 float32 unit-norm corpus -- half from a
16,384-centre Zipf(1.1) mixture (sigma 0.1), half anisotropic spread vectors --
with a 1,024-root / 32-children / rank-32 index, k = 10, queries drawn from the
same law, issued one at a time.  Synthetic and seeded; generated on the device.

Scaling is strong and the corpus is sharded by root cluster: every rank labels
1/N of the rows against the same root centres, the labels are all-gathered,
and the shard plan (whole roots largest first; a root larger than 1.05 x the
mean shard is cut between blocks of rows) gives each rank its parts, which it
builds into its own index (hierarchy.build.build_circuit_index_streaming).
At N = 1 the one rank holds every root.

A step is one query: root scan (with the seed sample) -> bounds -> main leaf
scan with fused top-k on every GPU; at N > 1 the shards' seed thresholds are
all-reduced (MAX) between the root scan and the bounds and the N local top-k
lists are merged after an NCCL all-gather.  `value` is queries/s of the whole
job from CUDA events (max over ranks); `e2e` is the same metric through the
public C ABI (circuit_search with host buffers) at N = 1, or the torch-level
equivalent with the NCCL merge at N > 1.  Inputs (19-154 GB per GPU) exceed the
126 MB L2, so no flush is needed between steps.  Every timed query is checked
against float64 brute force on the device.

`batched` (same line): --batch (4096) queries per step through
circuit_search_batch_async (2-SM tcgen05 tf32 filter GEMM with a rigorous error
band, exact fp32 rescoring), all-gather + per-query merge at N > 1.  Its
roofline is the scan kernel's tf32 rate against the dense tf32 peak derived
from the driver's measured bf16 GEMM rate.

`workloads` (N = 1, default workload): the other configurations measured after
the headline index is released: spread-200k single-query latency, the
clustered-50k pruning regime with its per-kernel split, the reference's own
exactness-test corpus (reftest-40k), clustered-4m, zipf-10m batches at k = 100,
and the 5,183-row flat path host-to-host.

`cpu_baseline`: the reference's CPU search path (brute force topk(X @ q),
circuit_rag/search.py:58-61; the oracle port) on a 12.5M-row sample of the same
workload, all host threads, timed before any GPU search runs.  `--impl
reference` times the same path as the reference arm (rank 0 only).
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "circuit-rag_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "queries/sec @k=10 on 100M x 384 fp32 (single-query exact search)"


def metric_name(n_total, dim, k):
    """The headline metric's wording for the workload actually run."""
    if (n_total, dim, k) == (100_000_000, 384, 10):
        return METRIC
    size = f"{n_total // 1_000_000}M" if n_total % 1_000_000 == 0 else str(n_total)
    return f"queries/sec @k={k} on {size} x {dim} fp32 (single-query exact search)"

# DRAM bytes (read + write) per algorithmic byte of the main leaf scan, from one
# ncu capture of that kernel on the 2,000,000-row case of this workload
# (3.0702 GB read + 4.19 MB written for 3.070 GB of scanned rows); the scan's
# traffic grows in proportion to the rows it reads, so a full launch is scaled by rows.
SCAN_TRAFFIC_PER_ALG_BYTE = 1.002
CPU_SAMPLE_ROWS = 12_500_000  # one eighth of the 100M corpus (the per-GPU shard at 8 GPUs)
TIE_ABS, SCORE_REL = 1e-6, 1e-5  # the parity rule: ids exact except ties within 1e-6, scores within 1e-5 rel


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="mixed-100m")
    ap.add_argument("--rows", type=int, default=0, help="total rows (default: the workload's N)")
    ap.add_argument("--e2e-steps", type=int, default=0)
    ap.add_argument("--cpu-queries", type=int, default=60, help="timed CPU-baseline queries (repo arm)")
    ap.add_argument("--cpu-queries-per-step", type=int, default=10, help="reference arm: queries per step")
    ap.add_argument("--cpu-rows", type=int, default=CPU_SAMPLE_ROWS)
    ap.add_argument("--batch", type=int, default=4096, help="queries per batch of the batched search (0: skip it)")
    ap.add_argument("--batch-steps", type=int, default=3)
    ap.add_argument("--batch-warmup", type=int, default=2)
    ap.add_argument("--batch-check", type=int, default=64, help="queries of the last batch checked in float64")
    ap.add_argument("--tf32-seconds", type=float, default=2.0, help="length of the in-process cuBLAS tf32 loop")
    ap.add_argument("--no-extra", action="store_true", help="skip the other workloads")
    ap.add_argument("--no-threshold-exchange", action="store_true",
                    help="N > 1: prune each shard with its own seed threshold only")
    ap.add_argument("--shared-threshold", action="store_true",
                    help="N > 1: also share the running threshold between the shards while their scans run "
                         "(circuit_search_finish_shared_async over CUDA IPC)")
    ap.add_argument("--no-seed-allreduce", action="store_true",
                    help="with --shared-threshold: skip the seed all-reduce, so each shard's bounds and scan "
                         "follow its own seed on the GPU and thresholds cross only through the shared words")
    return ap.parse_args()


def dist_setup(collectives=True):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and collectives:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local if world > 1 else 0)
    return world, rank, local


# ------------------------------------------------------------------ clocks and peaks
def clock_sampler(device_index):
    try:
        return subprocess.Popen(
            ["nvidia-smi", "-i", str(device_index),
             "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap",
             "--format=csv,noheader,nounits", "-lms", "100"],
            stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except OSError:
        return None


def clock_summary(proc):
    if proc is None:
        return None
    proc.terminate()
    try:
        out, _ = proc.communicate(timeout=5)
    except subprocess.TimeoutExpired:
        proc.kill()
        out, _ = proc.communicate()
    sm, mx, reasons = [], 0.0, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in out.strip().splitlines():
        f = [x.strip() for x in line.split(",")]
        if len(f) < 7:
            continue
        try:
            sm.append(float(f[0]))
            mx = max(mx, float(f[1]))
        except ValueError:
            continue
        for n, v in zip(names, f[3:7]):
            if v.lower() == "active":
                reasons.add(n)
    if not sm:
        return None
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    """(HBM GB/s, dense tf32 TFLOP/s, kind): the driver's measured copy bandwidth
    and half its sustained bf16 GEMM rate (tf32 runs at half the bf16 rate)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops_sustained"]) / 2.0, "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 700.0, "fallback"


def pctl(xs, q):
    xs = sorted(xs)
    return xs[min(len(xs) - 1, int(len(xs) * q))]


# ------------------------------------------------------------------ CPU baseline (reference CPU path)
def cpu_info():
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "threads": len(os.sched_getaffinity(0)), "loadavg": list(os.getloadavg())}


def cpu_sample(w, rows):
    """`rows` rows of the workload in host memory (generated on the GPU when
    there is one: the CPU generator would take minutes at this size)."""
    X = torch.empty((rows, w.dim), dtype=torch.float32, pin_memory=False)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    step = 1 << 20
    for a in range(0, rows, step):
        X[a:a + step] = w.corpus(a, min(rows, a + step), device=dev).cpu()
    return X


def cpu_baseline(w, n_total, rows, queries, k):
    """The reference CPU path (oracle port of circuit_rag/search.py:58-61),
    topk(X @ q) per query on a `rows`-row sample with every host thread;
    q/s scaled linearly to n_total rows (brute force is linear in rows)."""
    from oracle import oracle

    info = cpu_info()
    torch.set_num_threads(info["threads"])
    rows = min(rows, n_total)
    X = cpu_sample(w, rows)
    Q = w.query_batch(64, device="cpu")
    for j in range(3):  # warm pass (page-in, thread pool)
        oracle.torch_flat_search(X, Q[j], k)
    lat = []
    for j in range(queries):
        t0 = time.perf_counter()
        oracle.torch_flat_search(X, Q[j % len(Q)], k)
        lat.append(time.perf_counter() - t0)
    del X
    p50 = statistics.median(lat)
    scale = n_total / rows
    return {"value": 1.0 / (p50 * scale), "unit": "queries/s", "cores": info["threads"], "kind": "port",
            "sample": f"{rows} rows of the same workload, {queries} single queries after 3 warm ones, "
                      f"torch.topk(X @ q) on CPU ({info['cpu_model']}, {info['threads']} threads); "
                      f"per-query time scaled x{scale:.2f} to {n_total} rows",
            "p50_ms_on_sample": p50 * 1e3, "p99_ms_on_sample": pctl(lat, 0.99) * 1e3,
            "cpu_model": info["cpu_model"], "loadavg": info["loadavg"]}


def cpu_batched_baseline(w, n_total, rows, k, batch=256, reps=3):
    """The same brute force in batched form (Q @ X.T, topk per row) on a
    2M-row sample; queries/s scaled linearly to n_total rows."""
    from oracle import oracle

    info = cpu_info()
    torch.set_num_threads(info["threads"])
    rows = min(rows, n_total, 2_000_000)
    X = cpu_sample(w, rows)
    Q = w.query_batch(batch, device="cpu")
    oracle.torch_batch_flat_search(X, Q[:8], k)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.torch_batch_flat_search(X, Q, k)
        times.append(time.perf_counter() - t0)
    del X
    scale = n_total / rows
    return {"value": batch / (statistics.median(times) * scale), "unit": "queries/s", "cores": info["threads"],
            "kind": "port", "sample": f"{rows} rows, batches of {batch} x {reps}, torch.topk(Q @ X.T, k, dim=1) on "
                                      f"CPU; time scaled x{scale:.1f} to {n_total} rows"}


def run_reference(args, world, rank):
    """Reference arm: the reference's CPU search path (oracle port of
    circuit_rag/search.py:58-61) on this box's host cores.  A step is
    --cpu-queries-per-step single queries on the 12.5M-row sample."""
    from circuit_rag.synthetic import WORKLOADS
    from oracle import oracle

    if rank != 0:
        return
    w = WORKLOADS[args.workload]
    n_total = args.rows or w.n
    k = w.k
    info = cpu_info()
    torch.set_num_threads(info["threads"])
    rows = min(args.cpu_rows, n_total)
    X = cpu_sample(w, rows)
    Q = w.query_batch(64, device="cpu")
    per = args.cpu_queries_per_step
    lat, steps_ms = [], []
    j = 0
    for s in range(args.warmup + args.steps):
        t_step = time.perf_counter()
        for _ in range(per):
            t0 = time.perf_counter()
            oracle.torch_flat_search(X, Q[j % len(Q)], k)
            if s >= args.warmup:
                lat.append(time.perf_counter() - t0)
            j += 1
        if s >= args.warmup:
            steps_ms.append((time.perf_counter() - t_step) * 1e3)
    p50 = statistics.median(lat)
    scale = n_total / rows
    value = 1.0 / (p50 * scale)
    sample = (f"{rows} rows of the same workload; {args.steps} steps x {per} single queries (+{args.warmup} warm-up "
              f"steps), torch.topk(X @ q) on CPU ({info['cpu_model']}, {info['threads']} threads); per-query p50 "
              f"{p50 * 1e3:.1f} ms, p99 {pctl(lat, 0.99) * 1e3:.1f} ms on the sample, scaled x{scale:.2f} to "
              f"{n_total} rows")
    line = {
        "metric": metric_name(n_total, w.dim, k), "value": value, "unit": "queries/s", "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": statistics.mean(steps_ms), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": args.workload, "N": n_total, "D": w.dim, "k": k, "cpu_sample_rows": rows},
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": info["threads"], "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "p50_ms_on_sample": p50 * 1e3, "p99_ms_on_sample": pctl(lat, 0.99) * 1e3, "loadavg": info["loadavg"],
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ exactness (float64, on the device)
def exact_topk(leaf, ids, Q, k, extra=8):
    """float64 top-(k + extra) (scores, original ids) of every query over one
    index's rows, in one pass over the leaf rows."""
    kk = min(k + extra, leaf.shape[0])
    B = Q.shape[0]
    best_s = torch.full((B, kk), float("-inf"), dtype=torch.float64, device=leaf.device)
    best_i = torch.full((B, kk), -1, dtype=torch.int64, device=leaf.device)
    Qd = Q.double().T.contiguous()
    step = 1 << 20
    for a in range(0, leaf.shape[0], step):
        s = leaf[a:a + step].double() @ Qd
        v, r = torch.topk(s, min(kk, s.shape[0]), dim=0)
        cs = torch.cat([best_s, v.T], dim=1)
        ci = torch.cat([best_i, ids[a:a + step].long()[r].T], dim=1)
        t, o = torch.topk(cs, kk, dim=1)
        best_s, best_i = t, torch.gather(ci, 1, o)
    return best_s, best_i


def gather_exact(ex_s, ex_i, world):
    """Exact global top lists from every rank's local ones (N > 1)."""
    if world == 1:
        return ex_s, ex_i
    import torch.distributed as dist

    gs = [torch.empty_like(ex_s) for _ in range(world)]
    gi = [torch.empty_like(ex_i) for _ in range(world)]
    dist.all_gather(gs, ex_s)
    dist.all_gather(gi, ex_i)
    cs, ci = torch.cat(gs, dim=1), torch.cat(gi, dim=1)
    t, o = torch.topk(cs, ex_s.shape[1], dim=1)
    return t, torch.gather(ci, 1, o)


def count_mismatches(got_s, got_i, ex_s, ex_i, k):
    """Queries that break the parity rule: every id whose exact score is above
    the k-th by more than 1e-6 returned, no id below the k-th by more than
    1e-6, scores within 1e-5 relative (+1e-6) of exact, sorted, no duplicates.
    ex_s / ex_i are the exact top-(k + extra) lists; a returned id outside them
    scores at most their last entry, so it passes only where that last entry is
    still tied with the k-th (the list was cut inside a tie)."""
    got_s, got_i = got_s.cpu().numpy().astype(np.float64), got_i.cpu().numpy().astype(np.int64)
    ex_s, ex_i = ex_s.cpu().numpy(), ex_i.cpu().numpy()
    bad = 0
    for b in range(got_s.shape[0]):
        s, i, es, ei = got_s[b], got_i[b], ex_s[b], ex_i[b]
        kth = es[k - 1]
        ok = len(set(i.tolist())) == k and bool(np.all(np.diff(s) <= 0))
        ok = ok and set(ei[es > kth + TIE_ABS].tolist()) <= set(i.tolist())
        exact_of = dict(zip(ei.tolist(), es.tolist()))
        for sc, idv in zip(s, i):
            e = exact_of.get(int(idv))
            if e is None:
                ok = ok and es[-1] >= kth - TIE_ABS and sc >= kth - TIE_ABS - SCORE_REL * abs(kth)
            else:
                ok = ok and e >= kth - TIE_ABS and abs(sc - e) <= SCORE_REL * abs(e) + TIE_ABS
        bad += 0 if ok else 1
    return bad


# ------------------------------------------------------------------ single-query measurement
class Searcher:
    """One rank's single-query search (+ threshold exchange and all-gather
    merge at N > 1) on preallocated buffers."""

    _shared = None  # one SharedThreshold per process (its set-up is collective)

    def __init__(self, idx, k, world, exchange, dev, min_hier=0):
        from circuit_rag import _native

        self.min_hier = min_hier
        if exchange in ("shared", "running") and Searcher._shared is None:
            from circuit_rag.shard import SharedThreshold

            Searcher._shared = SharedThreshold(torch.device(dev), None)
        self.shared = Searcher._shared if exchange in ("shared", "running") else None
        self.L = _native.lib()
        self.h = idx.native_handle()
        self.k, self.world, self.exchange = k, world, exchange
        self.stream = torch.cuda.current_stream()
        self.s = torch.empty(k, device=dev)
        self.i = torch.empty(k, dtype=torch.int32, device=dev)
        self.T = torch.empty(1, device=dev)
        self.gs = torch.empty(world * k, device=dev) if world > 1 else None
        self.gi = torch.empty(world * k, dtype=torch.int32, device=dev) if world > 1 else None

    def local(self, q, e0=None, e1=None):
        from circuit_rag.search import _launch

        if not self.exchange:
            _launch(self.h, q, self.k, self.min_hier, self.s, self.i, None, self.stream, e0, e1)
            return
        import torch.distributed as dist

        assert self.L.circuit_search_seed_async(self.h, q.data_ptr(), self.k, self.T.data_ptr(),
                                                self.stream.cuda_stream) == 0
        if self.exchange != "running":
            dist.all_reduce(self.T, op=dist.ReduceOp.MAX)
        if self.shared is not None:
            sh = self.shared
            sh.tag = ((sh.tag + 1) & 0xFFFFFFFF) or 1
            assert self.L.circuit_search_finish_shared_async(
                self.h, q.data_ptr(), self.k, self.T.data_ptr(), sh.word.data_ptr(), sh.peers.data_ptr(), sh.n_peers,
                sh.tag, self.s.data_ptr(), self.i.data_ptr(), None, self.stream.cuda_stream,
                e0.cuda_event if e0 is not None else None, e1.cuda_event if e1 is not None else None) == 0
            return
        assert self.L.circuit_search_finish_async(self.h, q.data_ptr(), self.k, self.T.data_ptr(), self.s.data_ptr(),
                                                  self.i.data_ptr(), None, self.stream.cuda_stream,
                                                  e0.cuda_event if e0 is not None else None,
                                                  e1.cuda_event if e1 is not None else None) == 0

    def search(self, q, e0=None, e1=None):
        self.local(q, e0, e1)
        if self.world == 1:
            return self.s, self.i
        import torch.distributed as dist

        from circuit_rag.shard import merge_topk

        dist.all_gather_into_tensor(self.gs, self.s)
        dist.all_gather_into_tensor(self.gi, self.i)
        return merge_topk(self.gs, self.gi, self.k)


def single_query(idx, Q, k, warm, steps, world, exchange, dev, scan_events=True, min_hier=0):
    """Timed single queries: returns dict(value, p50, p99, scan_ms, main_rows,
    seed_rows, streamed_rows, scan_rows, out_s, out_i, elapsed_ms).

    scan_events: CUDA events around the main scan inside the timed loop.  An
    event between the bounds kernel and the main scan makes the scan wait for
    the bounds (it normally streams beside them), so the latency-bound
    workloads time the queries without them and time the scan in a separate
    pass.  main_rows = rows of the children that survive the seed threshold's
    bounds; streamed_rows = rows the pipelined scan read; scan_rows = rows the
    scans timed by scan_ms read."""
    import torch.distributed as dist

    from circuit_rag import _native

    se = Searcher(idx, k, world, exchange, dev, min_hier)
    stream = se.stream
    out_s = torch.empty((steps, k), device=dev)
    out_i = torch.empty((steps, k), dtype=torch.int32, device=dev)
    q_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    s_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for pair in s_ev:  # torch creates the CUDA event on first record; the C ABI records them afterwards
        for e in pair:
            e.record(stream)
    for j in range(warm):
        se.search(Q[j])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record(stream)
    for j in range(steps):
        q_ev[j][0].record(stream)
        rs, ri = se.search(Q[warm + j], *(s_ev[j] if scan_events else ()))
        out_s[j].copy_(rs)
        out_i[j].copy_(ri)
        q_ev[j][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([elapsed], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    lat = [a.elapsed_time(b) * 1000.0 for a, b in q_ev]
    scan_ms = [a.elapsed_time(b) for a, b in s_ev] if scan_events else None
    # rows per query: untimed replays with trace snapshots, with the scan events
    # (the mode scan_ms is measured in) and without them (the pipelined search)
    snap = torch.empty(_native.TRACE_SNAPSHOT_BYTES, dtype=torch.uint8, device=dev)
    main_rows, seed_rows, streamed_rows, scan_rows = [], [], [], []
    for with_events in (True, False):
        for j in range(steps):
            se.local(Q[warm + j], *(s_ev[j] if with_events else ()))  # (scan_ms is read already if timed)
            se.L.circuit_trace_snapshot_async(se.h, snap.data_ptr(), stream.cuda_stream)
            raw = snap.cpu().numpy().view(np.uint64)
            if with_events:
                scan_rows.append(int(raw[9] >> 32))
            else:
                seed_rows.append(int(raw[1] & 0xFFFFFFFF))
                main_rows.append(int(raw[2] & 0xFFFFFFFF))
                streamed_rows.append(int(raw[9] >> 32))
    if not scan_events:
        scan_ms = [a.elapsed_time(b) for a, b in s_ev]
    return {"value": steps / (elapsed / 1000.0), "elapsed_ms": elapsed, "p50_us": pctl(lat, 0.5),
            "p99_us": pctl(lat, 0.99), "scan_ms": scan_ms, "main_rows": main_rows, "seed_rows": seed_rows,
            "streamed_rows": streamed_rows, "scan_rows": scan_rows, "out_s": out_s, "out_i": out_i}


def phase_split(idx, Q, k, dev, n=20):
    """Per-kernel split of a single query from CUDA events between the kernels
    (root scan + seed sample | bounds | main scan + merge).  The events turn the
    programmatic dependent launches into full kernel boundaries, so the phases
    add up to more than the pipelined query."""
    from circuit_rag import _native

    L = _native.lib()
    h = idx.native_handle()
    st = torch.cuda.current_stream()
    s = torch.empty(k, device=dev)
    i = torch.empty(k, dtype=torch.int32, device=dev)
    T = torch.empty(1, device=dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n)]
    for e in ev:
        for x in e:
            x.record(st)
    torch.cuda.synchronize()
    for j in range(n):
        e = ev[j]
        e[0].record(st)
        assert L.circuit_search_seed_async(h, Q[j].data_ptr(), k, T.data_ptr(), st.cuda_stream) == 0
        e[1].record(st)
        assert L.circuit_search_finish_async(h, Q[j].data_ptr(), k, None, s.data_ptr(), i.data_ptr(), None,
                                             st.cuda_stream, e[2].cuda_event, e[3].cuda_event) == 0
    torch.cuda.synchronize()
    med = lambda f: round(statistics.median(f(e) for e in ev) * 1000.0, 2)  # noqa: E731
    return {"root_scan_and_seed_sample_us": med(lambda e: e[0].elapsed_time(e[1])),
            "bounds_us": med(lambda e: e[1].elapsed_time(e[2])),
            "main_scan_us": med(lambda e: e[2].elapsed_time(e[3])),
            "how": "CUDA events between the kernels (median of %d queries); the events serialise the kernels that "
                   "otherwise overlap through programmatic dependent launch" % n}


def host_to_host(idx, Q, k, n):
    """circuit_search (C ABI, host buffers, blocking) latency per query."""
    from circuit_rag import _native

    L = _native.lib()
    h = idx.native_handle()
    hq = np.ascontiguousarray(Q.cpu().numpy())
    hs = np.zeros(k, np.float32)
    hi = np.zeros(k, np.int32)
    for j in range(min(20, len(hq))):
        assert L.circuit_search(h, hq[j].ctypes.data, k, hs.ctypes.data, hi.ctypes.data, None) == 0
    lat = []
    t_all = time.perf_counter()
    for j in range(n):
        t0 = time.perf_counter()
        rc = L.circuit_search(h, hq[j % len(hq)].ctypes.data, k, hs.ctypes.data, hi.ctypes.data, None)
        lat.append(time.perf_counter() - t0)
        assert rc == 0, _native.last_error()
    total = time.perf_counter() - t_all
    return {"value": n / total, "unit": "queries/s", "p50_us": round(pctl(lat, 0.5) * 1e6, 2),
            "p99_us": round(pctl(lat, 0.99) * 1e6, 2), "h2d_bytes_per_step": hq.shape[1] * 4,
            "d2h_bytes_per_step": k * 8, "api": "circuit_search (C ABI, host buffers)"}


# ------------------------------------------------------------------ batched measurement
def tf32_gemm_in_process(dev, seconds=2.0):
    """cuBLAS tf32 8192^3 GEMM on this GPU: best of 5 (burst) and the mean of a
    back-to-back loop of about `seconds` (sustained)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    n = 8192
    a = torch.randn(n, n, device=dev)
    b = torch.randn(n, n, device=dev)
    c = torch.empty(n, n, device=dev)
    for _ in range(3):
        torch.matmul(a, b, out=c)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = 1e30
    for _ in range(5):
        e0.record()
        torch.matmul(a, b, out=c)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    reps = max(3, int(seconds * 1000.0 / best))
    e0.record()
    for _ in range(reps):
        torch.matmul(a, b, out=c)
    e1.record()
    torch.cuda.synchronize()
    mean = e0.elapsed_time(e1) / reps
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b, c
    torch.cuda.empty_cache()
    fl = 2.0 * n ** 3
    return fl / best / 1e9, fl / mean / 1e9


def batched(idx, QB, k, n_local, D, world, dev, warm, steps, n_check, tf32_seconds, cpu=None, e2e=True):
    """Batched exact search of QB [warm + steps, B, D]; every rank's shard,
    one all-gather of [B, k] and the per-query merge at N > 1."""
    import torch.distributed as dist

    from circuit_rag import _native
    from circuit_rag.search import _launch
    from circuit_rag.shard import merge_topk_batch

    L = _native.lib()
    handle = idx.native_handle()
    stream = torch.cuda.current_stream()
    Bq = QB.shape[1]
    s = torch.empty(Bq, k, device=dev)
    i = torch.empty(Bq, k, dtype=torch.int32, device=dev)
    gs = torch.empty(world * Bq, k, device=dev) if world > 1 else None
    gi = torch.empty(world * Bq, k, dtype=torch.int32, device=dev) if world > 1 else None
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for pair in ev:
        for e in pair:
            e.record(stream)
    n_over = ctypes.c_int(0)
    fallbacks = [0]
    res = [None]

    def step(j, timed):
        e0, e1 = ev[j - warm] if timed else (None, None)
        rc = L.circuit_search_batch_async(handle, QB[j].data_ptr(), Bq, k, s.data_ptr(), i.data_ptr(),
                                          stream.cuda_stream, e0.cuda_event if e0 else None,
                                          e1.cuda_event if e1 else None)
        assert rc == 0, _native.last_error()
        assert L.circuit_batch_overflow(handle, ctypes.byref(n_over)) == 0, _native.last_error()
        if n_over.value:
            for q in torch.nonzero(i[:, 0] == -2).flatten().tolist():
                _launch(handle, QB[j, q], k, 0, s[q], i[q], None, stream)
                fallbacks[0] += 1
        if world > 1:
            dist.all_gather_into_tensor(gs, s)
            dist.all_gather_into_tensor(gi, i)
            res[0] = merge_topk_batch(gs.view(world, Bq, k), gi.view(world, Bq, k), k)
        else:
            res[0] = (s, i)

    for j in range(warm):
        step(j, False)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    fallbacks[0] = 0
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for j in range(warm, warm + steps):
        step(j, True)
    t1.record(stream)
    torch.cuda.synchronize()
    elapsed = t0.elapsed_time(t1)
    scan_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    if world > 1:
        t = torch.tensor([elapsed, scan_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, scan_ms = float(t[0]), float(t[1])
    ms_s, ms_i = res[0]
    # exactness: the first n_check queries of the last timed batch against float64
    nc = min(n_check, Bq)
    Qc = QB[warm + steps - 1, :nc]
    ex_s, ex_i = gather_exact(*exact_topk(idx.leaf_vectors, idx.original_ids, Qc, k), world)
    bad = count_mismatches(ms_s[:nc], ms_i[:nc], ex_s, ex_i, k)
    out = {"value": round(Bq * steps / (elapsed / 1000.0), 1), "unit": "queries/s", "batch": Bq, "k": k,
           "steps": steps, "warmup": warm, "ms_per_batch": round(elapsed / steps, 3),
           "overflow_fallbacks": fallbacks[0], "check": {"checked_queries": nc, "mismatches": bad},
           "scan_ms": scan_ms}
    # end to end through the public API with host buffers
    if e2e and world == 1:
        hq = np.ascontiguousarray(QB[0].cpu().numpy())
        hs = np.zeros((Bq, k), np.float32)
        hi = np.zeros((Bq, k), np.int32)
        assert L.circuit_search_batch(handle, hq.ctypes.data, Bq, k, hs.ctypes.data, hi.ctypes.data) == 0
        tt = time.perf_counter()
        for _ in range(2):
            assert L.circuit_search_batch(handle, hq.ctypes.data, Bq, k, hs.ctypes.data, hi.ctypes.data) == 0
        out["e2e"] = {"value": round(2 * Bq / (time.perf_counter() - tt), 1), "unit": "queries/s",
                      "h2d_bytes_per_step": Bq * D * 4, "d2h_bytes_per_step": Bq * k * 8,
                      "api": "circuit_search_batch (C ABI, host buffers)"}
    elif e2e:
        hq = QB[0].cpu().pin_memory()
        hres_s = torch.empty(Bq, k, pin_memory=True)
        hres_i = torch.empty(Bq, k, dtype=torch.int32, pin_memory=True)
        dq = torch.empty(Bq, D, device=dev)
        torch.cuda.synchronize()
        dist.barrier()
        tt = time.perf_counter()
        for _ in range(2):
            dq.copy_(hq, non_blocking=True)
            assert L.circuit_search_batch_async(handle, dq.data_ptr(), Bq, k, s.data_ptr(), i.data_ptr(),
                                                stream.cuda_stream, None, None) == 0
            dist.all_gather_into_tensor(gs, s)
            dist.all_gather_into_tensor(gi, i)
            a, b = merge_topk_batch(gs.view(world, Bq, k), gi.view(world, Bq, k), k)
            hres_s.copy_(a, non_blocking=True)
            hres_i.copy_(b, non_blocking=True)
            torch.cuda.synchronize()
        t = torch.tensor([(time.perf_counter() - tt) / 2], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out["e2e"] = {"value": round(Bq / float(t.item()), 1), "unit": "queries/s", "h2d_bytes_per_step": Bq * D * 4,
                      "d2h_bytes_per_step": Bq * k * 8,
                      "api": "circuit_search_batch_async + NCCL all-gather + circuit_merge_topk_batch"}
    _, tf32_peak, kind = measured_peaks()
    flops = 2.0 * Bq * n_local * D
    achieved = flops / (scan_ms * 1e-3) / 1e12
    roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(tf32_peak, 1), "unit": "TFLOP/s",
            "frac": round(achieved / tf32_peak, 4),
            "peak_kind": f"{kind}: dense tf32 = half of MEASURED_PEAKS bf16_tflops_sustained",
            "peak_nominal": 1125.0, "frac_of_nominal": round(achieved / 1125.0, 4),
            "kernel": "k_batch_scan (2-SM tcgen05 kind::tf32 filter GEMM, fused candidate epilogue)",
            "algorithmic_flops_per_launch": flops, "mean_launch_ms": round(scan_ms, 3)}
    if tf32_seconds > 0:
        burst, sust = tf32_gemm_in_process(dev, tf32_seconds)
        roof["side_in_process_cublas_tf32"] = {"burst": round(burst, 1), "sustained": round(sust, 1),
                                               "frac_of_sustained": round(achieved / sust, 4)}
    out["roofline"] = roof
    out["gpu_launches_per_step"] = 8 + (1 if world > 1 else 0)
    if cpu is not None:
        out["cpu_baseline"] = cpu
    return out


# ------------------------------------------------------------------ other workloads (N = 1)
def other_workloads(dev, hbm_peak):
    from circuit_rag import build_circuit_index
    from circuit_rag.synthetic import WORKLOADS

    out = {}
    for name, n_q, flat in (("spread-200k", 300, False), ("clustered-50k", 300, False), ("reftest-40k", 300, False),
                            ("clustered-4m", 100, False), ("spread-5k", 300, True)):
        w = WORKLOADS[name]
        X = w.corpus(0, w.n, device=dev)
        idx = build_circuit_index(X, num_roots=w.num_roots, children_per_root=w.children_per_root, rank=w.rank,
                                  device=dev)
        Q = w.query_batch(n_q + 20, device=dev)
        r = {"N": w.n, "D": w.dim, "k": w.k, "num_roots": w.num_roots, "children_per_root": w.children_per_root,
             "rank": w.rank}
        if not flat:
            sq = single_query(idx, Q, w.k, 20, n_q, 1, False, dev, scan_events=False)
            ex_s, ex_i = exact_topk(idx.leaf_vectors, idx.original_ids, Q[20:20 + n_q], w.k)
            bad = count_mismatches(sq["out_s"], sq["out_i"], ex_s, ex_i, w.k)
            # the same queries through the flat scan (no bounds): where pruning pays
            fq = single_query(idx, Q, w.k, 20, n_q, 1, False, dev, scan_events=False, min_hier=1 << 40)
            bad += count_mismatches(fq["out_s"], fq["out_i"], ex_s, ex_i, w.k)
            mean_rows = statistics.mean(sq["main_rows"])
            scan = statistics.mean(sq["scan_ms"])
            scan_rows = statistics.mean(sq["scan_rows"])
            leaf_bytes = mean_rows * w.dim * 4
            R, C, D, rk = idx.num_roots, idx.num_total_children, w.dim, w.rank
            meta_bytes = 4 * R * D + 4 * R * D * rk + 4 * C * (2 * rk + 2) + statistics.mean(sq["seed_rows"]) * D * 4
            r.update({"single_query_qps": round(sq["value"], 1), "p50_us": round(sq["p50_us"], 2),
                      "p99_us": round(sq["p99_us"], 2),
                      "flat_scan": {"p50_us": round(fq["p50_us"], 2), "p99_us": round(fq["p99_us"], 2)},
                      "pruned_leaf_fraction": round(1 - mean_rows / w.n, 5),
                      "rows_streamed_fraction": round(statistics.mean(sq["streamed_rows"]) / w.n, 5),
                      "main_scan": {"rows": scan_rows, "mean_launch_us": round(scan * 1000, 2),
                                    "frac_of_hbm": round(scan_rows * w.dim * 4 / (scan * 1e-3) / 1e9 / hbm_peak, 4),
                                    "timed": "alone, after the bounds (events around it)"},
                      "query_roofline": {"bytes": round(leaf_bytes + meta_bytes),
                                         "leaf_bytes": round(leaf_bytes), "bound_metadata_bytes": round(meta_bytes),
                                         "frac_of_hbm_at_p50": round((leaf_bytes + meta_bytes) / (sq["p50_us"] * 1e-6)
                                                                     / 1e9 / hbm_peak, 4)},
                      "phase_split": phase_split(idx, Q, w.k, dev),
                      "check": {"checked_queries": 2 * n_q, "mismatches": bad,
                                "how": "float64 brute force on the device, hierarchical and flat"}})
        r["host_to_host"] = host_to_host(idx, Q, w.k, 2000)
        out[name] = r
        idx.close()
        del idx, X
        torch.cuda.empty_cache()
    # zipf-10m: batches of 1,024 at k = 100, and single queries at k = 100
    from circuit_rag.hierarchy.build import build_circuit_index_streaming

    w = WORKLOADS["zipf-10m"]
    idx = build_circuit_index_streaming(lambda s_, e_: w.corpus(s_, e_, device=dev), w.n, w.dim, w.num_roots,
                                        w.children_per_root, w.rank, device=dev)
    QB = w.query_batch(1024 * 5, device=dev).view(5, 1024, w.dim)
    b = batched(idx, QB, w.k, w.n, w.dim, 1, dev, 2, 3, 64, 0.0, e2e=False)
    Q1 = w.query_batch(40, device=dev)
    sq = single_query(idx, Q1, w.k, 5, 30, 1, False, dev, scan_events=False)
    ex_s, ex_i = exact_topk(idx.leaf_vectors, idx.original_ids, Q1[5:35], w.k)
    out["zipf-10m"] = {"N": w.n, "D": w.dim, "k": w.k, "num_roots": w.num_roots,
                       "children_per_root": w.children_per_root, "rank": w.rank,
                       "batched": {kk: b[kk] for kk in ("value", "unit", "batch", "ms_per_batch", "overflow_fallbacks",
                                                        "check", "roofline")},
                       "single_query": {"qps": round(sq["value"], 1), "p50_us": round(sq["p50_us"], 1),
                                        "p99_us": round(sq["p99_us"], 1),
                                        "pruned_leaf_fraction": round(1 - statistics.mean(sq["main_rows"]) / w.n, 5),
                                        "rows_streamed_fraction": round(statistics.mean(sq["streamed_rows"]) / w.n,
                                                                        5),
                                        "check": {"checked_queries": 30,
                                                  "mismatches": count_mismatches(sq["out_s"], sq["out_i"], ex_s, ex_i,
                                                                                 w.k)}}}
    idx.close()
    return out


# ------------------------------------------------------------------ main
def main():
    args = parse()
    world, rank, local = dist_setup(collectives=args.impl == "ours")
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    import torch.distributed as dist

    from circuit_rag.hierarchy.build import build_circuit_index_streaming
    from circuit_rag.synthetic import WORKLOADS

    dev = torch.device("cuda", torch.cuda.current_device())
    w = WORKLOADS[args.workload]
    n_total = args.rows or w.n
    k, D = w.k, w.dim

    # the CPU baseline runs first, before any search loads the GPU or the host
    cpu = cpu_b = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline(w, n_total, args.cpu_rows, args.cpu_queries, k)
        if args.batch > 0:
            cpu_b = cpu_batched_baseline(w, n_total, args.cpu_rows, k)

    t0 = time.time()
    idx = build_circuit_index_streaming(lambda s, e: w.corpus(s, e, device=dev), n_total, D, w.num_roots,
                                        w.children_per_root, w.rank, device=dev, shard_rank=rank, world=world)
    torch.cuda.synchronize()
    build_s = time.time() - t0
    info = idx.shard_info
    n_local = idx.N
    exchange = world > 1 and not args.no_threshold_exchange
    if exchange and args.shared_threshold:
        exchange = "running" if args.no_seed_allreduce else "shared"

    steps, warm = args.steps, args.warmup
    Q = w.query_batch(steps + warm, device=dev)
    # clocks: sampled by nvidia-smi every 100 ms from just before the single-query
    # warm-up to the end of the batched timing (at 8 GPUs the single-query timed
    # region alone is shorter than one sampling interval)
    clk_proc = None
    if rank == 0:
        clk_proc = clock_sampler(local)
        time.sleep(0.5)  # nvidia-smi is up and sampling before the first timed launch
    sq = single_query(idx, Q, k, warm, steps, world, exchange, dev)
    ex_s, ex_i = gather_exact(*exact_topk(idx.leaf_vectors, idx.original_ids, Q[warm:], k), world)
    check = {"checked_queries": steps, "mismatches": count_mismatches(sq["out_s"], sq["out_i"], ex_s, ex_i, k),
             "how": "float64 brute force on the device" + (" per shard, gathered" if world > 1 else "")}

    # per-phase timing of the sharded query (untimed pass; events per phase)
    phases = None
    if world > 1:
        se = Searcher(idx, k, world, exchange, dev)
        st = torch.cuda.current_stream()
        evs = []
        for j in range(min(steps, 20)):
            e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            e[0].record(st)
            se.local(Q[warm + j])
            e[1].record(st)
            dist.all_gather_into_tensor(se.gs, se.s)
            dist.all_gather_into_tensor(se.gi, se.i)
            e[2].record(st)
            from circuit_rag.shard import merge_topk

            merge_topk(se.gs, se.gi, k)
            e[3].record(st)
            evs.append(e)
        torch.cuda.synchronize()
        loc = statistics.median(e[0].elapsed_time(e[1]) for e in evs)
        ag = statistics.median(e[1].elapsed_time(e[2]) for e in evs)
        mg = statistics.median(e[2].elapsed_time(e[3]) for e in evs)
        t = torch.tensor([loc, ag, mg], device=dev)
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tmin = t.clone()
        dist.all_reduce(tmin, op=dist.ReduceOp.MIN)
        phases = {"local_search_ms_max_min": [round(float(tmax[0]), 4), round(float(tmin[0]), 4)],
                  "all_gather_ms_max": round(float(tmax[1]), 4), "merge_ms_max": round(float(tmax[2]), 4),
                  "how": "median of 20 untimed queries per rank; local search includes the seed all-reduce "
                         "(when one runs)"}

    # e2e through the public API
    e2e_steps = args.e2e_steps or min(steps, 50)
    if world == 1:
        e2e = host_to_host(idx, Q[warm:warm + e2e_steps], k, e2e_steps)
    else:
        se = Searcher(idx, k, world, exchange, dev)
        hq = Q[warm:warm + e2e_steps].cpu().pin_memory()
        hres = torch.empty((2, k), pin_memory=True)
        dq = torch.empty(D, device=dev)
        torch.cuda.synchronize()
        dist.barrier()
        tt = time.perf_counter()
        for j in range(e2e_steps):
            dq.copy_(hq[j], non_blocking=True)
            ms, mi = se.search(dq)
            if rank == 0:
                hres[0].copy_(ms, non_blocking=True)
                hres[1].copy_(mi.float(), non_blocking=True)
            torch.cuda.synchronize()
        t = torch.tensor([time.perf_counter() - tt], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e = {"value": e2e_steps / float(t.item()), "unit": "queries/s", "h2d_bytes_per_step": D * 4,
               "d2h_bytes_per_step": k * 8,
               "api": {False: "circuit_search_async",
                       True: "circuit_search_seed_async + NCCL all-reduce(MAX) + circuit_search_finish_async",
                       "shared": "circuit_search_seed_async + NCCL all-reduce(MAX) + "
                                 "circuit_search_finish_shared_async",
                       "running": "circuit_search_seed_async + circuit_search_finish_shared_async"}[exchange]
               + " + NCCL all-gather + circuit_merge_topk"}

    bat = None
    if args.batch > 0:
        Bq, bw, bs = args.batch, max(1, args.batch_warmup), args.batch_steps
        QB = w.query_batch(Bq * (bw + bs), device=dev).view(bw + bs, Bq, D)
        bat = batched(idx, QB, k, n_local, D, world, dev, bw, bs, args.batch_check, 0.0, cpu=cpu_b)
        del QB
    clocks = clock_summary(clk_proc)
    if clocks:
        clocks["window"] = "single-query warm-up to the end of the batched timing, 100 ms samples"
    if bat is not None and args.tf32_seconds > 0:
        burst, sust = tf32_gemm_in_process(dev, args.tf32_seconds)
        roof = bat["roofline"]
        roof["side_in_process_cublas_tf32"] = {"burst": round(burst, 1), "sustained": round(sust, 1),
                                               "frac_of_sustained": round(roof["achieved"] / sust, 4)}

    hbm_peak, _, peak_kind = measured_peaks()
    mean_scan_ms = statistics.mean(sq["scan_ms"])
    mean_rows = statistics.mean(sq["scan_rows"])  # rows the timed scans read
    alg_bytes = mean_rows * D * 4
    achieved = alg_bytes / (mean_scan_ms * 1e-3) / 1e9
    if world > 1:
        t = torch.tensor([achieved], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        achieved_min = float(t.item())
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
            "frac_of_nominal_8000": round(achieved / 8000.0, 4),
            "traffic": round(alg_bytes * SCAN_TRAFFIC_PER_ALG_BYTE),
            "traffic_source": "ncu capture of the main scan on 2M rows, scaled by rows scanned",
            "kernel": "k_scan (main leaf scan, fused top-k)",
            "algorithmic_bytes_per_launch": alg_bytes, "mean_launch_ms": mean_scan_ms}
    if world > 1:
        roof["frac_min_over_ranks"] = round(achieved_min / hbm_peak, 4)

    rows_all = [n_local]
    if world > 1:
        t = torch.tensor([n_local], device=dev, dtype=torch.int64)
        g = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(g, t)
        rows_all = [int(x.item()) for x in g]
    idx.close()
    del idx
    import gc

    gc.collect()
    torch.cuda.empty_cache()

    extra = None
    if rank == 0 and world == 1 and not args.no_extra and args.workload == "mixed-100m" and not args.rows:
        extra = other_workloads(dev, hbm_peak)

    if rank == 0:
        value = steps / (sq["elapsed_ms"] / 1000.0)
        line = {
            "metric": metric_name(n_total, D, k), "value": round(value, 3), "unit": "queries/s", "n_gpus": world,
            "steps": steps,
            "warmup": warm, "ms_per_step": round(sq["elapsed_ms"] / steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "N": n_total, "D": D, "k": k, "num_roots": w.num_roots,
                       "children_per_root": w.children_per_root, "rank": w.rank, "rows_per_gpu": rows_all,
                       "parallelism": f"root-cluster shards x{world}", "l2": "inputs larger than L2, no flush needed"},
            "p50_us": round(sq["p50_us"], 2), "p99_us": round(sq["p99_us"], 2),
            "pruned_leaf_fraction": round(1.0 - statistics.mean(sq["main_rows"]) / n_local, 5),
            "rows_streamed_fraction": round(statistics.mean(sq["streamed_rows"]) / n_local, 5),
            "roofline": roof, "cpu_baseline": ({kk: cpu[kk] for kk in ("value", "unit", "cores", "kind", "sample")}
                                               if cpu else None),
            "e2e": e2e, "gpu_launches": (4 if world == 1 else 5) * steps, "clocks": clocks, "build_s": round(build_s, 1),
            "check": check, "threshold_exchange": exchange, "batched": bat,
            "shards": {"rows": rows_all, "max_over_mean": round(max(rows_all) / statistics.mean(rows_all), 4),
                       "parts_total": info["parts_total"], "roots": info["roots"]},
        }
        if cpu:
            line["cpu_baseline_detail"] = {kk: cpu[kk] for kk in ("p50_ms_on_sample", "p99_ms_on_sample", "cpu_model",
                                                                  "loadavg")}
        if phases:
            line["phases"] = phases
        if extra:
            line["workloads"] = extra
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
