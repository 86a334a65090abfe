#!/usr/bin/env python
"""Benchmark: batched IVF-PQ search QPS at recall@10 on the B200 engine.

One step = one batched search of the configuration's query batch on every
rank.  `value` runs with queries and results resident in HBM; `e2e` goes
through the same C-ABI call with pinned host buffers (host->device copy of the
queries and device->host copy of the results inside every timed step).  L2 is
flushed between timed steps: a 512 MiB write, then a 512 MiB read of another
buffer so that the flush's own dirty lines are written back before the timed
step starts rather than inside it.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl engine|reference]

The default workload is configuration 3 (1e7 vectors, 4-bit codes, inverted
lists sharded by list across 1/2/4/8 GPUs).  N > 1 runs under torchrun, one
rank per GPU: every rank builds the same index (training is deterministic),
keeps only the lists it owns (vg_ivfpq_shard) and searches a batch of its own
(the configuration's batch size per rank: weak scaling); the ranks exchange
queries, probes, a pruning seed and per-rank top-k over NCCL.  value = all
ranks' queries / the slowest rank's device time.  --shard queries instead
keeps a whole index replica per rank (no collective on the data path).
Configuration 2 (exact flat search) runs the flat index on the same contract.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "IVF-PQ queries/sec at recall@10 (1/2/4/8 B200); ADC scan HBM GB/s vs peak"
FALLBACK_HBM_GBS = 6650.0
RECALL_QUERIES = 1000  # both arms report recall@10 on the batch's first 1,000 queries


def workload_config(cfg, nq: int, train_sample: int, train_iters: int) -> dict:
    """The workload, identical in the engine and reference lines."""
    if cfg["centre"] == "flat":
        return {"workload": cfg["name"], "n": cfg["n"], "d": cfg["d"], "k": cfg["k"], "batch_per_rank": nq,
                "l2": "not flushed: the database (400 MB of f32 rows, 256 MB binary16 image) exceeds L2"}
    return {"workload": cfg["name"], "n": cfg["n"], "d": cfg["d"], "nlist": cfg["nlist"], "M": cfg["M"],
            "codebook_size": cfg["ks"], "nprobe": cfg["nprobe"], "k": cfg["k"], "batch_per_rank": nq,
            "train_sample": train_sample, "train_iters": train_iters,
            "training": "seeded sample, spherical Lloyd (lists) + Euclidean Lloyd per subspace, to convergence "
                        "or train_iters",
            "l2": "flushed between the GPU arm's timed steps (512 MiB write, then 512 MiB read of another buffer)"}


def exact_top_k_cpu(xn: np.ndarray, q: np.ndarray, k: int) -> np.ndarray:
    """Exact top-k rows of normalised `xn` by inner product with the
    normalised queries (CPU matmul in blocks): the recall ground truth."""
    import torch

    qs = q / np.maximum(np.linalg.norm(q, axis=1, keepdims=True), 1e-30)
    qt = torch.from_numpy(np.ascontiguousarray(qs.astype(np.float32)).T.copy())
    best_v = torch.full((q.shape[0], k), -1e30)
    best_i = torch.zeros((q.shape[0], k), dtype=torch.int64)
    for s0 in range(0, xn.shape[0], 1 << 20):
        sc = torch.from_numpy(xn[s0:s0 + (1 << 20)]) @ qt
        v, i = torch.topk(sc, min(k, sc.shape[0]), dim=0)
        allv = torch.cat([best_v, v.T], dim=1)
        alli = torch.cat([best_i, (i + s0).T], dim=1)
        top = torch.topk(allv, k, dim=1)
        best_v, best_i = top.values, torch.gather(alli, 1, top.indices)
    return best_i.numpy()


def recall_at_k(ids: np.ndarray, counts, truth: np.ndarray) -> float:
    """Mean |returned ∩ true top-k| / k over the rows of `truth`."""
    k = truth.shape[1]
    hits = 0
    for r in range(truth.shape[0]):
        c = k if counts is None else int(counts[r])
        hits += len(set(ids[r, :c].tolist()) & set(truth[r].tolist()))
    return hits / truth.size


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", type=int, default=3)
    p.add_argument("--impl", choices=["engine", "reference"], default="engine")
    p.add_argument("--train-sample", type=int, default=None,
                   help="k-means training rows (default: the configuration's, else 131072; at most n)")
    p.add_argument("--train-iters", type=int, default=20)
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--nq", type=int, default=None, help="query batch (default: the configuration's)")
    p.add_argument("--n", type=int, default=None,
                   help="database vectors (default: the configuration's; smaller only for profiler captures)")
    p.add_argument("--shard", choices=["queries", "lists"], default="lists",
                   help="multi-GPU layout: inverted lists sharded by list (default), or index replicas")
    return p.parse_args()


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except Exception:
            pass
    return {"hbm_gbs": FALLBACK_HBM_GBS}, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons sampled every 10 ms during the timed steps.

    Sampled in-process through NVML (the library nvidia-smi reads): an
    nvidia-smi process polling every 50 ms stalled this GPU for ~90 ms now
    and then inside timed steps, the same queries made in-process did not.
    Falls back to nvidia-smi when NVML bindings are missing.  Only samples
    taken between begin() and end() are reported; the 10 ms period leaves
    several inside even a timed region of a few tens of milliseconds.
    """

    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int):
        self.device = device
        self.rows: list[tuple[float, float, float, int]] = []  # (time, sm MHz, max MHz, reason mask)
        self.window = (0.0, float("inf"))
        self.source = None
        self._stop = threading.Event()
        self.thread = None
        self.proc = None

    def start(self):
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(self.device).uuid)
                h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.device)

            def loop():
                while not self._stop.is_set():
                    try:
                        self.rows.append((time.monotonic(),
                                          float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                          float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                          int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))))
                    except Exception:
                        pass
                    self._stop.wait(0.01)

            self.source = "nvml"
            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-lms", "50", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except FileNotFoundError:
            return
        self.source = "nvidia-smi"

        def read():
            for line in self.proc.stdout:
                c = [x.strip() for x in line.split(",")]
                try:
                    self.rows.append((time.monotonic(), float(c[0]), float(c[1]), int(c[2], 16)))
                except (ValueError, IndexError):
                    pass

        self.thread = threading.Thread(target=read, daemon=True)
        self.thread.start()

    def wait_ready(self, samples: int = 10, timeout_s: float = 15.0):
        """Block until the sampler has delivered `samples` rows (start-up before
        any measured work)."""
        deadline = time.monotonic() + timeout_s
        while self.source and len(self.rows) < samples and time.monotonic() < deadline:
            time.sleep(0.05)

    def begin(self):
        self.window = (time.monotonic(), float("inf"))

    def end(self):
        self.window = (self.window[0], time.monotonic() + 0.012)

    def stop(self) -> dict:
        if not self.source:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        lo, hi = self.window
        rows = [r for r in self.rows if lo <= r[0] <= hi]
        reasons = sorted({name for r in rows for name, bit in self.REASON_BITS.items() if r[3] & bit})
        return {"sm_mhz": statistics.median(r[1] for r in rows) if rows else None,
                "sm_max_mhz": max(r[2] for r in rows) if rows else None,
                "reasons": reasons, "samples": len(rows), "source": self.source}


# --------------------------------------------------------------------------
# engine arm
# --------------------------------------------------------------------------

def run_engine(args):
    import torch
    import torch.distributed as dist

    from vicinity_b200 import FlatIndex, IVFPQIndex, _lib, nccl_unique_id
    from vicinity_b200.synthetic import CONFIGS, config_data

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo", timeout=timedelta(seconds=900))

    cfg = CONFIGS[args.config]
    if cfg["centre"] == "flat":
        return run_flat(args, cfg, world, rank, local)
    n, d, k = args.n or cfg["n"], cfg["d"], cfg["k"]
    nq = args.nq or cfg["nq"]
    train_sample = min(args.train_sample or cfg.get("train_sample", 131_072), n)
    on_device = cfg.get("generated") == "device"
    by_lists = world > 1 and args.shard == "lists"
    t0 = time.time()
    ix = IVFPQIndex(d, num_clusters=cfg["nlist"], num_codebooks=cfg["M"], codebook_size=cfg["ks"],
                    nprobe=cfg["nprobe"], seed=42, device=local)
    # every rank searches a batch of its own: rows [rank*nq, (rank+1)*nq) of
    # the configuration's query stream (rank 0's batch is the one-GPU batch)
    x = None
    if on_device:  # the database is drawn on the GPU chunk by chunk and never held on the host
        from vicinity_b200.synthetic import device_mixture

        _, chunks, q_all = device_mixture(args.config, seed=0, device=local, n=n, nq=nq * world)
        for xc in chunks:
            torch.cuda.synchronize()  # the chunk is complete before the engine's stream reads it
            ix.add_device(xc.data_ptr(), xc.shape[0])
            del xc
        torch.cuda.empty_cache()
    else:
        x, q_all = config_data(args.config, seed=0, n=n, nq=nq * world)
        ix.add_items(x)
    q = np.ascontiguousarray(q_all[rank * nq:(rank + 1) * nq])
    ix.build(training_sample_size=train_sample, kmeans_max_iter=args.train_iters)
    build_s = time.time() - t0

    # exact top-k of this rank's normalised queries over the normalised
    # database (engine flat search), for recall@10; before any vectors are dropped
    rq = nq if not on_device else min(nq, 1000)
    vec_d = torch.empty((n, d), dtype=torch.float32, device="cuda")
    _lib.check(ix._lib.vg_ivfpq_export(ix.handle, _lib.EXPORT_VECTORS, vec_d.data_ptr(), vec_d.numel() * 4))
    qn = q[:rq] / np.maximum(np.linalg.norm(q[:rq], axis=1, keepdims=True), 1e-30)
    flat = FlatIndex.from_device(vec_d.data_ptr(), n, d, device=local)
    truth, _ = flat.search(qn.astype(np.float32), k)
    flat.close()
    del vec_d
    torch.cuda.empty_cache()

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and x is not None:
        cpu_baseline = cpu_baseline_port(ix, x, q, cfg, args.cpu_seconds, truth)
    unsharded = ix.batch_search(q, k)[0] if by_lists and rank == 0 else None
    ix.compact()  # codes and ids stay resident; the raw vectors are dropped
    bytes_full = int(ix.info().device_bytes)
    if by_lists:
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ix.shard(rank, world, obj[0], timeout_ms=120_000)
    bytes_rank = int(ix.info().device_bytes)
    queries_total = nq * world  # queries all ranks answer per step

    # One explicit stream carries everything timed: the L2 flush, the CUDA
    # events and the engine's kernels (torch's default stream has handle 0,
    # which the engine reads as "use the index's own stream", unordered with it).
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    assert stream.cuda_stream != 0
    ix.set_stream(stream.cuda_stream)
    qd = torch.from_numpy(q).cuda()
    ids_d = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    dist_d = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    cnt_d = torch.empty((nq,), dtype=torch.int32, device="cuda")
    flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
    flush_read = torch.zeros((512 << 20) // 4, dtype=torch.float32, device="cuda")
    flush_sink = torch.empty((), dtype=torch.float32, device="cuda")

    def step_device():
        ix.search_raw(qd.data_ptr(), nq, k, 0, ids_d.data_ptr(), dist_d.data_ptr(), cnt_d.data_ptr())

    def barrier():
        if world > 1:
            dist.barrier()

    def reduce(v: float, op) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=op)
        return float(t.item())

    def timed(step, steps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        barrier()
        torch.cuda.synchronize()
        for a, b in evs:
            flush.zero_()  # L2 flush between timed steps (not timed) ...
            torch.amax(flush_read, dim=0, out=flush_sink)  # ... leaving no dirty lines behind
            a.record(stream)
            step()
            b.record(stream)
        torch.cuda.synchronize()
        barrier()
        return sum(a.elapsed_time(b) for a, b in evs)

    clocks = ClockSampler(local)
    clocks.start()
    clocks.wait_ready()
    # warm-up runs the timed loop itself (flush, read sweep, events, search with
    # profiling on) so that first-use costs -- lazy loading of every kernel the
    # timed steps launch included -- fall outside the timed steps
    ix.set_profiling(True)
    timed(step_device, args.warmup)
    ix.reset_profile()
    clocks.begin()
    dev_ms = timed(step_device, args.steps)
    clocks.end()
    clock_info = clocks.stop()
    prof = ix.profile()
    ix.set_profiling(False)
    dev_ms_max = reduce(dev_ms, dist.ReduceOp.MAX if world > 1 else None)
    value = queries_total * args.steps / (dev_ms_max / 1e3)
    shard_check = None
    if unsharded is not None:
        got = ids_d.cpu().numpy().astype(np.int64)
        got[np.arange(k)[None, :] >= cnt_d.cpu().numpy().astype(np.int64)[:, None]] = -1
        shard_check = {"rows": int(nq), "identical_to_unsharded_search": bool(np.array_equal(got, unsharded))}

    # end to end through the same call with pinned host buffers
    q_h = torch.from_numpy(q).pin_memory()
    ids_h = torch.empty((nq, k), dtype=torch.int32).pin_memory()
    dist_h = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    cnt_h = torch.empty((nq,), dtype=torch.int32).pin_memory()

    def step_e2e():
        ix.search_raw(q_h.data_ptr(), nq, k, 0, ids_h.data_ptr(), dist_h.data_ptr(), cnt_h.data_ptr())

    timed(step_e2e, max(1, args.warmup // 2))
    e2e_ms = reduce(timed(step_e2e, args.steps), dist.ReduceOp.MAX if world > 1 else None)
    e2e_value = queries_total * args.steps / (e2e_ms / 1e3)

    # recall@10 of this rank's rows, averaged over ranks: on the first
    # RECALL_QUERIES queries (the reference arm's recall queries at N = 1) and
    # on every row with a ground truth
    got = ids_h.numpy()[:rq].astype(np.int64)
    rs = min(RECALL_QUERIES, rq)
    recall = reduce(recall_at_k(got[:rs], None, truth[:rs]), dist.ReduceOp.SUM if world > 1 else None) / world
    recall_batch = reduce(recall_at_k(got, None, truth), dist.ReduceOp.SUM if world > 1 else None) / world

    # roofline of the scan kernel (live CUDA events on the launching stream)
    peaks, peak_kind = measured_peaks()
    calls = max(1, int(prof["calls"]))
    scan_ms = prof["scan_ms"] / calls
    scan_bytes = prof["scanned_code_bytes"] / calls
    achieved = scan_bytes / (scan_ms * 1e-3) / 1e9 if scan_ms > 0 else 0.0
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    # what the kernel actually scored: lists left after exact pruning (0 when
    # the kernel that ran does not count them)
    code_bytes = cfg["M"] if cfg["ks"] == 256 else (cfg["M"] + 1) // 2
    scored_vecs = prof["scored_vectors"] / calls
    probed_vecs = prof["scanned_vectors"] / calls
    scored_bytes = scored_vecs * code_bytes if scored_vecs > 0 else None
    traffic = scan_traffic_from_profiles(args.config)
    scored_gbs = None if scored_bytes is None else scored_bytes / (scan_ms * 1e-3) / 1e9

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "queries/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_ms_max / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": ("synthetic: seeded Gaussian mixture drawn on the GPU chunk by chunk (torch generator), "
                     "never held on the host" if on_device else
                     "synthetic: seeded Gaussian mixture with the configuration's generator (no dataset)"),
            "config": workload_config(cfg, nq, train_sample, args.train_iters),
            "recall_at_10": round(recall, 4),
            "recall_queries": rs,
            "recall_at_10_batch": round(recall_batch, 4),
            "recall_queries_batch": rq,
            "parallelism": ("single GPU" if world == 1 else
                            f"inverted lists sharded by list x{world}, {nq} queries per rank" if by_lists
                            else f"index replica per GPU, {nq} queries per rank x{world}"),
            "index_bytes_one_gpu": bytes_full, "index_bytes_per_rank": bytes_rank,
            "index_build_s": round(build_s, 1),
            "e2e": {"value": round(e2e_value, 1), "unit": "queries/s",
                    "h2d_bytes_per_step": nq * d * 4, "d2h_bytes_per_step": nq * k * 8 + nq * 4},
            "roofline": {
                "kernel": "ivfpq scan (fused residual + ADC + code scan + top-k; warp per query at this batch)",
                "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_kind,
                "algorithmic_bytes_per_launch": int(scan_bytes), "launch_ms": round(scan_ms, 4),
                "scored_bytes_per_launch": None if scored_bytes is None else int(scored_bytes),
                "scored_gbs": None if scored_gbs is None else round(scored_gbs, 1),
                "scored_frac": None if scored_gbs is None else round(scored_gbs / peak, 4),
                "dram_frac": None if traffic is None or scan_ms <= 0 else round(
                    traffic / (scan_ms * 1e-3) / 1e9 / peak, 4),
                "pruned_fraction": None if scored_bytes is None or probed_vecs <= 0
                else round(1.0 - scored_vecs / probed_vecs, 4),
                "note": ("algorithmic bytes count every probed list, as the reference scans them; exact list "
                         "pruning and early exit leave only the scored bytes to read, so achieved can exceed "
                         "the HBM peak; scored_frac and dram_frac measure the bytes read"),
            },
            "phases_ms_per_step": {key: round(prof[key] / calls, 4) for key in
                                   ("normalize_ms", "coarse_ms", "select_ms", "pairs_ms", "scan_ms", "merge_ms",
                                    "collective_ms", "total_ms")},
            "scan_counters_per_step": {key: round(prof[key] / calls, 1) for key in
                                       ("scored_lists", "scored_vectors", "tables_built", "code_groups",
                                        "seed_scored_lists", "seed_scored_vectors", "seed_tables_built",
                                        "seed_code_groups")},
            "gpu_launches": int(prof["kernel_launches"]),
            "clocks": clock_info,
            "cpu_baseline": cpu_baseline,
        }
        if shard_check is not None:
            line["shard_check"] = shard_check
        if on_device and cpu_baseline is None:
            line["cpu_baseline_note"] = ("not run: the CPU port would need the whole database on the host "
                                         f"({n * d * 4 / 1e9:.0f} GB f32) and a CPU encode of it")
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        ix.close()
        dist.destroy_process_group()


def run_flat(args, cfg, world, rank, local):
    """Configuration 2: exact inner-product top-100 over 1e6 unit vectors
    (distance.rs:125-130; the ground truth of evaluation.rs:250-268).  One
    step = one vg_flat_search of the 10,000-query batch; every rank holds the
    database and answers its own batch (weak scaling, no collective)."""
    import torch
    import torch.distributed as dist

    from vicinity_b200 import FlatIndex
    from vicinity_b200.synthetic import config_data

    n, d, k = args.n or cfg["n"], cfg["d"], cfg["k"]
    nq = args.nq or cfg["nq"]
    t0 = time.time()
    x, q = config_data(args.config, seed=0, n=n, nq=nq * world)
    q = np.ascontiguousarray(q[rank * nq:(rank + 1) * nq])
    f = FlatIndex(x, device=local)
    build_s = time.time() - t0
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    qd = torch.from_numpy(q).cuda()
    ids_d = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    dist_d = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    cnt_d = torch.empty((nq,), dtype=torch.int32, device="cuda")

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(step, steps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        barrier()
        torch.cuda.synchronize()
        for a, b in evs:
            a.record(stream)
            step()
            b.record(stream)
        torch.cuda.synchronize()
        barrier()
        return sum(a.elapsed_time(b) for a, b in evs)

    def step_device():
        f.search_raw(qd.data_ptr(), nq, k, stream.cuda_stream, ids_d.data_ptr(), dist_d.data_ptr(), cnt_d.data_ptr())

    clocks = ClockSampler(local)
    clocks.start()
    clocks.wait_ready()
    f.set_profiling(True)
    timed(step_device, args.warmup)
    f.set_profiling(True)  # clears the warm-up totals
    clocks.begin()
    dev_ms = timed(step_device, args.steps)
    clocks.end()
    clock_info = clocks.stop()
    prof = f.profile()
    f.set_profiling(False)
    dev_ms_max = max_over_ranks(dev_ms)
    value = nq * world * args.steps / (dev_ms_max / 1e3)

    q_h = torch.from_numpy(q).pin_memory()
    ids_h = torch.empty((nq, k), dtype=torch.int32).pin_memory()
    dist_h = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    cnt_h = torch.empty((nq,), dtype=torch.int32).pin_memory()

    def step_e2e():
        f.search_raw(q_h.data_ptr(), nq, k, stream.cuda_stream, ids_h.data_ptr(), dist_h.data_ptr(), cnt_h.data_ptr())

    timed(step_e2e, max(1, args.warmup // 2))
    e2e_ms = max_over_ranks(timed(step_e2e, args.steps))
    e2e_value = nq * world * args.steps / (e2e_ms / 1e3)

    peaks, peak_kind = measured_peaks()
    calls = max(1, int(prof["calls"]))
    win_ms = prof["scan_ms"] / calls
    flops = 2.0 * nq * n * d  # the reference's multiply-adds over every row
    achieved = flops / (win_ms * 1e-3) / 1e12 if win_ms > 0 else 0.0
    peak = float(peaks.get("bf16_tflops", 1590.0))
    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_baseline = cpu_baseline_flat(x, q, k, ids_h.numpy(), dist_h.numpy(), args.cpu_seconds)
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "queries/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_ms_max / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic: N(0,1) rows L2-normalised, seeded (no dataset)",
            "config": workload_config(cfg, nq, 0, 0),
            "parallelism": "single GPU" if world == 1 else f"database replica per GPU, {nq} queries per rank x{world}",
            "index_build_s": round(build_s, 1),
            "e2e": {"value": round(e2e_value, 1), "unit": "queries/s", "h2d_bytes_per_step": nq * d * 4,
                    "d2h_bytes_per_step": nq * k * 8 + nq * 4},
            "roofline": {
                "kernel": ("tc_gemm_f16_kernel (tcgen05 binary16 products, TMEM accumulators): chunk maxima of "
                           "every 4th column tile, per-query thresholds, then a gather pass over every column"),
                "bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": None, "peak_source": f"bf16_tflops ({peak_kind})",
                "algorithmic_flops_per_launch": flops, "launch_ms": round(win_ms, 4),
                "note": ("algorithmic FLOPs = 2 nq n d (the reference's multiply-adds) over the product passes' "
                         "time (sample pass, thresholds, gather pass); the tensor pipe runs 1.25 x that over K "
                         "padded to whole steps of 16 (112 for d = 100)"),
            },
            "phases_ms_per_step": {"query_image_ms": round(prof["normalize_ms"] / calls, 4),
                                   "products_ms": round(win_ms, 4),
                                   "rescore_ms": round(prof["merge_ms"] / calls, 4)},
            "gpu_launches": int(prof["kernel_launches"]),
            "clocks": clock_info,
            "cpu_baseline": cpu_baseline,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    f.close()


def cpu_baseline_flat(x, q, k, eng_ids, eng_dist, budget_s):
    """The oracle's exhaustive -dot scan (distance.rs:125-130) on a sample of
    the batch on all host threads; its rows are compared with the engine's."""
    import oracle as orc

    threads = host_threads()
    t = time.time()
    orc.flat_search_ip(x, q[:threads], k, threads=threads)
    per_q = (time.time() - t) / threads
    s = int(min(q.shape[0], max(threads, budget_s / max(per_q, 1e-9))))
    t = time.time()
    ri, rd, rc = orc.flat_search_ip(x, q[:s], k, threads=threads)
    el = time.time() - t
    same = bool(np.array_equal(ri.astype(np.int64), eng_ids[:s].astype(np.int64)) and
                np.array_equal(rd.view(np.uint32), eng_dist[:s].view(np.uint32)))
    return {"value": round(s / el, 1), "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{s} queries of the batch ({el:.1f} s), oracle exhaustive scan on {threads} host threads",
            "rows_identical_to_engine": same}


def scan_traffic_from_profiles(config: int):
    """DRAM bytes per launch of the probe kernel from the committed ncu
    summary of this workload (None until one exists)."""
    path = ROOT / "profiles" / f"ivfpq_scan_c{config}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip()))
            except ValueError:
                return None
    return None


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline_port(ix, x, q, cfg, budget_s, truth):
    """The oracle port of the reference search (search.rs:1175-1391) on the
    same index (same centroids, codebooks, codes): all host threads for about
    budget_s, and the reference-faithful serial loop (one query at a time on
    one thread, as python.rs:745-795 batch_search does) on a small sample.
    Its rows are compared with the engine's on the sampled queries, and both
    recalls reported on them."""
    import oracle as orc

    threads = host_threads()
    k = cfg["k"]
    info = ix.info()
    ref = orc.OracleIndex(cfg["d"], int(info.num_centroids), cfg["M"], cfg["ks"], cfg["nprobe"])
    ref.set_trained(ix.centroids(), ix.codebooks())
    ref.add(ix.doc_ids(), x)
    ref.adopt_codes(ix.assignments(), ix.codes())
    probe = q[: max(threads * 2, 16)]
    t = time.time()
    ref.search_batch(probe, k, threads=threads)
    per_q = (time.time() - t) / probe.shape[0]
    target = int(max(probe.shape[0], budget_s / max(per_q, 1e-9)))  # queries for ~budget_s seconds
    done, el, first = 0, 0.0, None
    while done < target:
        s = min(q.shape[0], target - done)
        t = time.time()
        out = ref.search_batch(q[:s], k, threads=threads)
        el += time.time() - t
        if first is None:
            first = (s, out)
        done += s
    # reference-faithful: serial, one thread, a bounded sample
    serial_n = int(max(4, min(q.shape[0], 2.0 / max(per_q * threads, 1e-9))))
    t = time.time()
    for i in range(serial_n):
        ref.search_batch(q[i:i + 1], k, threads=1)
    serial = serial_n / (time.time() - t)
    # the oracle's rows against the engine's on the sampled queries
    s, (rid, rd, rc) = first
    rid = rid.astype(np.int64)
    rid[np.arange(k)[None, :] >= rc.astype(np.int64)[:, None]] = -1
    eid, ed = ix.batch_search(q[:s], k)
    same = bool(np.array_equal(rid, eid) and np.array_equal(rd.view(np.uint32), ed.view(np.uint32)))
    m = min(s, truth.shape[0])
    rec = lambda rows: float(np.mean([len(set(a) & set(b)) / k for a, b in zip(rows[:m].tolist(),
                                                                              truth[:m].tolist())]))
    return {"value": round(done / el, 1), "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{done} queries (batch queries reused, {el:.1f} s), oracle port of the reference search "
                      f"(search.rs:1175-1391) on the same index, {threads} host threads",
            "single_thread": {"value": round(serial, 1), "unit": "queries/s", "cores": 1,
                              "sample": f"{serial_n} queries one at a time (python.rs:745-795 loop)"},
            "rows_identical_to_engine": same, "compared_rows": int(s),
            "recall_at_10_oracle": round(rec(rid), 4), "recall_at_10_engine": round(rec(eid), 4)}


# --------------------------------------------------------------------------
# reference arm: the reference's CPU algorithm (oracle port) on host cores
# --------------------------------------------------------------------------

_MASK64 = (1 << 64) - 1


def seeded_prefix(n: int, take: int, seed: int) -> np.ndarray:
    """First `take` entries of a seeded Fisher-Yates permutation of [0, n),
    one splitmix64 draw per swap: how the engine picks its training rows and
    initial centroids (index.cu seeded_prefix)."""
    idx = np.arange(n, dtype=np.int64)
    s = seed & _MASK64
    for i in range(min(take, n - 1)):
        s = (s + 0x9E3779B97F4A7C15) & _MASK64
        z = ((s ^ (s >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK64
        z ^= z >> 31
        j = i + z % (n - i)
        idx[i], idx[j] = idx[j], idx[i]
    return idx[:take]


def _segment_means(rows: np.ndarray, labels: np.ndarray, nseg: int, old: np.ndarray) -> np.ndarray:
    """Per-label means of `rows` (sums in double); labels without rows keep
    `old`."""
    counts = np.bincount(labels, minlength=nseg)
    nz = counts > 0
    out = old.copy()
    for j in range(rows.shape[1]):
        sums = np.bincount(labels, weights=rows[:, j], minlength=nseg)
        out[nz, j] = (sums[nz] / counts[nz]).astype(np.float32)
    return out


def host_train_like_engine(xn: np.ndarray, cfg, sample: int, iters: int, seed: int = 42):
    """CPU restatement of the engine's index training, for the reference arm
    (untimed): the same seeded training rows and initial centroids, spherical
    Lloyd for the coarse lists and Euclidean Lloyd per PQ subspace from seeded
    rows, each stopping when no assignment changes (index.cu train()).  The
    reference trains with the third-party `clump` k-means; restating the
    engine's training instead gives both arms the same index recipe, so their
    recalls are comparable.  Returns centroids, codebooks, assignments and codes
    of every row of `xn` (L2-normalised)."""
    import torch  # CPU matmuls on every host thread (index construction only)

    torch.set_num_threads(host_threads())
    n, d = xn.shape
    M, ks = cfg["M"], cfg["ks"]
    dsub = d // M
    n_train = min(sample, n)
    rows = np.sort(seeded_prefix(n, n_train, seed)) if n_train < n else np.arange(n)
    X = np.ascontiguousarray(xn[rows])
    Lc = min(cfg["nlist"], n_train)
    cent = np.ascontiguousarray(X[seeded_prefix(n_train, Lc, seed)])

    def assign(data: np.ndarray, c: np.ndarray) -> np.ndarray:
        # nearest centroid by cosine distance 1 - dot (kmeans.rs:97-107): the
        # largest dot, the lowest list on ties.  One score buffer is reused
        # (a fresh 100 MB block per matmul costs more in page faults than the
        # matmul itself)
        out = torch.empty(data.shape[0], dtype=torch.int64)
        ct = torch.from_numpy(np.ascontiguousarray(c.T))
        blk = max(1, (1 << 25) // c.shape[0])
        buf = torch.empty((blk, c.shape[0]), dtype=torch.float32)
        for s0 in range(0, data.shape[0], blk):
            rows = min(blk, data.shape[0] - s0)
            torch.mm(torch.from_numpy(data[s0:s0 + rows]), ct, out=buf[:rows])
            torch.argmax(buf[:rows], dim=1, out=out[s0:s0 + rows])
        return out.numpy()

    prev = None
    for _ in range(iters):
        a = assign(X, cent)
        mean = _segment_means(X, a, Lc, cent)
        norm = np.sqrt((mean.astype(np.float64) ** 2).sum(axis=1)).astype(np.float32)
        moved = (np.bincount(a, minlength=Lc) > 0) & (norm > 1e-10)
        mean[moved] /= norm[moved, None]
        cent = mean
        done = prev is not None and np.array_equal(a, prev)
        prev = a
        if done:
            break

    def encode(res: np.ndarray, cb: np.ndarray) -> np.ndarray:
        # argmin over codewords of the squared distance (pq.rs:136-160), the
        # lowest codeword on ties: summed in coordinate order for small
        # codebooks; |c|^2 - 2 r.c by CPU matmul for 256-word codebooks (equal
        # but for near-ties, which do not move recall)
        codes = np.empty((res.shape[0], M), np.uint8)
        if ks * dsub <= 64:
            blk = max(1, (1 << 20) // (ks * dsub))
            for s0 in range(0, res.shape[0], blk):
                r = res[s0:s0 + blk]
                for m in range(M):
                    diff = r[:, None, m * dsub:(m + 1) * dsub] - cb[m][None, :, :]
                    dd = diff[..., 0] * diff[..., 0]
                    for j in range(1, dsub):
                        dd = dd + diff[..., j] * diff[..., j]
                    codes[s0:s0 + blk, m] = np.argmin(dd, axis=1)
            return codes
        cbt = torch.from_numpy(np.ascontiguousarray(cb.transpose(0, 2, 1)))  # [M][dsub][ks]
        cn = torch.from_numpy((cb.astype(np.float32) ** 2).sum(axis=2))[:, None, :]  # [M][1][ks]
        blk = max(1, (1 << 25) // (M * ks))
        for s0 in range(0, res.shape[0], blk):
            sub = torch.from_numpy(np.ascontiguousarray(res[s0:s0 + blk])).view(-1, M, dsub).transpose(0, 1)
            dd = torch.baddbmm(cn, sub, cbt, alpha=-2.0)  # [M][rows][ks]
            codes[s0:s0 + blk] = torch.argmin(dd, dim=2).T.numpy()
        return codes

    res = X - cent[assign(X, cent)]
    cb = np.empty((M, ks, dsub), np.float32)
    for m in range(M):
        cb[m] = res[seeded_prefix(n_train, ks, seed + m), m * dsub:(m + 1) * dsub]
    prev = None
    for _ in range(iters):
        codes = encode(res, cb)
        for m in range(M):
            cb[m] = _segment_means(res[:, m * dsub:(m + 1) * dsub], codes[:, m].astype(np.int64), ks, cb[m])
        done = prev is not None and np.array_equal(codes, prev)
        prev = codes
        if done:
            break
    assign_all = assign(xn, cent)
    codes_all = np.empty((n, M), np.uint8)
    blk = 1 << 20
    blk = 1 << 16
    for s0 in range(0, n, blk):
        codes_all[s0:s0 + blk] = encode(xn[s0:s0 + blk] - cent[assign_all[s0:s0 + blk]], cb)
    return cent, cb, assign_all.astype(np.uint32), codes_all


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return  # rank 0 alone runs the CPU reference arm
    import oracle as orc
    from vicinity_b200.synthetic import CONFIGS, config_data

    cfg = dict(CONFIGS[args.config])
    if cfg.get("generated") == "device":
        print(json.dumps({"impl": "reference", "unavailable": (
            f"configuration {args.config} is generated on the GPU and never held on the host; the CPU "
            f"reference would need a {cfg['n'] * cfg['d'] * 4 / 1e9:.0f} GB f32 host corpus")}), flush=True)
        return
    if args.nq:
        cfg["nq"] = args.nq
    threads = host_threads()
    x, q = config_data(args.config, seed=0, nq=cfg["nq"])
    if cfg["centre"] == "flat":
        return run_reference_flat(args, cfg, x, q, threads)
    train_sample = min(args.train_sample or cfg.get("train_sample", 131_072), x.shape[0])
    t0 = time.time()
    xn = orc.normalize(x)
    cent, cb, assign, codes = host_train_like_engine(xn, cfg, train_sample, args.train_iters)
    ref = orc.OracleIndex(cfg["d"], cfg["nlist"], cfg["M"], cfg["ks"], cfg["nprobe"])
    ref.set_trained(cent, cb)
    ref.add(np.arange(x.shape[0], dtype=np.uint32), x)
    ref.adopt_codes(assign, codes)
    build_s = time.time() - t0
    # recall@10 of this index on the batch's first RECALL_QUERIES queries
    # (exact top-10 of the normalised rows by CPU matmul), the same queries
    # the engine arm reports its recall on
    rs = min(RECALL_QUERIES, q.shape[0])
    truth = exact_top_k_cpu(xn, q[:rs], cfg["k"])
    del xn
    rid, _, rcnt = ref.search_batch(q[:rs], cfg["k"], threads=threads)
    ref_recall = recall_at_k(rid.astype(np.int64), rcnt, truth)
    probe = q[: max(2 * threads, 16)]
    t = time.time()
    ref.search_batch(probe, cfg["k"], threads=threads)
    per_q = (time.time() - t) / probe.shape[0]
    # each step: a bounded sample sized so warm-up + steps take about two minutes
    per_step_s = 120.0 / max(1, args.steps + args.warmup)
    s = int(min(q.shape[0], max(threads, per_step_s / max(per_q, 1e-9))))
    for i in range(args.warmup):
        ref.search_batch(q[:s], cfg["k"], threads=threads)
    total = 0.0
    for i in range(args.steps):
        sl = q[(i * s) % max(1, q.shape[0] - s):][:s]
        t = time.time()
        ref.search_batch(sl, cfg["k"], threads=threads)
        total += time.time() - t
    value = s * args.steps / total
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "queries/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded Gaussian mixture with the configuration's generator (no dataset)",
        "config": workload_config(cfg, cfg["nq"], train_sample, args.train_iters),
        "recall_at_10": round(ref_recall, 4),
        "recall_queries": rs,
        "step_sample": s,
        "index_build_s": round(build_s, 1),
        "cpu_baseline": {"value": round(value, 1), "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": f"{s} queries per step of the {cfg['nq']}-query batch, oracle port of the reference search on all host threads"},
        "e2e": {"value": round(value, 1), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_flat(args, cfg, x, q, threads):
    """Reference arm of configuration 2: the exhaustive -dot scan
    (distance.rs:125-130, evaluation.rs:250-268) of the oracle port on all
    host threads, a bounded sample of the batch per step."""
    import oracle as orc

    k = cfg["k"]
    t = time.time()
    orc.flat_search_ip(x, q[:threads], k, threads=threads)
    per_q = (time.time() - t) / threads
    per_step_s = 120.0 / max(1, args.steps + args.warmup)
    s = int(min(q.shape[0], max(threads, per_step_s / max(per_q, 1e-9))))
    for _ in range(args.warmup):
        orc.flat_search_ip(x, q[:s], k, threads=threads)
    total = 0.0
    for i in range(args.steps):
        sl = q[(i * s) % max(1, q.shape[0] - s):][:s]
        t = time.time()
        orc.flat_search_ip(x, sl, k, threads=threads)
        total += time.time() - t
    value = s * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "queries/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic: N(0,1) rows L2-normalised, seeded (no dataset)",
        "config": workload_config(cfg, cfg["nq"], 0, 0),
        "step_sample": s,
        "cpu_baseline": {"value": round(value, 1), "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": f"{s} queries per step, oracle exhaustive scan on all host threads"},
        "e2e": {"value": round(value, 1), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_engine(args)


if __name__ == "__main__":
    main()
