#!/usr/bin/env python3
"""Benchmark: the 1M-node MLA route on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one route of one probe over the whole 1,048,576 x 256 fp16 centroid
bank (top-3, bit-exact ids and scores); with --workload mla_1m_b64 a step
routes a batch of 64 probes (config 2's batch case, tensor-core path) and the
value counts probes.  At N > 1 (torchrun, one process per
GPU) the bank is node-range sharded: each GPU routes its 1/N of the nodes, the
per-shard top-3 candidates are all-gathered over NCCL and merged on the device
(strong scaling: the bank is fixed at 1M nodes).

Printed (rank 0, one JSON line):
  value      probes/s of the whole job, inputs resident in HBM, CUDA-event
             timing of each step on the launching stream, max over ranks;
  e2e        the same metric through the public route API with the query
             copied host->device and the result device->host every step;
  roofline   the scan kernel alone: bank bytes / its event-timed duration vs
             the measured HBM copy peak (MEASURED_PEAKS.json);
  cpu_baseline  the reference's own CPU route (cpp/grm_runtime.cpp compiled
             from source, OpenMP, all host cores) on the same bank;
  clocks     SM clock and throttle reasons sampled (NVML) during the run.
--impl reference times that reference CPU route alone (rank 0; other ranks
exit): each step routes one probe over the same full 1,048,576-node bank.

Both arms use config 2's recipe from one generator (synth.mla_config: rows
N(0,1), L2-normalised in fp32, stored fp16, then the queries as the next
draws of default_rng(1)), so they route identical inputs.  After the timed
region the outputs of timed steps are checked against the reference runtime
(ids) and the C restatement (scores); the line reports how many were checked.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "1M-node MLA route throughput (1,048,576 x 256 fp16 centroids, top-3, bit-exact)"
UNIT = "probes/s"
NODES, DIM, TOPK = 1 << 20, 256, 3
CFG_SEED = 1   # synth.mla_config seed: config 2 (config 1 is seed 0, 10,000 nodes)
L2_BYTES = 126 * 1024 * 1024


def l2_flush(buf) -> None:
    """Evict L2 between timed steps: write a buffer twice the L2 size, then read
    it back, so the write's dirty lines go to DRAM here and not inside the next
    timed region (where they would be charged to the step as extra writes)."""
    import torch

    buf.zero_()
    buf.sum(dtype=torch.int64)


def launch_gate(steps: int, per_step_us: float = 25.0) -> None:
    """Keep the stream busy with a fixed-length sleep kernel (torch.cuda._sleep:
    a clock-count spin that ends by itself) while the host queues the timed
    steps behind it, so the device-timed region holds back-to-back steps and
    no host launch gaps (the host path is what e2e measures)."""
    import torch

    us = min(200_000.0, max(1_000.0, steps * per_step_us))
    torch.cuda._sleep(int(us * 2_000))     # ~2,000 cycles per us at the B200's 1,965 MHz


def batch_of(workload: str) -> int:
    """Queries per step of an MLA workload (config 2: batch 1 and batch 64)."""
    return 64 if workload == "mla_1m_b64" else 1


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--gqa-prefix-gb", type=float, default=150.0,
                   help="gqa_100k on one GPU: size of the resident node prefix (the whole "
                        "216.5 GB bank does not fit one B200)")
    p.add_argument("--workload", default="mla_1m_b1",
                   choices=["mla_1m_b1", "mla_1m_b64", "mla_10k", "gqa_512", "gqa_100k", "mount_int4",
                            "mount_int6", "mount_int8", "mount_ref8", "mount_int4_rope",
                            "mount_ref8_rope", "mla_1m_policy", "mla_1m_multi", "mla_1m_int4"],
                   help="mla_1m_b1 is the headline (BASELINE config 2); mla_10k is config 1; "
                        "the others measure the GQA route (configs 3/4) and the quantised "
                        "mount (config 5)")
    return p.parse_args()


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(batch: int = 1):
    """dram bytes per scan launch from the committed ncu summary, if any (the
    summaries describe the 1M bank)."""
    if NODES != 1 << 20:
        return None
    f = ROOT / "profiles" / ("mla_scan_1m.md" if batch == 1 else "mla_batch_1m_b64.md")
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip()))
            except ValueError:
                return None
    return None


class ClockSampler:
    """NVML samples of SM clock and throttle reasons on one GPU."""

    REASONS = {
        0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x2: "applications_clocks_setting",
    }

    def __init__(self, index: int):
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except AttributeError:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                self.samples.append((mhz, int(r)))
            except Exception:
                pass
            self._stop.wait(0.02)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
            t_end = time.perf_counter() + 1.0   # first sample before the timed region
            while not self.samples and time.perf_counter() < t_end:
                time.sleep(0.002)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = set()
        for _, r in self.samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples": len(self.samples)}


def cpu_reference_full(rows_f32: np.ndarray, queries: np.ndarray, budget_s: float = 8.0,
                       check=None):
    """The reference's CPU route on the full bank (oracle/_ref OpenMP build),
    falling back to the C restatement when the reference was not built.
    check(store) runs the parity checker with the loaded store before timing."""
    import oracle as O

    cores = len(os.sched_getaffinity(0))
    if O.ref_available(omp=True):
        st = O.RefStore(omp=True).load_mla(rows_f32)
        st.route(queries[0], TOPK)                  # first call: arena rebuild + snapshot
        kind = "reference"
        route = lambda q: st.route(q, TOPK)  # noqa: E731
        if check is not None:
            check(st)
    else:
        if check is not None:
            check(None)
        norms = O.mla_row_norms(rows_f32)
        kind = "port"
        route = lambda q: O.mla_route(rows_f32, q, TOPK, norms=norms)  # noqa: E731
    times = []
    t_end = time.perf_counter() + budget_s
    i = 1
    while (time.perf_counter() < t_end or len(times) < 3) and len(times) < 64:
        t0 = time.perf_counter()
        route(queries[i % len(queries)])
        times.append(time.perf_counter() - t0)
        i += 1
    if kind == "reference":
        st.close()
    return {"value": 1.0 / statistics.median(times), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"full {rows_f32.shape[0]}-node bank, {len(times)} probes, median route "
                      f"{statistics.median(times) * 1e3:.1f} ms (OpenMP, {cores} threads)"}


def mla_inputs(n_queries: int):
    """Config 2's bank and queries (one generator, identical in both arms)."""
    from graftrepository_b200 import synth

    return synth.mla_config(CFG_SEED, NODES, queries=n_queries)


def reference_cuda_probe(rows_f32: np.ndarray, queries: np.ndarray, want_ids=None):
    """The reference's own GPU route (scripts/grm_mla_cuda_probe.py: cuBLAS
    Sgemv dots over the fp32 arena, fp64 query norm, cosine scores, a
    one-block top-k kernel), compiled from its CUDA_SOURCE for sm_100a by
    oracle/Makefile (ref_cuda) and timed here with the probe's own CUDA-event
    timing of its device query loop, on the same bank and queries.  Returns
    None when the probe library was not built."""
    import ctypes

    lib_path = ROOT / "oracle" / "_ref" / "libgrm_mla_cuda_probe.so"
    if not lib_path.exists():
        return None
    lib = ctypes.CDLL(str(lib_path))
    fp = ctypes.POINTER(ctypes.c_float)
    lib.grm_mla_cuda_arena_create.argtypes = [fp, ctypes.c_int, ctypes.c_int,
                                              ctypes.POINTER(ctypes.c_void_p)]
    lib.grm_mla_cuda_arena_route.argtypes = [ctypes.c_void_p, fp, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, ctypes.c_int,
                                             ctypes.POINTER(ctypes.c_uint64), fp]
    lib.grm_mla_cuda_arena_destroy.argtypes = [ctypes.c_void_p]
    rows = np.ascontiguousarray(rows_f32, dtype=np.float32)
    q = np.ascontiguousarray(queries, dtype=np.float32)
    h = ctypes.c_void_p()
    rc = lib.grm_mla_cuda_arena_create(rows.ctypes.data_as(fp), rows.shape[0], rows.shape[1],
                                       ctypes.byref(h))
    if rc != 0:
        return {"unavailable": f"probe arena create returned {rc}"}
    out = np.empty((q.shape[0], TOPK), dtype=np.uint64)
    ms = ctypes.c_float()
    rc = lib.grm_mla_cuda_arena_route(h, q.ctypes.data_as(fp), q.shape[0], q.shape[1], 3, TOPK,
                                      out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
                                      ctypes.byref(ms))
    lib.grm_mla_cuda_arena_destroy(h)
    if rc != 0:
        return {"unavailable": f"probe route returned {rc}"}
    per_q = ms.value / q.shape[0]
    res = {"value": 1e3 / per_q, "unit": UNIT, "ms_per_probe": per_q,
           "kernels": "cublasSgemv + query_norm + cosine_score + 1-block topk, fp32 arena",
           "sample": f"{q.shape[0]} probes after 3 warm-up probes, the probe's own event timing"}
    if want_ids is not None:
        want = [w[0] if isinstance(w, tuple) else w for w in want_ids]  # (ids, scores) or ids
        res["ids_equal_exact_route"] = f"{sum([int(x) for x in a] == [int(x) for x in b] for a, b in zip(out, want))}/{len(want)}"
    return res


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O

    cores = len(os.sched_getaffinity(0))
    n_q = max(8, min(args.warmup + args.steps, 4096))
    rows16, qs = mla_inputs(n_q)
    rows = rows16.astype(np.float32)
    del rows16
    if O.ref_available(omp=True):
        st = O.RefStore(omp=True).load_mla(rows)
        st.route(qs[0], TOPK)          # first call: the reference's arena rebuild + snapshot
        route = lambda q: st.route(q, TOPK)  # noqa: E731
        kind = "reference"
    else:
        st = None
        norms = O.mla_row_norms(rows)
        route = lambda q: O.mla_route(rows, q, TOPK, norms=norms)  # noqa: E731
        kind = "port"
    for i in range(args.warmup):
        route(qs[i % n_q])
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        route(qs[(args.warmup + i) % n_q])
        times.append(time.perf_counter() - t0)
    dt = sum(times)
    # the reference's own GPU route kernels on the same bank (same box), with
    # their top-3 compared to the exact route's (outside the timed steps)
    n_gpu_q = 8
    want = [route(qv) for qv in qs[:n_gpu_q]]
    if st is not None:
        st.close()
    value = args.steps / dt
    try:
        probe = reference_cuda_probe(rows, qs[:n_gpu_q], want)
    except Exception as exc:  # no GPU on this host, or the probe failed
        probe = {"unavailable": f"{type(exc).__name__}: {exc}"}
    one = None
    if O.ref_available(omp=False):   # the default single-threaded build CMake ships
        st1 = O.RefStore(omp=False).load_mla(rows)
        st1.route(qs[0], TOPK)
        ts = []
        t_end = time.perf_counter() + 10.0
        while (time.perf_counter() < t_end and len(ts) < 20) or len(ts) < 2:
            t0 = time.perf_counter()
            st1.route(qs[(len(ts) + 1) % n_q], TOPK)
            ts.append(time.perf_counter() - t0)
        st1.close()
        one = {"value": 1.0 / statistics.median(ts), "unit": UNIT, "cores": 1,
               "kind": "reference",
               "sample": f"{len(ts)} probes over the full bank, median "
                         f"{statistics.median(ts) * 1e3:.2f} ms (default build, no OpenMP)"}
    sample = (f"each step routes one probe over the full {NODES}-node bank "
              f"(grm_store_route, OpenMP, {cores} threads); median step "
              f"{statistics.median(times) * 1e3:.1f} ms")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 bank (fp16 values), f64 dot", "data": "synthetic",
        "config": {"workload": args.workload, "nodes": NODES, "dim": DIM, "topk": TOPK,
                   "batch": 1, "bank_dtype": "fp16 values (reference stores fp32)",
                   "recipe": "synth.mla_config(1): default_rng(1), rows then queries"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_cuda_probe": probe,
        "cpu_1thread": one,
    }), flush=True)


def run_reference_gqa(args):
    """Reference arm of the GQA workload gqa_512 (config 3): the reference's CPU
    route (grm_store_route_gqa, OpenMP and single-threaded builds) on a node
    prefix scaled per token, and its own GPU route (scripts/grm_gqa_cuda_probe.py:
    a zero-padded dense fp32 bank, per-kv-head cublasSgemm, an abs-max reduce
    kernel, a one-block top-k) on the whole bank, same box.  The bank is drawn
    by the same device generator as the other arm (synth.gqa_bank_device)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import ctypes

    import torch

    import oracle as O
    from graftrepository_b200 import synth

    KH, D, H = 32, 128, 128
    lengths = synth.gqa_lengths(2, 512, "uniform")
    keys_dev, off = synth.gqa_bank_device(2 * 1000, lengths)
    n_q = max(4, min(args.warmup + args.steps, 64))
    qs = synth.gqa_query(2, count=n_q)
    tokens = int(off[-1])
    cpu = cpu_gqa_baseline(keys_dev, off, qs[0], KH, D)
    keys16 = keys_dev.view(torch.int16).cpu().numpy().view(np.uint16)
    del keys_dev
    torch.cuda.empty_cache()
    one = None
    n_pre = int(np.searchsorted(off, 40_000, side="right")) - 1
    t_pre = int(off[n_pre])
    if O.ref_available(omp=False):
        with O.RefStore(omp=False).load_gqa(keys16[: t_pre * KH * D], off[: n_pre + 1], KH,
                                             D) as st1:
            st1.route(qs[0], TOPK)
            ts = []
            for i in range(3):
                t0 = time.perf_counter()
                st1.route(qs[i % n_q], TOPK)
                ts.append(time.perf_counter() - t0)
        per_tok = statistics.median(ts) / t_pre
        one = {"value": 1.0 / (per_tok * tokens), "unit": UNIT, "cores": 1, "kind": "reference",
               "sample": f"{n_pre}-node prefix ({t_pre} tokens), median "
                         f"{statistics.median(ts) * 1e3:.1f} ms, scaled per token to {tokens}"}
    probe = None
    lib_path = ROOT / "oracle" / "_ref" / "libgrm_gqa_cuda_probe.so"
    if lib_path.exists():
        tmax = int(lengths.max())
        dense = np.zeros((len(lengths), KH, tmax, D), np.float32)
        bits = keys16.astype(np.uint32) << 16
        f32 = bits.view(np.float32)
        for i in range(len(lengths)):
            t = int(lengths[i])
            dense[i, :, :t] = f32[int(off[i]) * KH * D: int(off[i + 1]) * KH * D].reshape(KH, t, D)
        del bits, f32
        lib = ctypes.CDLL(str(lib_path))
        fp = ctypes.POINTER(ctypes.c_float)
        lib.grm_gqa_cuda_arena_create.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
        lib.grm_gqa_cuda_arena_route.argtypes = [ctypes.c_void_p, fp, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                 ctypes.POINTER(ctypes.c_uint64), fp]
        lib.grm_gqa_cuda_arena_destroy.argtypes = [ctypes.c_void_p]
        h = ctypes.c_void_p()
        rc = lib.grm_gqa_cuda_arena_create(dense.ctypes.data_as(fp), len(lengths), KH, tmax, D,
                                           ctypes.byref(h))
        del dense
        if rc != 0:
            probe = {"unavailable": f"probe arena create returned {rc}"}
        else:
            nq = min(8, n_q)
            qv = np.ascontiguousarray(qs[:nq], dtype=np.float32)
            out = np.empty((nq, TOPK), dtype=np.uint64)
            ms = ctypes.c_float()
            rc = lib.grm_gqa_cuda_arena_route(h, qv.ctypes.data_as(fp), nq, H, 1, 3, TOPK,
                                              out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
                                              ctypes.byref(ms))
            lib.grm_gqa_cuda_arena_destroy(h)
            if rc != 0:
                probe = {"unavailable": f"probe route returned {rc}"}
            else:
                want = [O.gqa_route(keys16, off, KH, D, q, TOPK)[0] for q in qv[:2]]
                same = sum([int(x) for x in a] == [int(x) for x in b] for a, b in zip(out, want))
                probe = {"value": 1e3 / (ms.value / nq), "unit": UNIT,
                         "ms_per_probe": ms.value / nq,
                         "kernels": "per-kv-head cublasSgemm over a zero-padded fp32 bank + "
                                    "abs-max reduce + 1-block topk",
                         "padded_bank_bytes": len(lengths) * KH * tmax * D * 4,
                         "sample": f"{nq} probes after 3 warm-up probes, the probe's own event "
                                   f"timing",
                         "ids_equal_exact_route": f"{same}/{len(want)}"}
    value = cpu["value"]
    print(json.dumps({
        "impl": "reference", "metric": f"ragged GQA route throughput ({args.workload})",
        "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 / value, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32 keys (bf16 values), f32 dots",
        "data": "synthetic",
        "config": {"workload": args.workload, "nodes": int(len(lengths)), "tokens_total": tokens,
                   "kv_heads": KH, "q_heads": H, "head_dim": D, "topk": TOPK},
        "cpu_baseline": cpu, "cpu_1thread": one,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_cuda_probe": probe,
    }), flush=True)


def mla_parity(rows_f32, queries, got_ids, got_scores, ref_store=None):
    """Checker (outside every timed region): each routed query's ids against
    the reference runtime's route when a store is given, else against the C
    restatement, and its scores against the restatement's exact scores.
    Returns the number of queries checked; raises on a mismatch."""
    import oracle as O

    norms = O.mla_row_norms(rows_f32)
    for q, ids, sc in zip(queries, got_ids, got_scores):
        want, want_s = O.mla_route(rows_f32, q, TOPK, norms=norms)
        if ref_store is not None:
            ref_ids = ref_store.route(q, TOPK)
            if [int(x) for x in want] != ref_ids:
                raise RuntimeError(f"restatement {want} != reference {ref_ids}")
        if [int(x) for x in ids] != [int(x) for x in want] or not np.array_equal(sc, want_s):
            raise RuntimeError(f"timed route result {ids} {sc} != reference {want} {want_s}")
    return len(queries)


def run_ours(args):
    import torch
    import torch.distributed as dist

    from graftrepository_b200 import _lib, synth
    from graftrepository_b200.sharded import ShardedMLARoute, mla_shard_range

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    lib = _lib.load()

    B = batch_of(args.workload)   # queries per step
    # distinct queries every step (a pool of batches, cycled for long runs)
    n_q = min(args.warmup + args.steps, 4096 // B)
    rows16, qs_np = mla_inputs(n_q * B)
    a, b = mla_shard_range(NODES, world, rank)
    shard = torch.from_numpy(rows16[a:b]).cuda()
    route = ShardedMLARoute(group, shard, a, DIM, max_queries=64, device=local) if world > 1 \
        else None
    if world == 1:
        from graftrepository_b200.cuda_router import CudaMLARouteSidecar
        bank = CudaMLARouteSidecar(device=local).create_bank_device(shard.data_ptr(), 1, b - a, DIM)
        bank.reserve(64)
    else:
        bank = route.bank
    rows_host = rows16.astype(np.float32) if rank == 0 else None
    del rows16
    qs_host = torch.from_numpy(qs_np).pin_memory()
    qs_dev = qs_host.cuda()
    # route results go straight into one packed block per rank (ids, scores,
    # padding: 16 B per entry), so the exchange is a single all-gather
    n_out = B * TOPK
    blk = torch.empty(16 * n_out, dtype=torch.uint8, device="cuda")
    out_i = blk[:8 * n_out].view(torch.int64).view(B, TOPK)
    out_s = blk[8 * n_out:12 * n_out].view(torch.float32).view(B, TOPK)
    gblk = torch.empty(world * 16 * n_out, dtype=torch.uint8, device="cuda")
    gv = gblk.view(world, 16 * n_out)
    shard_bytes = (b - a) * DIM * 2
    flush = None
    if shard_bytes <= L2_BYTES:   # a shard larger than L2 cannot stay resident between steps
        flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    gi = gv[:, :8 * n_out].view(torch.int64)
    gs = gv[:, 8 * n_out:12 * n_out].view(torch.float32)
    ms_s = torch.empty((B, TOPK), dtype=torch.float32, device="cuda")
    ms_i = torch.empty((B, TOPK), dtype=torch.int64, device="cuda")

    def batch(i):
        j = i % n_q
        return qs_dev[j * B:(j + 1) * B]

    def step(i, ev):
        """One route of B queries: scan + resolve (programmatic dependent launch)
        [+ gather + merge].  ev: [start, end] or, at N > 1, [start, routed,
        gathered, end] for the per-phase split."""
        q = batch(i)
        if ev:
            ev[0].record(stream)
        rc = lib.grm_b200_mla_route_async(bank._h, q.data_ptr(), B, TOPK, a, out_i.data_ptr(),
                                          out_s.data_ptr(), sptr)
        if world > 1:
            if ev and len(ev) == 4:
                ev[1].record(stream)
            dist.all_gather_into_tensor(gblk, blk)
            if ev and len(ev) == 4:
                ev[2].record(stream)
            rc |= lib.grm_b200_merge_topk_strided(gs.data_ptr(), gs.stride(0), gi.data_ptr(),
                                                  gi.stride(0), B, world, TOPK, TOPK,
                                                  ms_s.data_ptr(), ms_i.data_ptr(), sptr)
        if ev:
            ev[-1].record(stream)
        if rc:
            raise RuntimeError("route launch failed")

    def scan_only(i, ev):
        """The scan phase alone, event-timed on its stream (roofline)."""
        q = batch(i)
        ev[0].record(stream)
        rc = lib.grm_b200_mla_scan_async(bank._h, q.data_ptr(), B, TOPK, a, out_i.data_ptr(),
                                         out_s.data_ptr(), sptr)
        ev[1].record(stream)
        rc |= lib.grm_b200_mla_resolve_async(bank._h, q.data_ptr(), B, TOPK, a,
                                             out_i.data_ptr(), out_s.data_ptr(), sptr)
        if rc:
            raise RuntimeError("scan launch failed")

    for i in range(args.warmup):
        if flush is not None:
            l2_flush(flush)
        step(i, None)
    torch.cuda.synchronize()
    # Without an L2 flush the K steps run back to back between one event pair
    # (routes chain through programmatic dependent launch, as in serving); with
    # a flush each step is bracketed by its own events so the flush is not
    # timed.  A second pass with per-step events gives the step distribution.
    n_dist = min(args.steps, 1000)
    n_ev = 4 if world > 1 else 2
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
           for _ in range(args.steps if flush is not None else n_dist)]
    ev_all = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    n_scan = min(args.steps, 1000)
    sevs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(n_scan)]
    fb0 = bank.stats()[1]
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        wall0 = time.perf_counter()
        if flush is None:
            launch_gate(args.steps)
            ev_all[0].record(stream)
            for i in range(args.steps):
                step(args.warmup + i, None)
            ev_all[1].record(stream)
        else:
            for i in range(args.steps):
                l2_flush(flush)
                step(args.warmup + i, evs[i])
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
        # the last timed step's result, kept for the parity check
        last_q = qs_host[((args.warmup + args.steps - 1) % n_q) * B:][:B].numpy().copy()
        last_i = (ms_i if world > 1 else out_i).cpu().numpy().view(np.uint64).copy()
        last_s = (ms_s if world > 1 else out_s).cpu().numpy().copy()
        fallbacks = bank.stats()[1] - fb0
        if world > 1:
            dist.barrier()
        if flush is None:
            for i in range(n_dist):
                step(args.warmup + i, evs[i])
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
        for i in range(n_scan):
            if flush is not None:
                l2_flush(flush)
            scan_only(args.warmup + i, sevs[i])
        torch.cuda.synchronize()
    step_ms = [e[0].elapsed_time(e[-1]) for e in evs]
    phases = None
    if world > 1:   # per-phase medians, max over ranks
        ph = torch.tensor([statistics.median(e[0].elapsed_time(e[1]) for e in evs),
                           statistics.median(e[1].elapsed_time(e[2]) for e in evs),
                           statistics.median(e[2].elapsed_time(e[3]) for e in evs)],
                          dtype=torch.float64, device="cuda")
        dist.all_reduce(ph, op=dist.ReduceOp.MAX)
        phases = {"route_us": ph[0].item() * 1e3, "allgather_us": ph[1].item() * 1e3,
                  "merge_us": ph[2].item() * 1e3,
                  "note": "medians of per-step event pairs (second pass), max over ranks; "
                          "route = this rank's scan + resolve"}
    scan_ms = [e[0].elapsed_time(e[1]) for e in sevs]
    timed_ms = ev_all[0].elapsed_time(ev_all[1]) if flush is None else sum(step_ms)
    tot = torch.tensor([timed_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    total_ms = float(tot.item())
    value = args.steps * B / (total_ms / 1e3)

    # e2e: the public API with host buffers every step
    e2e_steps = min(args.steps, 500)
    if world == 1:
        qn = qs_host.numpy().reshape(n_q, B, DIM)
        for i in range(5):
            bank.route_topk(qn[i % n_q], topk=TOPK)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            bank.route_topk(qn[(args.warmup + i) % n_q], topk=TOPK)
        e2e_s = time.perf_counter() - t0
        h2d, d2h = B * DIM * 4, B * TOPK * 12
    else:
        qbuf = torch.empty((B, DIM), dtype=torch.float32, device="cuda")
        for i in range(5):
            j = i % n_q
            qbuf.copy_(qs_host[j * B:(j + 1) * B], non_blocking=True)
            ids, sc = route.route(qbuf, TOPK)
            ids.cpu(), sc.cpu()
        dist.barrier()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            j = (args.warmup + i) % n_q
            qbuf.copy_(qs_host[j * B:(j + 1) * B], non_blocking=True)
            ids, sc = route.route(qbuf, TOPK)
            ids.cpu(), sc.cpu()
        e2e_s = time.perf_counter() - t0
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
        h2d, d2h = B * DIM * 4, B * TOPK * 12
    e2e_value = e2e_steps * B / e2e_s

    peak, peak_kind = peaks()
    scan_mean = statistics.mean(scan_ms)
    bytes_per_launch = shard_bytes + B * DIM * 4
    achieved = bytes_per_launch / (scan_mean / 1e3) / 1e9
    flops_per_launch = 2 * (b - a) * DIM * B
    # parity of timed outputs: the last timed step's result, plus the results
    # of the last e2e (public API) calls, all on queries of the timed pool
    checked = {"n": 0}
    if world == 1:
        e2e_q = qn[(args.warmup + e2e_steps - 1) % n_q]
        e2e_ids = bank.route_topk(e2e_q, topk=TOPK)[0]
        e2e_s = bank.last_scores.copy()
        chk_q = np.concatenate([last_q[:2], e2e_q[:1]])
        chk_i = np.concatenate([last_i[:2], e2e_ids[:1]])
        chk_s = np.concatenate([last_s[:2], e2e_s[:1]])
    else:
        chk_q, chk_i, chk_s = last_q[:3], last_i[:3], last_s[:3]

    def check(store):
        checked["n"] = mla_parity(rows_host, chk_q, chk_i, chk_s, store)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_full(rows_host, qs_np[:64], check=check)
    elif rank == 0:
        check(None)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    clocks = clk.summary()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": ("f16 bank, f32 scan, f64 exact refine" if B == 1 else
                  "f16 bank x f16 queries on tensor cores (f32 accumulate), f64 exact refine"),
        "data": "synthetic",
        "config": {"workload": args.workload, "nodes": NODES, "dim": DIM, "topk": TOPK, "batch": B,
                   "bank_dtype": "fp16", "shard_nodes": b - a,
                   "parallelism": f"node-sharded x{world}" if world > 1 else "single GPU",
                   "l2": ("bank shard larger than L2, no flush" if flush is None else
                          "256 MB L2 flush (written, then read back) before every step, outside the timed events")},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "kernel": ("mla_scan_bulk_kernel<256, half>" if B == 1 else
                                "mla_batch_kernel<256> (timed with its prep and merge kernels)"),
                     "algorithmic_bytes_per_launch": bytes_per_launch,
                     "traffic": profile_traffic(B),
                     "tensor_tflops": (flops_per_launch / (scan_mean / 1e3) / 1e12
                                       if B > 1 else None),
                     "scan_us_mean": scan_mean * 1e3,
                     "step_us_median": statistics.median(step_ms) * 1e3,
                     "step_us_p99": sorted(step_ms)[int(0.99 * (len(step_ms) - 1))] * 1e3},
        "exact_fallbacks_in_timed_steps": fallbacks,
        "parity_checked": checked["n"],
        "parity": ("timed-step results: ids == reference runtime route (full bank), scores == "
                   "exact restatement" if world == 1 and not args.no_cpu_baseline else
                   "timed-step results: ids and scores == exact restatement (full bank)"),
        "phases": phases,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "api": "CudaMLARouteBank.route_topk" if world == 1 else "ShardedMLARoute.route"},
        "gpu_launches": args.steps * ((2 if B == 1 else 4) + (0 if world == 1 else 1)),
        "timing": ("one event pair around the K back-to-back steps, queued behind a sleep "
                   "kernel so no host launch gap is timed" if flush is None else
                   "per-step event pairs, L2 flush between steps outside them"),
        "roofline_launches": n_scan,
        "clocks": clocks,
        "wall_s_timed_region": wall,
    }
    print(json.dumps(line), flush=True)
    if world == 1:
        bank.close()


# ------------------------------------------------------------ secondary workloads

def _dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def run_gqa(args):
    """Ragged GQA route: config 3 (512 nodes, T ~ U{16..1024}) or config 4
    (100k nodes, lognormal T).  A step routes one probe over the whole bank
    (1 GPU: the largest node prefix that fits, for config 4); at N GPUs the
    bank is node-range sharded balanced by tokens, candidates all-gathered."""
    import torch
    import torch.distributed as dist

    from graftrepository_b200 import _lib, synth
    from graftrepository_b200.cuda_router import CudaGQARouteSidecar
    from graftrepository_b200.sharded import gqa_shard_range

    world, rank, local = _dist_setup()
    lib = _lib.load()
    KH, D, H = 32, 128, 128
    if args.workload == "gqa_512":
        lengths = synth.gqa_lengths(2, 512, "uniform")
        seed = 2
    else:
        lengths = synth.gqa_lengths(3, 100_000, "lognormal")
        seed = 3
    off_all = synth.offsets(lengths)
    a, b = gqa_shard_range(off_all, world, rank)
    prefix_note = None
    if world == 1 and args.workload == "gqa_100k":
        cap_tokens = int(args.gqa_prefix_gb * 1e9 // (KH * D * 2))  # resident prefix
        b = int(np.searchsorted(off_all, cap_tokens, side="right")) - 1
        prefix_note = f"resident prefix of {b} of 100000 nodes ({int(off_all[b])} tokens)"
    sub_len = lengths[a:b]
    # draw this shard's keys directly (the seed is offset by the shard's first node)
    keys, off = synth.gqa_bank_device(seed * 1000 + a, sub_len)
    bank = CudaGQARouteSidecar(device=local).create_bank_device(
        keys.data_ptr(), 2, off, KH, D, keepalive=keys)
    tokens = int(off[-1])
    bytes_per_probe = tokens * KH * D * 2
    n_q = args.warmup + args.steps
    qs_host = torch.from_numpy(synth.gqa_query(seed, count=n_q)).pin_memory()
    qs_dev = qs_host.cuda()
    k = TOPK
    blk = torch.empty(16 * k, dtype=torch.uint8, device="cuda")   # ids, scores, padding
    out_i = blk[:8 * k].view(torch.int64).view(1, k)
    out_s = blk[8 * k:12 * k].view(torch.float32).view(1, k)
    gblk = torch.empty(world * 16 * k, dtype=torch.uint8, device="cuda")
    gi = gblk.view(world, 16 * k)[:, :8 * k].view(torch.int64)
    gs = gblk.view(world, 16 * k)[:, 8 * k:12 * k].view(torch.float32)
    ms_s = torch.empty((1, k), dtype=torch.float32, device="cuda")
    ms_i = torch.empty((1, k), dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream()
    qsz = H * D

    def step(i):
        rc = lib.grm_b200_gqa_route_async(bank._h, qs_dev[i].data_ptr(), 1, H, 1, k, a,
                                          out_i.data_ptr(), out_s.data_ptr(), stream.cuda_stream)
        if world > 1:
            dist.all_gather_into_tensor(gblk, blk)
            rc |= lib.grm_b200_merge_topk_strided(gs.data_ptr(), gs.stride(0), gi.data_ptr(),
                                                  gi.stride(0), 1, world, k, k, ms_s.data_ptr(),
                                                  ms_i.data_ptr(), stream.cuda_stream)
        if rc:
            raise RuntimeError(bank._err())

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            evs[i][0].record(stream)
            step(args.warmup + i)
            evs[i][1].record(stream)
        torch.cuda.synchronize()
    step_ms = [e[0].elapsed_time(e[1]) for e in evs]
    # this rank's result of the last timed step (its shard's top-k), for the check
    last_q = qs_host[(args.warmup + args.steps - 1) % n_q].numpy().copy()
    last_i = out_i.cpu().numpy().view(np.uint64)[0].copy()
    last_s = out_s.cpu().numpy()[0].copy()
    tot = torch.tensor([sum(step_ms)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    total_ms = float(tot.item())
    value = args.steps / (total_ms / 1e3)
    # e2e: public API, host query in, host ids out
    e2e_steps = min(args.steps, 50)
    qn = qs_host.numpy()
    if world == 1:
        for i in range(2):
            bank.route_topk(qn[i], topk=k)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            bank.route_topk(qn[(args.warmup + i) % n_q], topk=k)
        e2e_s = time.perf_counter() - t0
    else:
        qbuf = torch.empty((H, 1, D), dtype=torch.float32, device="cuda")
        dist.barrier()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            qbuf.copy_(qs_host[(args.warmup + i) % n_q], non_blocking=True)
            lib.grm_b200_gqa_route_async(bank._h, qbuf.data_ptr(), 1, H, 1, k, a,
                                         out_i.data_ptr(), out_s.data_ptr(), stream.cuda_stream)
            dist.all_gather_into_tensor(gblk, blk)
            lib.grm_b200_merge_topk_strided(gs.data_ptr(), gs.stride(0), gi.data_ptr(),
                                            gi.stride(0), 1, world, k, k, ms_s.data_ptr(),
                                            ms_i.data_ptr(), stream.cuda_stream)
            ms_i.cpu(), ms_s.cpu()
        e2e_s = time.perf_counter() - t0
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    routes, refined = bank.stats()
    peak, peak_kind = peaks()
    step_mean = statistics.mean(step_ms)
    achieved = bytes_per_probe / (step_mean / 1e3) / 1e9
    # every rank checks its own timed top-k (the merge is exact given them)
    checked = gqa_parity(keys, off, a, last_q, last_i, last_s, KH, D)
    if world > 1:
        c = torch.tensor([checked], dtype=torch.int64, device="cuda")
        dist.all_reduce(c)
        checked = int(c.item())
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_gqa_baseline(keys, off, qn[0], KH, D)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    total_tokens = int(off_all[-1]) if prefix_note is None else tokens
    print(json.dumps({
        "metric": f"ragged GQA route throughput ({args.workload})", "value": value,
        "unit": "probes/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16 keys, bf16x2 tensor-core q.k, f32 exact refine",
        "data": "synthetic",
        "config": {"workload": args.workload, "nodes": int(len(lengths)) if prefix_note is None
                   else b, "tokens_total": total_tokens, "kv_heads": KH, "q_heads": H,
                   "head_dim": D, "topk": k, "prefix": prefix_note,
                   "shard_tokens_rank0": tokens,
                   "l2": "bank larger than L2" if bytes_per_probe > 4 * L2_BYTES else "small bank"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "kernel": "whole route step (gqa_scan_kernel dominant)",
                     "algorithmic_bytes_per_launch": bytes_per_probe, "traffic": None,
                     "step_us_mean": step_mean * 1e3},
        "refined_nodes_per_route": refined / max(routes, 1),
        "parity_checked": checked,
        "parity": ("each rank's last timed top-k: scores == exact restatement of those nodes, "
                   "and no node of a <=300k-token shard prefix outranks them (restatement)"),
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_steps / e2e_s, "unit": "probes/s", "h2d_bytes_per_step": qsz * 4,
                "d2h_bytes_per_step": 400 if world == 1 else k * 12, "steps": e2e_steps},
        "gpu_launches": args.steps * (6 + (1 if world > 1 else 0)),
        "clocks": clk.summary(),
    }), flush=True)


def gqa_parity(keys_dev, off, id_offset, q, ids, scores, KH, D, max_tokens=300_000):
    """Checker (outside every timed region) of one timed GQA result over a
    shard: the returned nodes' scores equal the C restatement's exact scores
    of those nodes, and no node of the shard's first <= max_tokens tokens that
    is not returned outranks the k-th returned one (score desc, id asc).
    Returns the number of checks passed; raises on a mismatch."""
    import torch

    import oracle as O

    row = KH * D
    flat = keys_dev.view(torch.int16)

    def host_keys(t0, t1):
        return flat[t0 * row: t1 * row].cpu().numpy().view(np.uint16)

    fin = ids != np.iinfo(np.uint64).max
    loc = (ids[fin] - np.uint64(id_offset)).astype(np.int64)
    parts, lens = [], []
    for n in loc:
        t0, t1 = int(off[n]), int(off[n + 1])
        parts.append(host_keys(t0, t1))
        lens.append(t1 - t0)
    mini_off = np.zeros(len(lens) + 1, dtype=np.uint64)
    mini_off[1:] = np.cumsum(lens)
    exact = O.gqa_scores(np.concatenate(parts) if parts else np.zeros(0, np.uint16), mini_off,
                         KH, D, q)
    if not np.array_equal(exact, scores[fin]):
        raise RuntimeError(f"timed GQA scores {scores[fin]} != exact {exact}")
    n_pre = max(1, int(np.searchsorted(off, max_tokens, side="right")) - 1)
    s_pre = O.gqa_scores(host_keys(0, int(off[n_pre])), off[: n_pre + 1], KH, D, q)
    if fin.sum() == len(ids):
        ks, kid = float(scores[-1]), int(loc[-1])
        chosen = set(int(x) for x in loc)
        for i in np.nonzero(np.isfinite(s_pre) & (s_pre >= ks))[0]:
            i = int(i)
            if i not in chosen and (s_pre[i] > ks or i < kid):
                raise RuntimeError(f"node {i} (score {s_pre[i]}) outranks the timed top-k")
    return 2


def cpu_gqa_baseline(keys_dev, off, q, KH, D, max_tokens=40_000, budget_s=8.0):
    """Reference GQA route (oracle/_ref OpenMP build) on a node prefix of the
    bank with <= max_tokens tokens (its store keeps ~5 fp32 copies per key),
    reported per token scaled to the measured bank's token count."""
    import oracle as O

    n = int(np.searchsorted(off, max_tokens, side="right")) - 1
    n = max(1, n)
    t = int(off[n])
    keys = keys_dev[: t * KH * D].view(__import__("torch").int16).cpu().numpy().view(np.uint16)
    cores = len(os.sched_getaffinity(0))
    if O.ref_available(omp=True):
        st = O.RefStore(omp=True).load_gqa(keys, off[: n + 1], KH, D)
        st.route(q, TOPK)
        route = lambda: st.route(q, TOPK)  # noqa: E731
        kind = "reference"
    else:
        route = lambda: O.gqa_route(keys, off[: n + 1], KH, D, q, TOPK)  # noqa: E731
        kind = "port"
    times = []
    t_end = time.perf_counter() + budget_s
    while (time.perf_counter() < t_end or len(times) < 3) and len(times) < 50:
        t0 = time.perf_counter()
        route()
        times.append(time.perf_counter() - t0)
    per_token = statistics.median(times) / t
    return {"value": 1.0 / (per_token * int(off[-1])), "unit": "probes/s", "cores": cores,
            "kind": kind,
            "sample": f"{n}-node prefix ({t} tokens), median {statistics.median(times)*1e3:.1f} ms,"
                      f" scaled per token to {int(off[-1])} tokens"}


def run_mount(args):
    """Config 5: 3 grafts x 62 layers x 2048 tokens x 288 values, quantised,
    dequantised + scattered into a bf16 arena [62, 8192, 288].  A step is one
    mount of all three grafts.  `_rope` workloads also re-RoPE the 32-wide
    k_pe columns (256..287) at the arena seats in the same kernel.  Replicas
    only at N > 1 (no collective)."""
    import torch
    import torch.distributed as dist

    import oracle as O
    from graftrepository_b200 import graft_mount, synth

    world, rank, local = _dist_setup()
    G, L, T, W, S = 3, 62, 2048, 288, 8192
    vals = synth.grafts(4, G, L, T, W)
    seats = synth.seat_offsets(4, G, T, S)
    arena = graft_mount.ArenaMount(L, S, W, device=f"cuda:{local}", fill=0x7F81)
    stream = torch.cuda.current_stream()
    V = G * L * T * W
    base = args.workload.removesuffix("_rope")
    rope = None
    if base != args.workload:
        rc, rs = graft_mount.rope_tables(S, 32)
        rope = graft_mount.RopeSpec(torch.from_numpy(rc).cuda(), torch.from_numpy(rs).cuda(),
                                    256, 32)
    if base == "mount_ref8":
        c, sc = O.quant_ref(vals, 8)              # graft_quant format (group 32, fp32 scales)
        codes = torch.from_numpy(c.reshape(G, L, -1)).cuda()
        scales = torch.from_numpy(sc.reshape(G, L, -1)).cuda()
        bytes_per = V + V // 32 * 4 + 2 * V
        fn = lambda: arena.mount_ref(codes, scales, seats, T, rope=rope,  # noqa: E731
                                     stream=stream)
        bits = 8
    else:
        bits = int(base[-1])
        c, sc = graft_mount.quantize_packed(vals.reshape(G, L, -1), bits)
        codes = torch.from_numpy(c).cuda()
        scales = torch.from_numpy(sc.view(np.uint16)).cuda()
        bytes_per = V * bits // 8 + V // 64 * 2 + 2 * V
        fn = lambda: arena.mount_packed(codes, scales, seats, T, bits, rope=rope,  # noqa: E731
                                        stream=stream)
    if rope is not None:
        bytes_per += G * T * 32 * 4 * 2            # the cos/sin rows of the mounted seats
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            l2_flush(flush)
            evs[i][0].record(stream)
            fn()
            evs[i][1].record(stream)
        torch.cuda.synchronize()
    ms = [e[0].elapsed_time(e[1]) for e in evs]
    total_ms = sum(ms)
    # e2e: host codes/scales -> device, mount, arena checksum back to host
    ch, sh = torch.from_numpy(c).pin_memory(), torch.from_numpy(np.ascontiguousarray(sc)).pin_memory()
    e2e_steps = min(args.steps, 20)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        codes.view(-1).copy_(ch.view(-1).view(codes.dtype), non_blocking=True)
        scales.view(-1).copy_(sh.view(-1).view(scales.dtype), non_blocking=True)
        fn()
        arena.arena[0, 0, :8].cpu()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_mount_baseline(vals, bits, args.workload, rope is not None)
    peak, peak_kind = peaks()
    achieved = bytes_per / (statistics.mean(ms) / 1e3) / 1e9
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    print(json.dumps({
        "metric": f"quantised graft mount ({args.workload})", "value": args.steps / (total_ms / 1e3),
        "unit": "mounts/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": f"int{bits} codes -> bf16", "data": "synthetic",
        "config": {"workload": args.workload, "grafts": G, "layers": L, "tokens": T, "width": W,
                   "arena_seats": S, "l2": "256 MB L2 flush (written, then read back) before every step, outside events"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": bytes_per, "traffic": None,
                     "kernel": ("mount_ref_tiled_kernel" if base == "mount_ref8"
                                else f"mount_packed_tiled_kernel<{bits}>")
                     + (" (rope)" if rope is not None else "")},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_steps / e2e_s, "unit": "mounts/s",
                "h2d_bytes_per_step": int(c.nbytes + sc.nbytes), "d2h_bytes_per_step": 16,
                "steps": e2e_steps},
        "gpu_launches": args.steps, "clocks": clk.summary(),
    }), flush=True)


def cpu_mount_baseline(vals, bits, workload, rope=False):
    """The reference's CPU dequant (core/graft_quant.dequantize_symmetric_group32
    restated by the oracle, group 32, fp32 scales) + the bf16 cast, per mount,
    on one graft layer scaled to the 3 x 62 layers (the reference does it per
    layer on the host, core/graft_arena.py:3485-3492); with `rope`, plus the
    re-RoPE of that layer's k_pe columns at its seats (orc_mount_rope)."""
    import oracle as O
    from graftrepository_b200 import graft_mount

    one = vals[0, 0]
    c, s = O.quant_ref(one, 8 if bits == 8 else bits)
    if rope:
        T, W = one.shape
        rc, rs = graft_mount.rope_tables(8192, 32)
        layer = np.zeros((1, 8192, W), np.uint16)
    times = []
    for _ in range(5):
        t0 = time.perf_counter()
        _, bf = O.dequant_ref(c, s)
        if rope:
            layer[0, 100:100 + T] = bf.reshape(T, W)
            O.mount_rope(layer, 1, 1, T, [100], rc, rs, 256, 32)
        times.append(time.perf_counter() - t0)
    per_layer = statistics.median(times)
    layers = vals.shape[0] * vals.shape[1]
    return {"value": 1.0 / (per_layer * layers), "unit": "mounts/s", "cores":
            len(os.sched_getaffinity(0)), "kind": "port",
            "sample": f"dequant{' + re-RoPE' if rope else ''} of one [2048, 288] layer x {layers} layers "
                      f"(median {per_layer*1e3:.2f} ms/layer, OpenMP C restatement)"}


def run_policy(args):
    """The 1M-node MLA route with its policy channels on: every probe carries
    three lexical keys (two that nodes carry, one the bank lacks) and a kind
    filter of three kinds, over a bank whose nodes carry two Zipf-drawn keys,
    a kind and an active flag (1 % inactive).  A step is one probe through
    the public policy route (host query in, host ids out); the value is the
    route's device time (query upload excluded, the filter bitmap, scan,
    exact pass and lexical kernels included), e2e its wall time."""
    import torch

    import oracle as O
    from graftrepository_b200 import synth
    from graftrepository_b200.cuda_router import CudaMLARouteSidecar

    world, rank, local = _dist_setup()
    rows16 = synth.mla_bank(1, NODES)
    lexical, kinds, active = synth.route_policy(1, NODES)
    side = CudaMLARouteSidecar(device=local)
    bank = side.create_bank_raw(rows16, 1)
    t0 = time.perf_counter()
    bank.set_route_policy(lexical_keys=lexical, kinds=kinds, active=active)
    attach_s = time.perf_counter() - t0
    qs = synth.mla_queries(1, max(4, args.steps + args.warmup))
    qkeys = [synth.route_policy_query(i) for i in range(qs.shape[0])]
    kind_filter = ["turn", "doc", "fact"]
    from graftrepository_b200 import _lib
    L = _lib.load()
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=f"cuda:{local}")

    def one(i):
        ids, _ = bank.route_policy_topk(qs[i], topk=TOPK, lexical_keys=[qkeys[i]],
                                        kinds=kind_filter)
        return ids

    for i in range(args.warmup):
        one(i)
    dev_ms, walls = [], []
    with ClockSampler(local) as clk:
        for j in range(args.steps):
            i = args.warmup + j
            l2_flush(flush)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            one(i)
            walls.append(time.perf_counter() - t0)
            dev_ms.append(float(bank._last_elapsed_ms))
    cpu = None
    if rank == 0 and not args.no_cpu_baseline and O.ref_available(omp=True):
        per = NODES // 32
        rows = rows16.astype(np.float32)
        with O.RefStore(omp=True).load_mla_policy(rows[:per], lexical[:per],
                                                  [kinds[:per], None, None, None],
                                                  active[:per]) as st:
            st.route_policy(qs[0], TOPK, qkeys[0], [kind_filter, None, None, None])
            ts = []
            for i in range(min(20, qs.shape[0])):
                t0 = time.perf_counter()
                st.route_policy(qs[i], TOPK, qkeys[i], [kind_filter, None, None, None])
                ts.append(time.perf_counter() - t0)
        per_probe = statistics.median(ts) * 32
        cpu = {"value": 1.0 / per_probe, "unit": UNIT, "cores": len(os.sched_getaffinity(0)),
               "kind": "reference",
               "sample": f"grm_store_route_filtered over a {per}-node slice (1/32) of the bank "
                         f"with the same policy data, median of {len(ts)} probes "
                         f"({statistics.median(ts)*1e3:.2f} ms), x32"}
    bank.close()
    peak, peak_kind = peaks()
    mean_ms = statistics.mean(dev_ms)
    achieved = NODES * DIM * 2 / (mean_ms / 1e3) / 1e9
    if rank != 0:
        return
    print(json.dumps({
        "metric": "1M-node MLA route with lexical bonus + kind filter (policy channels on device)",
        "value": 1.0 / (mean_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean_ms, "higher_is_better": True,
        "scaling": "replicas", "vs_baseline": None, "dtype": "f16 bank, f32/f64 exact",
        "data": "synthetic",
        "config": {"workload": "mla_1m_policy", "nodes": NODES, "dim": DIM, "topk": TOPK,
                   "query_keys": 3, "node_keys": 2, "kind_filter": kind_filter,
                   "policy_attach_s": attach_s,
                   "l2": "256 MB L2 flush (written, then read back) before every step, outside the route"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": NODES * DIM * 2, "traffic": None,
                     "note": "bank bytes over the whole policy route's device time"},
        "cpu_baseline": cpu,
        "e2e": {"value": len(walls) / sum(walls), "unit": UNIT,
                "h2d_bytes_per_step": DIM * 4, "d2h_bytes_per_step": TOPK * 12},
        "step_ms_p50": statistics.median(dev_ms), "gpu_launches": None,
        "clocks": clk.summary(),
    }), flush=True)


def run_int4(args):
    """The reference's INT4 bulk/refine mode (route_mla_int4) on config 2's
    bank: a step is one probe through grm_b200_mla_route_int4_async (device
    query in, device ids out) with the reference's default refine set (4,096
    rows).  The INT4 arena (~134 MB) barely exceeds L2, so L2 is flushed
    before every step, outside the step's events.  The bank and arena are
    built during warm-up (the arena by the first INT4 route)."""
    import torch

    import oracle as O
    from graftrepository_b200.cuda_router import CudaMLARouteSidecar

    world, rank, local = _dist_setup()
    M = 4096
    n_q = max(8, min(args.warmup + args.steps, 4096))
    rows16, qs = mla_inputs(n_q)
    shard = torch.from_numpy(rows16).cuda()
    bank = CudaMLARouteSidecar(device=local).create_bank_device(shard.data_ptr(), 1, NODES, DIM)
    del shard
    qs_host = torch.from_numpy(qs).pin_memory()
    qd = qs_host.cuda()
    oi = torch.empty((1, TOPK), dtype=torch.int64, device="cuda")
    osc = torch.empty((1, TOPK), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")

    def step(i):
        bank.route_int4_async(qd[i % n_q].data_ptr(), 1, TOPK, oi.data_ptr(), osc.data_ptr(),
                              stream.cuda_stream, 0, M)

    for i in range(args.warmup):
        l2_flush(flush)
        step(i)
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            l2_flush(flush)
            evs[i][0].record(stream)
            step(args.warmup + i)
            evs[i][1].record(stream)
        torch.cuda.synchronize()
    step_ms = [e[0].elapsed_time(e[1]) for e in evs]
    last_i = oi.cpu().numpy().view(np.uint64)[0].copy()
    last_s = osc.cpu().numpy()[0].copy()
    last_q = qs[(args.warmup + args.steps - 1) % n_q]
    walls = []
    e2e_steps = min(args.steps, 200)
    for i in range(e2e_steps):
        t0 = time.perf_counter()
        bank.route_topk_int4(qs[(args.warmup + i) % n_q], topk=TOPK, refine_m=M)
        walls.append(time.perf_counter() - t0)
    rows = rows16.astype(np.float32)
    norms = O.mla_row_norms(rows)
    want, want_s = O.mla_int4_route(rows, last_q, TOPK, refine_m=M, norms=norms)
    if not (np.array_equal(last_i, want) and np.array_equal(last_s, want_s)):
        raise RuntimeError(f"timed INT4 route {last_i} {last_s} != restatement {want} {want_s}")
    cpu = None
    if rank == 0 and not args.no_cpu_baseline and O.ref_available(omp=True):
        os.environ["GRM_ROUTER_INT4"] = "1"
        os.environ["GRM_ROUTER_INT4_REFINE_M"] = str(M)
        with O.RefStore(omp=True).load_mla(rows) as st:
            st.route(qs[0], TOPK)
            ts = []
            t_end = time.perf_counter() + 8.0
            i = 1
            while (time.perf_counter() < t_end or len(ts) < 3) and len(ts) < 64:
                t0 = time.perf_counter()
                st.route(qs[i % n_q], TOPK)
                ts.append(time.perf_counter() - t0)
                i += 1
        del os.environ["GRM_ROUTER_INT4"]
        cpu = {"value": 1.0 / statistics.median(ts), "unit": UNIT,
               "cores": len(os.sched_getaffinity(0)), "kind": "reference",
               "sample": f"grm_store_route with GRM_ROUTER_INT4=1 (route_mla_int4, OpenMP) over "
                         f"the full bank, median of {len(ts)} probes "
                         f"({statistics.median(ts) * 1e3:.1f} ms)"}
    bank.close()
    peak, peak_kind = peaks()
    mean_ms = statistics.mean(step_ms)
    algo = NODES * DIM // 2 + 3 * 4 * NODES + M * DIM * 2
    achieved = algo / (mean_ms / 1e3) / 1e9
    if rank != 0:
        return
    print(json.dumps({
        "metric": "1M-node MLA route, INT4 bulk/refine mode (route_mla_int4, refine set 4,096)",
        "value": 1.0 / (mean_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean_ms, "higher_is_better": True,
        "scaling": "replicas", "vs_baseline": None,
        "dtype": "INT4 values, f32 sequential bulk dot, f64 exact refine", "data": "synthetic",
        "config": {"workload": "mla_1m_int4", "nodes": NODES, "dim": DIM, "topk": TOPK,
                   "refine_m": M, "recipe": "synth.mla_config(1)",
                   "l2": "256 MB L2 flush (written, then read back) before every step, outside "
                         "the step's events"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": algo, "traffic": None,
                     "note": "packed INT4 arena + norm scales + bulk keys written and read + "
                             "the refine set's fp16 rows, over the whole route's device time "
                             "(4 kernels)"},
        "parity_checked": 1,
        "parity": "last timed step: ids and scores == the INT4-mode restatement",
        "cpu_baseline": cpu,
        "e2e": {"value": len(walls) / sum(walls), "unit": UNIT,
                "h2d_bytes_per_step": DIM * 4, "d2h_bytes_per_step": TOPK * 12,
                "api": "CudaMLARouteBank.route_topk_int4"},
        "step_us_p50": statistics.median(step_ms) * 1e3, "gpu_launches": 4 * args.steps,
        "clocks": clk.summary(),
    }), flush=True)


def run_multi(args):
    """Multi-row entries: the 1,048,576 x 256 fp16 rows of config 2 grouped
    into entries of 1..4 rows (a digest's centroid and child centroids), an
    entry scoring the max of its rows.  A step is one probe through the
    public route (host query in, host ids out); value = the route's device
    time, e2e its wall time."""
    import torch

    import oracle as O
    from graftrepository_b200 import synth
    from graftrepository_b200.cuda_router import CudaMLARouteSidecar

    world, rank, local = _dist_setup()
    rows16 = synth.mla_bank(1, NODES)
    rng = np.random.default_rng(5)
    counts = rng.integers(1, 5, NODES)
    off = np.zeros(NODES + 1, np.uint64)
    off[1:] = np.cumsum(counts)
    entries = int(np.searchsorted(off, NODES, side="right") - 1)
    off = off[: entries + 1]
    off[-1] = NODES
    side = CudaMLARouteSidecar(device=local)
    bank = side.create_bank_multi(rows16.astype(np.float32), off)
    qs = synth.mla_queries(1, max(4, args.steps + args.warmup))
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=f"cuda:{local}")
    for i in range(args.warmup):
        bank.route_topk(qs[i], topk=TOPK)
    dev_ms, walls = [], []
    with ClockSampler(local) as clk:
        for j in range(args.steps):
            l2_flush(flush)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            _, rec = bank.route_topk(qs[args.warmup + j], topk=TOPK)
            walls.append(time.perf_counter() - t0)
            dev_ms.append(rec.device_route_ms_total)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline and O.ref_available(omp=True):
        per_e = entries // 32
        r_end = int(off[per_e])
        with O.RefStore(omp=True).load_mla_multi(rows16[:r_end].astype(np.float32),
                                                 off[: per_e + 1]) as st:
            st.route(qs[0], TOPK)
            ts = []
            for i in range(min(20, qs.shape[0])):
                t0 = time.perf_counter()
                st.route(qs[i], TOPK)
                ts.append(time.perf_counter() - t0)
        per_probe = statistics.median(ts) * 32
        cpu = {"value": 1.0 / per_probe, "unit": UNIT, "cores": len(os.sched_getaffinity(0)),
               "kind": "reference",
               "sample": f"grm_store_route over the first {per_e} entries ({r_end} rows, 1/32) "
                         f"with the same rows, median of {len(ts)} probes "
                         f"({statistics.median(ts)*1e3:.2f} ms), x32"}
    bank.close()
    peak, peak_kind = peaks()
    mean_ms = statistics.mean(dev_ms)
    achieved = NODES * DIM * 2 / (mean_ms / 1e3) / 1e9
    if rank != 0:
        return
    print(json.dumps({
        "metric": "1M-row MLA route over multi-row entries (max over each entry's rows)",
        "value": 1.0 / (mean_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean_ms, "higher_is_better": True,
        "scaling": "replicas", "vs_baseline": None, "dtype": "f16 bank, f32/f64 exact",
        "data": "synthetic",
        "config": {"workload": "mla_1m_multi", "rows": NODES, "entries": entries, "dim": DIM,
                   "rows_per_entry": "1..4 uniform", "topk": TOPK,
                   "l2": "256 MB L2 flush (written, then read back) before every step, outside the route"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": NODES * DIM * 2, "traffic": None,
                     "note": "row bytes over the whole route's device time"},
        "cpu_baseline": cpu,
        "e2e": {"value": len(walls) / sum(walls), "unit": UNIT,
                "h2d_bytes_per_step": DIM * 4, "d2h_bytes_per_step": TOPK * 12},
        "step_ms_p50": statistics.median(dev_ms), "gpu_launches": 6 * args.steps,
        "clocks": clk.summary(),
    }), flush=True)


def main():
    global NODES, METRIC, CFG_SEED
    args = parse()
    if args.workload == "mla_10k":   # seed 0, 10,000 x 256, top-3
        NODES, CFG_SEED = 10_000, 0
        METRIC = "10k-node MLA route throughput (config 1: 10,000 x 256 fp16, top-3, bit-exact)"
    if args.impl == "reference":
        if args.workload.startswith("gqa"):
            run_reference_gqa(args)
        else:
            run_reference(args)
    elif args.workload.startswith("gqa"):
        run_gqa(args)
    elif args.workload.startswith("mount"):
        run_mount(args)
    elif args.workload == "mla_1m_policy":
        run_policy(args)
    elif args.workload == "mla_1m_multi":
        run_multi(args)
    elif args.workload == "mla_1m_int4":
        run_int4(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
