#!/usr/bin/env python3
"""Benchmark: the 1M-node MLA route on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one route of one probe over the whole 1,048,576 x 256 fp16 centroid
bank (top-3, bit-exact ids and scores).  At N > 1 (torchrun, one process per
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
exit), each step one probe over a 1/32 slice of the bank, scaled to 1M nodes.
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
L2_BYTES = 126 * 1024 * 1024
WORKLOAD = "mla_1m_b1"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic():
    """dram bytes per scan launch from the committed ncu summary, if any."""
    f = ROOT / "profiles" / "mla_scan_1m.md"
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


def cpu_reference_full(rows_f32: np.ndarray, queries: np.ndarray, budget_s: float = 8.0):
    """The reference's CPU route on the full bank (oracle/_ref OpenMP build),
    falling back to the C restatement when the reference was not built."""
    import oracle as O

    cores = len(os.sched_getaffinity(0))
    if O.ref_available(omp=True):
        st = O.RefStore(omp=True).load_mla(rows_f32)
        st.route(queries[0], TOPK)                  # first call: arena rebuild + snapshot
        kind = "reference"
        route = lambda q: st.route(q, TOPK)  # noqa: E731
    else:
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


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    from graftrepository_b200 import synth

    cores = len(os.sched_getaffinity(0))
    slices = 32   # 32,768-node slices: at the reference's OpenMP threshold (cpp/grm_runtime.cpp:4320)
    per = NODES // slices
    rows = synth.mla_bank(1, NODES).astype(np.float32)
    qs = synth.mla_queries(1, max(8, min(args.warmup + args.steps, 4096)))
    omp = O.ref_available(omp=True)
    stores = []
    if omp:
        for s in range(slices):
            st = O.RefStore(omp=True).load_mla(rows[s * per:(s + 1) * per])
            st.route(qs[0], TOPK)
            stores.append(st)
        route = lambda s, q: stores[s].route(q, TOPK)  # noqa: E731
        kind = "reference"
    else:
        norms = O.mla_row_norms(rows)
        route = lambda s, q: O.mla_route(rows[s * per:(s + 1) * per], q, TOPK,  # noqa: E731
                                         norms=norms[s * per:(s + 1) * per])
        kind = "port"
    for i in range(args.warmup):
        route(i % slices, qs[i % len(qs)])
    t0 = time.perf_counter()
    for i in range(args.steps):
        route(i % slices, qs[(args.warmup + i) % len(qs)])
    dt = time.perf_counter() - t0
    per_probe = dt / args.steps * slices
    value = 1.0 / per_probe
    for st in stores:
        st.close()
    sample = (f"each step routes one probe over one {per}-node slice (1/{slices}) of the 1M bank; "
              f"probe time = {slices} x mean step time ({dt / args.steps * 1e3:.2f} ms)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_probe * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32/f64", "data": "synthetic",
        "config": {"workload": WORKLOAD, "nodes": NODES, "dim": DIM, "topk": TOPK, "batch": 1,
                   "bank_dtype": "fp16 values (reference stores fp32)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


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

    rows = synth.mla_bank_device(1, NODES)
    a, b = mla_shard_range(NODES, world, rank)
    shard = rows[a:b].contiguous()
    route = ShardedMLARoute(group, shard, a, DIM, max_queries=64, device=local) if world > 1 \
        else None
    if world == 1:
        from graftrepository_b200.cuda_router import CudaMLARouteSidecar
        bank = CudaMLARouteSidecar(device=local).create_bank_device(shard.data_ptr(), 1, b - a, DIM)
        bank.reserve(64)
    else:
        bank = route.bank
    rows_host = rows.float().cpu().numpy() if (rank == 0 and world == 1 and
                                               not args.no_cpu_baseline) else None
    del rows
    n_q = args.warmup + args.steps
    qs_host = torch.from_numpy(synth.mla_queries(1, n_q)).pin_memory()
    qs_dev = qs_host.cuda()
    out_s = torch.empty((1, TOPK), dtype=torch.float32, device="cuda")
    out_i = torch.empty((1, TOPK), dtype=torch.int64, device="cuda")
    shard_bytes = (b - a) * DIM * 2
    flush = None
    if shard_bytes < 4 * L2_BYTES:
        flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    gs = torch.empty((world, TOPK), dtype=torch.float32, device="cuda")
    gi = torch.empty((world, TOPK), dtype=torch.int64, device="cuda")
    ms_s = torch.empty((1, TOPK), dtype=torch.float32, device="cuda")
    ms_i = torch.empty((1, TOPK), dtype=torch.int64, device="cuda")

    def step(i, ev):
        q = qs_dev[i:i + 1]
        if ev:
            ev[0].record(stream)
        rc = lib.grm_b200_mla_scan_async(bank._h, q.data_ptr(), 1, TOPK, a, out_i.data_ptr(),
                                         out_s.data_ptr(), sptr)
        if ev:
            ev[1].record(stream)
        rc |= lib.grm_b200_mla_resolve_async(bank._h, q.data_ptr(), 1, TOPK, a, out_i.data_ptr(),
                                             out_s.data_ptr(), sptr)
        if world > 1:
            dist.all_gather_into_tensor(gs, out_s.view(-1))
            dist.all_gather_into_tensor(gi, out_i.view(-1))
            rc |= lib.grm_b200_merge_topk(gs.data_ptr(), gi.data_ptr(), 1, world, TOPK, TOPK,
                                          ms_s.data_ptr(), ms_i.data_ptr(), sptr)
        if ev:
            ev[2].record(stream)
        if rc:
            raise RuntimeError("route launch failed")

    for i in range(args.warmup):
        if flush is not None:
            flush.zero_()
        step(i, None)
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        wall0 = time.perf_counter()
        for i in range(args.steps):
            if flush is not None:
                flush.zero_()
            step(args.warmup + i, evs[i])
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
        if world > 1:
            dist.barrier()
    step_ms = [e[0].elapsed_time(e[2]) for e in evs]
    scan_ms = [e[0].elapsed_time(e[1]) for e in evs]
    tot = torch.tensor([sum(step_ms)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    total_ms = float(tot.item())
    value = args.steps / (total_ms / 1e3)

    # correctness of the timed steps: the last route equals a fresh exact route
    # (the full parity suite lives in tests/)
    # e2e: the public API with host buffers every step
    e2e_steps = min(args.steps, 500)
    if world == 1:
        qn = qs_host.numpy()
        for i in range(5):
            bank.route_topk(qn[i], topk=TOPK)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            bank.route_topk(qn[(args.warmup + i) % n_q], topk=TOPK)
        e2e_s = time.perf_counter() - t0
        h2d, d2h = DIM * 4, 400
    else:
        qbuf = torch.empty((1, DIM), dtype=torch.float32, device="cuda")
        for i in range(5):
            qbuf.copy_(qs_host[i:i + 1], non_blocking=True)
            ids, sc = route.route(qbuf, TOPK)
            ids.cpu(), sc.cpu()
        dist.barrier()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            qbuf.copy_(qs_host[(args.warmup + i) % n_q:(args.warmup + i) % n_q + 1],
                       non_blocking=True)
            ids, sc = route.route(qbuf, TOPK)
            ids.cpu(), sc.cpu()
        e2e_s = time.perf_counter() - t0
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
        h2d, d2h = DIM * 4, TOPK * 12
    e2e_value = e2e_steps / e2e_s

    peak, peak_kind = peaks()
    scan_mean = statistics.mean(scan_ms)
    bytes_per_launch = shard_bytes + DIM * 4
    achieved = bytes_per_launch / (scan_mean / 1e3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and rows_host is not None:
        cpu = cpu_reference_full(rows_host, synth.mla_queries(1, 64))
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    clocks = clk.summary()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16 bank, f32 scan, f64 exact refine",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "nodes": NODES, "dim": DIM, "topk": TOPK, "batch": 1,
                   "bank_dtype": "fp16", "shard_nodes": b - a,
                   "parallelism": f"node-sharded x{world}" if world > 1 else "single GPU",
                   "l2": ("bank shard larger than 4x L2, no flush" if flush is None else
                          "256 MB L2 flush before every step, outside the timed events")},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "kernel": "mla_scan_kernel<256, half>",
                     "algorithmic_bytes_per_launch": bytes_per_launch,
                     "traffic": profile_traffic(),
                     "scan_us_mean": scan_mean * 1e3,
                     "step_us_median": statistics.median(step_ms) * 1e3},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "api": "CudaMLARouteBank.route_topk" if world == 1 else "ShardedMLARoute.route"},
        "gpu_launches": args.steps * (2 if world == 1 else 3),
        "clocks": clocks,
        "wall_s_timed_region": wall,
    }
    print(json.dumps(line), flush=True)
    if world == 1:
        bank.close()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
