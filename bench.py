"""Benchmark of the B200 token sampler (one JSON line on rank 0).

A step is one batched sampling pass -- max, sum-exp, exact top-k, top-p and the seeded
draw for every row -- over one batch of seeded synthetic logits.

  N=1 workload: B=256 x V=151936 fp32 rows with heterogeneous per-row parameters (the
  "c4" configuration: bf16(N(0,4^2)) logits, 5% spiked rows, T~U[0.3,1.5],
  top-k in {0,20,100,1000}, top-p~U[0.5,1]); pool cap MAX_TOP_K = 1024.
  N>1 (torchrun, one rank per GPU): batch rows split across GPUs, no data-path
  collective (weak scaling: every rank samples its own 256 rows per step).

  value      rows/s over all ranks, logits already in HBM, device-timed with CUDA events
             on the launch stream, max over ranks. Inputs rotate over 4 batches (622 MB,
             larger than the 126 MB L2) so every step reads HBM.
  e2e        the same metric through the public host-buffer call tabby_sample_rows():
             pinned host logits -> device, sample, outcomes -> host, every step.
  roofline   algorithmic bytes = B * V * 4 per launch (each logit read once) / average
             time of one tabby_sample_rows_async call (one row_kernel launch; CUDA events
             on the launch stream), against MEASURED_PEAKS.json hbm_gbs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--profile]
  python bench.py --sweep    rows/s and HBM rate for B in 1..256 (c4 rows), one JSON line
  python bench.py --softmax  softmax_rows (attention scores) time and HBM rate, one JSON line
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ROWS = 256
VOCAB = 151936
CAP = 1024
ROTATE = 4
WORKLOAD = "c4_heterogeneous_B256_V151936"
METRIC = "sampled rows/s (B=256 x V=151936 fp32 logits, heterogeneous T/top-k/top-p)"
NOMINAL_HBM_GBS = 8000.0


def bench_config(world):
    """The workload both arms report (identical dicts, so the records compare)."""
    return {"workload": WORKLOAD, "rows_per_gpu": ROWS, "vocab": VOCAB, "max_top_k": CAP,
            "parallelism": f"rows split x{world}, no collective",
            "l2": f"inputs rotate over {ROTATE} resident batches "
                  f"({ROTATE * ROWS * VOCAB * 4 / 1e6:.0f} MB > 126 MB L2)"}


def parse_cpulist(text):
    """'0-3,8,10-11' -> {0, 1, 2, 3, 8, 10, 11} (the sysfs cpulist format)."""
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def gpu_numa_cpus(device_index):
    """(NUMA node, CPUs of that node this process may run on) for the PCI slot of CUDA
    device `device_index`, or (None, None) when the host does not say (no sysfs entry,
    node -1, or none of the node's CPUs in this process's affinity mask)."""
    try:
        import torch

        pr = torch.cuda.get_device_properties(device_index)
        slot = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{slot}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None, None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            cpus = parse_cpulist(f.read()) & os.sched_getaffinity(0)
        return (node, cpus) if cpus else (None, None)
    except (OSError, ValueError, AttributeError, RuntimeError):
        return None, None


class NumaLocal:
    """Runs the enclosed block on the CPUs of the GPU's NUMA node, so host buffers first
    touched inside it get pages on the node whose PCIe root holds the GPU (a pinned
    buffer on the other socket crosses the inter-socket link on every H2D copy); restores
    the previous affinity on exit. A no-op where the node is unknown."""

    def __init__(self, device_index):
        self.node, self.cpus = gpu_numa_cpus(device_index)
        self.prev = None

    def __enter__(self):
        if self.cpus:
            try:
                self.prev = os.sched_getaffinity(0)
                os.sched_setaffinity(0, self.cpus)
            except OSError:
                self.prev = None
                self.node = None
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            os.sched_setaffinity(0, self.prev)


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def node_probe():
    """Node.js on this box (the reference's own CPU sampler would run under it); the
    reference's TypeScript is not shipped with this repository, so without it the CPU
    baseline is the C restatement of sampler.ts."""
    import shutil

    path = shutil.which("node")
    if not path:
        return {"node": None}
    try:
        v = subprocess.run([path, "--version"], capture_output=True, text=True, timeout=10)
        return {"node": path, "version": v.stdout.strip()}
    except Exception as e:  # noqa: BLE001
        return {"node": path, "error": str(e)}


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes per launch of the dominant kernel on this workload, from the committed
    ncu summary (a line `traffic_bytes_per_launch: N`)."""
    path = os.path.join(ROOT, "profiles", "row_kernel_c4_B256.md")
    try:
        with open(path) as f:
            m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", f.read())
        return int(m.group(1)) if m else None
    except OSError:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 200 ms while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int, enabled: bool = True):
        self.gpu = gpu
        self.lines = []
        self.proc = None
        self.enabled = enabled

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference(x, params, u, seconds=10.0, threads=None):
    """The reference CPU path (full sort + sampleFromTopK per row, oracle restatement)
    on `threads` host cores (all of them by default) over a bounded sample of the
    workload's rows."""
    from oracle import oracle

    threads = threads or os.cpu_count() or 1
    rows_done, elapsed, reps = 0, 0.0, 0
    chunk = max(threads * 2, 16)
    r0 = 0
    while elapsed < seconds and reps < 1000:
        sl = slice(r0, r0 + chunk)
        elapsed += oracle.bench_rows(x[sl], params[sl], u[sl], CAP, threads)
        rows_done += x[sl].shape[0]
        r0 = (r0 + chunk) % x.shape[0]
        reps += 1
    return rows_done / elapsed, threads, f"{rows_done} rows of the workload in {elapsed:.1f} s"


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    from tabby_b200 import synth

    x, p, u = synth.config("c4", seed=0)
    vals = []
    # Bound the whole run to a few minutes whatever --steps/--warmup ask for.
    per_step = max(0.05, min(2.0, 150.0 / (args.warmup + args.steps)))
    threads, sample = 1, ""
    for i in range(args.warmup + args.steps):
        rate, threads, sample = cpu_reference(x, p, u, seconds=per_step)
        if i >= args.warmup:
            vals.append(rate)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * ROWS / value, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32/f64", "data": "synthetic (seeded)",
        "config": bench_config(world),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": sample + " per step (C restatement of sampler.ts topK "
                         "full sort + sampleFromTopK)"},
        "reference_runtime": node_probe(),
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, rank, local_rank, world):
    import torch

    from tabby_b200 import Sampler, synth
    from tabby_b200._lib import OUTCOME_DTYPE, check, lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pg = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)
        pg = dist

    x, p, u = synth.config("c4", seed=rank)
    sampler = Sampler(local_rank, max_top_k=CAP, max_rows=ROWS, max_vocab=VOCAB)
    h = sampler.handle
    # ROTATE resident batches (row-shifted copies) so consecutive steps miss L2.
    xt = torch.from_numpy(x)
    batches = [torch.roll(xt, shifts=i, dims=0).to(dev) for i in range(ROTATE)]
    p_dev = torch.from_numpy(p.view(np.uint8).copy()).to(dev)
    u_dev = torch.from_numpy(u).to(dev)
    out = torch.empty(ROWS * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    ids = torch.empty((ROWS, CAP), dtype=torch.int32, device=dev)
    vals = torch.empty((ROWS, CAP), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    L = lib()

    def step(i):
        b = batches[i % ROTATE]
        check(L.tabby_sample_rows_async(h, b.data_ptr(), VOCAB, ROWS, VOCAB, p_dev.data_ptr(),
                                        u_dev.data_ptr(), out.data_ptr(), ids.data_ptr(),
                                        vals.data_ptr(), CAP, sptr))

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)

    with ClockSampler(local_rank, enabled=not args.profile) as clocks:
        for i in range(args.warmup):
            step(i)
        # Keep the GPU loaded ~1 s before timing so the clock record reflects steady state.
        t_end = time.perf_counter() + (0.0 if args.profile else 1.0)
        i = 0
        while time.perf_counter() < t_end:
            for _ in range(200):
                step(i)
                i += 1
            torch.cuda.synchronize(dev)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1)
    if pg is not None:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = world * ROWS * args.steps / (ms / 1e3)

    # End-to-end through the public host-buffer API: pinned host logits in, outcomes out.
    e2e_steps = 0 if args.profile else max(3, min(args.steps, 50))
    e2e_value = None
    e2e_node = None
    hout = np.zeros(ROWS, OUTCOME_DTYPE)
    if e2e_steps:
        # Host buffers are allocated and first touched on the GPU's NUMA node.
        with NumaLocal(local_rank) as numa:
            e2e_node = numa.node
            host = torch.empty((ROWS, VOCAB), dtype=torch.float32, pin_memory=True)
            host.copy_(torch.from_numpy(x))
            hp = p.copy()
            hu = u.copy()
            hout = np.zeros(ROWS, OUTCOME_DTYPE)
            for _ in range(2):
                check(L.tabby_sample_rows(h, host.data_ptr(), VOCAB, ROWS, VOCAB,
                                          hp.ctypes.data, hu.ctypes.data, hout.ctypes.data,
                                          None, None, 0))
            barrier()
            t0 = time.perf_counter()
            for _ in range(e2e_steps):
                check(L.tabby_sample_rows(h, host.data_ptr(), VOCAB, ROWS, VOCAB,
                                          hp.ctypes.data, hu.ctypes.data, hout.ctypes.data,
                                          None, None, 0))
            e2e_s = time.perf_counter() - t0
        if pg is not None:
            t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            e2e_s = float(t.item())
        e2e_value = world * ROWS * e2e_steps / e2e_s

    sharded = sharded_peer = None
    if not args.profile:
        sharded = run_sharded(args, rank, local_rank, world, dev, pg)
        sharded_peer = run_sharded(args, rank, local_rank, world, dev, pg, "peer")
    sweep = None
    lmhead = None
    if world == 1 and not args.profile:
        sweep = sweep_points(sampler, x, p, u, dev, steps=200)
        lmhead, _, _ = lmhead_points((1, 128), 100)

    result = None
    if rank == 0:
        peak, peak_kind = measured_peak()
        bytes_per_launch = ROWS * VOCAB * 4
        achieved = bytes_per_launch / (ms_per_step / 1e3) / 1e9
        result = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (selection, sum-exp) / f64 (sampleFromTopK)",
            "data": "synthetic (seeded bf16-valued N(0,4^2) logits, heterogeneous params)",
            "config": bench_config(world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "frac_of_nominal_8tbs": achieved / NOMINAL_HBM_GBS,
                         "traffic": profiled_traffic(),
                         "algorithmic_bytes_per_launch": bytes_per_launch,
                         "kernel": "row_kernel (one cooperative launch per "
                                   "tabby_sample_rows_async call)"},
            "e2e": {"value": e2e_value, "unit": "rows/s",
                    "h2d_bytes_per_step": ROWS * VOCAB * 4 + p.nbytes + u.nbytes,
                    "d2h_bytes_per_step": hout.nbytes, "steps": e2e_steps,
                    "call": "tabby_sample_rows (pinned host buffers, synchronous)",
                    "host_numa_node": e2e_node},
            "gpu_launches": args.steps,  # one cooperative row_kernel launch per call
            "clocks": clocks.summary(),
        }
        if sharded is not None:
            result["sharded"] = sharded
        if sharded_peer is not None:
            result["sharded_peer"] = sharded_peer
        if lmhead is not None:
            result["lmhead"] = {"what": LMHEAD_WHAT, "points": lmhead}
        if sweep is not None:
            result["sweep"] = {"what": "c4 rows, V=151936, pool cap 1024, outcomes only; "
                                       "each call on a different window of a 255 MB pool",
                               "points": sweep}
    if pg is not None:
        pg.barrier()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline and not args.profile:
            rate, threads, sample = cpu_reference(x, p, u, seconds=args.cpu_seconds)
            rate1, _, sample1 = cpu_reference(x, p, u, seconds=max(2.0, args.cpu_seconds / 3),
                                              threads=1)
            result["cpu_baseline"] = {
                "value": rate, "unit": "rows/s", "cores": threads, "kind": "port",
                "single_thread_value": rate1, "cpu_model": cpu_model(),
                "sample": sample + " (C restatement of sampler.ts topK full sort + "
                "sampleFromTopK, all host threads); single thread: " + sample1,
                "reference_runtime": node_probe()}
        print(json.dumps(result), flush=True)
    sampler.close()
    if pg is not None:
        pg.destroy_process_group()
    return 0


SHARD_ROWS = 512  # the c5 configuration: B=512 x V=151936 split over the GPUs


def run_sharded(args, rank, local_rank, world, dev, pg, exchange="gather"):
    """Vocab-sharded sampling (c5): every rank holds columns [r*V/N, (r+1)*V/N) of 512
    rows; a step is the local top-64 blocks (row_kernel), then either one NCCL all-gather
    of the blocks (none at N=1) and the merge of every row on every rank (merge_kernel),
    or (exchange="peer") one xmerge_kernel that announces this rank's blocks, waits for
    the peers' announcements and merges every row reading the peers' blocks over NVLink.
    Every rank ends with the same tokens. Strong scaling: the job is 512 rows of the full
    vocabulary whatever N is. Device-timed with CUDA events on the launch stream, max
    over ranks, also per phase."""
    import torch

    from tabby_b200 import synth
    from tabby_b200._lib import OUTCOME_DTYPE
    from tabby_b200.sharded import SHARD_TOP_K, ShardedSampler, gather_blocks

    x, p, u = synth.config("c5", seed=0, rows=SHARD_ROWS)
    s = ShardedSampler(VOCAB, device=local_rank, max_rows=SHARD_ROWS, exchange=exchange)
    peer = exchange == "peer"
    local = torch.from_numpy(np.ascontiguousarray(x[:, s.lo:s.hi])).to(dev)
    p_dev = torch.from_numpy(p.view(np.uint8).copy()).to(dev)
    u_dev = torch.from_numpy(u).to(dev)
    out = torch.empty(SHARD_ROWS * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    ids = torch.empty((SHARD_ROWS, SHARD_TOP_K), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        if ev:
            ev[0].record(stream)
        if peer:
            s.local_into_exchange(local)
            if ev:
                ev[1].record(stream)
                ev[2].record(stream)
            s.exchange_merge_async(SHARD_ROWS, p_dev, u_dev, out)
            if ev:
                ev[3].record(stream)
            return
        block = s.local_blocks(local)
        if ev:
            ev[1].record(stream)
        gathered = gather_blocks(block) if pg is not None else block
        if ev:
            ev[2].record(stream)
        s.merge_async(gathered, world, p_dev, u_dev, out, ids, None)
        if ev:
            ev[3].record(stream)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    if pg is not None:
        pg.barrier()
    steps = max(10, min(args.steps, 200))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    total = e0.elapsed_time(e1) / steps
    # Per phase, on separate steps (events between the launches of each step).
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(20)]
    for ev in evs:
        step(ev)
    torch.cuda.synchronize(dev)
    phase = [sum(ev[j].elapsed_time(ev[j + 1]) for ev in evs) / len(evs) for j in range(3)]
    t = torch.tensor([total] + phase, dtype=torch.float64, device=dev)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    total, *phase = [float(v) for v in t.tolist()]
    if pg is not None:
        pg.barrier()  # every rank's last merge has returned before the buffers are freed
    s.close()
    if peer:
        return {"metric": "sampled rows/s, vocab-sharded (c5: B=512 x V=151936 split over "
                          f"{world} GPU(s), local top-64, merge with the exchange over "
                          "NVLink peer memory)",
                "value": SHARD_ROWS / (total / 1e3), "unit": "rows/s", "ms_per_step": total,
                "steps": steps, "scaling": "strong", "n_gpus": world,
                "phases_us": {"local_row_kernel": 1e3 * phase[0],
                              "xmerge_kernel (handshake + merge of every row)":
                                  1e3 * phase[2]},
                "local_columns": s.hi - s.lo,
                "launches_per_step": "row_kernel + xmerge_kernel (no collective library call)"}
    return {"metric": "sampled rows/s, vocab-sharded (c5: B=512 x V=151936 split over "
                      f"{world} GPU(s), local top-64, NCCL all-gather, merge)",
            "value": SHARD_ROWS / (total / 1e3), "unit": "rows/s", "ms_per_step": total,
            "steps": steps, "scaling": "strong", "n_gpus": world,
            "phases_us": {"local_row_kernel": 1e3 * phase[0],
                          "all_gather": 1e3 * phase[1] if pg is not None else 0.0,
                          "merge_kernel": 1e3 * phase[2]},
            "local_columns": s.hi - s.lo,
            "launches_per_step": "row_kernel + merge_kernel" + (
                " + NCCL all-gather" if pg is not None else "")}


def sweep_points(sampler, x, p, u, dev, steps):
    """B rows of the c4 workload per call for B in SWEEP_ROWS; each call reads a different
    window of a 420-row resident pool (255 MB > L2). CUDA-event timed over the calls."""
    import torch

    from tabby_b200._lib import OUTCOME_DTYPE, check, lib

    pool_rows = 420
    reps = (pool_rows + ROWS - 1) // ROWS
    pool = torch.from_numpy(np.ascontiguousarray(np.tile(x, (reps, 1))[:pool_rows])).to(dev)
    L = lib()
    sptr = torch.cuda.current_stream(dev).cuda_stream
    peak, _ = measured_peak()
    points = []
    for b in SWEEP_ROWS:
        pb = torch.from_numpy(p[:b].view(np.uint8).copy()).to(dev)
        ub = torch.from_numpy(u[:b].copy()).to(dev)
        out = torch.empty(b * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
        windows = pool_rows - b + 1

        def step(i):
            r0 = (i * b) % windows
            check(L.tabby_sample_rows_async(sampler.handle, pool[r0].data_ptr(), VOCAB, b,
                                            VOCAB, pb.data_ptr(), ub.data_ptr(),
                                            out.data_ptr(), None, None, 0, sptr))

        for i in range(3):
            step(i)
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            step(i)
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1e3 / steps
        gbs = b * VOCAB * 4 / (us * 1e-6) / 1e9
        points.append({"rows": b, "us_per_call": round(us, 2),
                       "rows_per_s": round(b / (us * 1e-6)), "gbs": round(gbs, 1),
                       "frac_of_peak": round(gbs / peak, 3)})
    del pool
    return points


SWEEP_ROWS = (1, 2, 4, 8, 16, 32, 64, 128, 256)


def run_sharded_only(args, rank, local_rank, world):
    """`--sharded`: the vocab-sharded c5 step alone (NCCL all-gather, then peer exchange)."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pg = None
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
        pg = dist
    lines = [run_sharded(args, rank, local_rank, world, dev, pg),
             run_sharded(args, rank, local_rank, world, dev, pg, "peer")]
    if rank == 0:
        for line in lines:
            print(json.dumps(line), flush=True)
    if pg is not None:
        dist.destroy_process_group()
    return 0


def run_sweep(args):
    """Batch sweep on one GPU (one JSON line)."""
    import torch

    from tabby_b200 import Sampler, synth

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    x, p, u = synth.config("c4", seed=0)
    sampler = Sampler(0, max_top_k=CAP, max_rows=ROWS, max_vocab=VOCAB)
    points = sweep_points(sampler, x, p, u, dev, steps=max(50, min(args.steps, 1000)))
    sampler.close()
    peak, peak_kind = measured_peak()
    print(json.dumps({"sweep": "c4 rows, V=151936, pool cap 1024, outcomes only",
                      "peak_gbs": peak, "peak_kind": peak_kind, "points": points}), flush=True)
    return 0


SOFTMAX_SHAPES = (  # (label, rows, row_len, causal_period, causal_offset)
    ("decode: 14 heads x 1 query, context 4096", 14, 4096, 1, 4095),
    ("prefill: 14 heads x 2048 queries, causal", 14 * 2048, 2048, 2048, 0),
    ("batch 64 x 14 heads x 1 query, context 8192", 64 * 14, 8192, 0, 0),
)


def run_softmax(args):
    """softmax_rows (the attention-score softmax next to the sampler, softmax_rows.wgsl):
    device time per call and HBM rate (4 bytes read per kept entry, 4 written per entry),
    on inputs rotated over enough copies to exceed L2."""
    import torch

    from tabby_b200._lib import check, lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = lib()
    sptr = torch.cuda.current_stream(dev).cuda_stream
    peak, peak_kind = measured_peak()
    points = []
    for label, rows, n, period, offset in SOFTMAX_SHAPES:
        nbuf = max(2, -(-256 * 2**20 // (rows * n * 4)))
        bufs = [torch.randn(rows, n, device=dev) * 4 for _ in range(nbuf)]

        def step(i):
            check(L.tabby_softmax_rows_async(bufs[i % nbuf].data_ptr(), rows, n, period, offset,
                                             sptr))

        for i in range(max(args.warmup, 3)):
            step(i)
        torch.cuda.synchronize(dev)
        steps = max(50, min(args.steps, 500))
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            step(i)
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1e3 / steps
        # Bytes: the kept prefix of every row is read, every entry is written.
        if period:
            kept = sum(min(offset + (r % period) + 1, n) for r in range(period)) * (rows // period)
        else:
            kept = rows * n
        gbs = (kept * 4 + rows * n * 4) / (us * 1e-6) / 1e9
        points.append({"shape": label, "us_per_call": round(us, 2), "gbs": round(gbs, 1),
                       "frac_of_peak": round(gbs / peak, 3)})
        del bufs
    print(json.dumps({"softmax_rows": points, "peak_gbs": peak, "peak_kind": peak_kind}),
          flush=True)
    return 0


LMHEAD_ROWS = (1, 8, 32, 64, 128)


def run_lmhead(args):
    rows = [int(x) for x in args.rows.split(",")] if args.rows else LMHEAD_ROWS
    points, peak, peak_kind = lmhead_points(rows, args.steps)
    print(json.dumps({"lmhead": LMHEAD_WHAT, "peak_gbs": peak, "peak_kind": peak_kind,
                      "points": points}), flush=True)
    return 0


LMHEAD_WHAT = ("fused LM head + sampling, V=151936 x hidden 896 bf16 (272 MB of weights a "
               "call), pool cap 64; unfused = torch.matmul (cuBLAS, bf16 logits) + fp32 "
               "conversion + tabby_sample_rows_async")


def lmhead_points(rows, steps):
    """Fused LM head + sampling (tabby_lmhead_sample_async) at V=151936, hidden 896
    (Qwen2.5-0.5B's lm_head, bf16 weights, 272 MB: every call reads them from HBM), against
    the unfused path of the same library: torch.matmul (cuBLAS bf16 -> fp32 logits) then
    tabby_sample_rows_async. Device time per call with CUDA events; roofline against the
    weight bytes (the dominant traffic) and the tensor FLOPs."""
    import ctypes

    import torch

    from tabby_b200 import Sampler
    from tabby_b200._lib import OUTCOME_DTYPE, check, lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = lib()
    V, H = VOCAB, 896
    g = torch.Generator(device="cuda").manual_seed(0)
    w = (torch.randn(V, H, device=dev, generator=g) * (3.0 / H ** 0.5)).to(torch.bfloat16)
    peak, peak_kind = measured_peak()
    sampler = Sampler(0, max_top_k=64, max_rows=128, max_vocab=V)
    sptr = torch.cuda.current_stream(dev).cuda_stream
    points = []
    for b in rows:
        h = torch.randn(b, H, device=dev, generator=g).to(torch.bfloat16)
        p = np.zeros(b, [("temperature", "<f8"), ("top_p", "<f8"), ("top_k", "<i4"),
                         ("reserved", "<i4")])
        p["temperature"], p["top_p"], p["top_k"] = 0.8, 0.95, 40
        pd = torch.from_numpy(p.view(np.uint8).copy()).to(dev)
        ud = torch.rand(b, dtype=torch.float64, device=dev)
        out = torch.empty(b * OUTCOME_DTYPE.itemsize, dtype=torch.uint8, device=dev)
        handle = ctypes.c_void_p()
        check(L.tabby_lmhead_create(0, b, V, H, ctypes.byref(handle)))

        def fused():
            check(L.tabby_lmhead_sample_async(handle, h.data_ptr(), w.data_ptr(), b,
                                              pd.data_ptr(), ud.data_ptr(), out.data_ptr(),
                                              None, None, 0, None, sptr))

        def unfused():
            logits = torch.matmul(h, w.T).float()
            check(L.tabby_sample_rows_async(sampler.handle, logits.data_ptr(), V, b, V,
                                            pd.data_ptr(), ud.data_ptr(), out.data_ptr(),
                                            None, None, 0, sptr))

        res = {}
        for name, fn in (("fused_us", fused), ("unfused_us", unfused)):
            for _ in range(5):
                fn()
            torch.cuda.synchronize(dev)
            n = max(20, min(steps, 200))
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(n):
                fn()
            e1.record()
            torch.cuda.synchronize(dev)
            res[name] = e0.elapsed_time(e1) * 1e3 / n
        L.tabby_lmhead_destroy(handle)
        wbytes = V * H * 2
        gbs = wbytes / (res["fused_us"] * 1e-6) / 1e9
        tflops = 2.0 * b * V * H / (res["fused_us"] * 1e-6) / 1e12
        points.append({"rows": b, "fused_us": round(res["fused_us"], 2),
                       "unfused_us": round(res["unfused_us"], 2),
                       "speedup": round(res["unfused_us"] / res["fused_us"], 3),
                       "weight_gbs": round(gbs, 1), "hbm_frac": round(gbs / peak, 3),
                       "tensor_tflops": round(tflops, 1)})
    sampler.close()
    return points, peak, peak_kind


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="batch sweep B=1..256 on one GPU")
    ap.add_argument("--softmax", action="store_true", help="softmax_rows shapes on one GPU")
    ap.add_argument("--lmhead", action="store_true", help="fused LM head + sampling on one GPU")
    ap.add_argument("--rows", default="", help="--lmhead: comma-separated batch sizes")
    ap.add_argument("--sharded", action="store_true",
                    help="only the vocab-sharded c5 step, both exchanges (one line each)")
    ap.add_argument("--profile", action="store_true",
                    help="only warm-up + timed steps (for ncu): no heat loop, e2e or CPU leg")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, local_rank, world = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.sweep:
        return run_sweep(args) if rank == 0 else 0
    if args.softmax:
        return run_softmax(args) if rank == 0 else 0
    if args.lmhead:
        return run_lmhead(args) if rank == 0 else 0
    if args.sharded:
        return run_sharded_only(args, rank, local_rank, world)
    return run_ours(args, rank, local_rank, world)


if __name__ == "__main__":
    sys.exit(main())
