"""Benchmark of the reduce / broadcast hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c5b|c2|...]

Metric: reduce/broadcast GB/s (algorithmic HBM bytes per second, whole job) and its fraction of
the B200 HBM roofline, against the reference's CPU path.

Headline workload (default, one "step"): benchmark config 5b, the largest config, a full Sum of
2^32 float32 values ~ N(0,1) (16 GiB), held as [8, 2^29] because 2^32 elements exceed the reference's
32-bit size_m, and evaluated as x.sum(1).sum(0).  The rows are sharded over the GPUs (one process per
GPU, torchrun); each rank reduces its rows with mtxc_reduce (sum(1), the HBM stream), and sum(0) over
the sharded axis is mtxc_reduce_sharded: the local sum of the rank's partials, an NCCL all-gather of
one value per rank and the ordered merge, all enqueued by the C ABI.  Strong scaling: the total is fixed
at 2^32 elements whatever N.  The exchange of step k runs on a side stream and overlaps the row
reduction of step k + 1; the last exchange is inside the timed region.  Algorithmic bytes per step:
17,179,869,184 (the input read once).  Inputs are synthetic (seeded per row), as no dataset is named.

`--impl reference` times the reference's own CPU Sum loop (Matrix.mm:15193-15205, compiled from the
reference tree into oracle/_ref/libmtx_ref.so) on a bounded sample of the same workload, one slice of
the flattened input per host thread.

`--workload c2` times config 2 (broadcast Add + Mul f32 a[256,1,4096] (op) b[1,512,4096], weak scaling,
no collective) with the same instrumentation; `--workload c1|c3|c4|c5a` time the other configs sharded
over the GPUs; `--suite` prints one device-time line per config (diagnostics, not the headline).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "reduce/broadcast GB/s and % of HBM peak at 1/2/4/8 B200 vs host-CPU ref"
UNIT = "GB/s"
A_SHAPE, B_SHAPE, OUT_SHAPE = [256, 1, 4096], [1, 512, 4096], [256, 512, 4096]
OP_BYTES = (256 * 512 * 4096 + 256 * 4096 + 512 * 4096) * 4  # 2,160,066,560


def c2_shapes(rows: int):
    """a, out shapes and algorithmic bytes per op when a has `rows` leading rows (256 = C2)."""
    return [rows, 1, 4096], [rows, 512, 4096], (rows * 512 * 4096 + rows * 4096 + 512 * 4096) * 4
OPS = ("add", "mul")
WORKLOAD = "C2: broadcast Add+Mul f32 a[256,1,4096] (op) b[1,512,4096] -> [256,512,4096]"
FALLBACK_HBM_GBS = 6650.0


# config 5b: the headline
C5B_ROWS, C5B_COLS = 8, 1 << 29
C5B_WORKLOAD = ("C5b: full Sum of f32 2^32 ~ N(0,1) held as [8, 2^29] (16 GiB), x.sum(1).sum(0); rows sharded "
                "over the GPUs, sum(0) over the sharded axis = NCCL all-gather of the per-rank partials + ordered merge")


def fill_c5b_rows(x, first_row: int) -> None:
    """Seeded synthetic input of config 5b: global row r ~ N(0,1) from its own seed (1000 + r), so the
    tensor is the same whatever the number of GPUs it is sharded over."""
    import torch

    g = torch.Generator(device=x.device)
    for r in range(x.shape[0]):
        g.manual_seed(1000 + first_row + r)
        x[r].normal_(generator=g)


def measured_peak():
    p = REPO / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic():
    """DRAM bytes (read + write) per launch of the dominant kernel, from the committed ncu summary."""
    p = REPO / "profiles" / "broadcast_group_c2_traffic.txt"
    try:
        for line in p.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


def profile_traffic_c5b():
    """DRAM bytes (read + write) per input byte of reduce_rows_kernel's C5b launch, from the committed
    ncu summary of a smaller case of the same kernel (the traffic grows in proportion to the input)."""
    p = REPO / "profiles" / "reduce_rows_c5b_traffic.txt"
    try:
        for line in p.read_text().splitlines():
            if line.startswith("dram_bytes_per_input_byte:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


# ------------------------------------------------------------------------------------------
# clocks
# ------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids):
        self.uuids = {u.lower() for u in uuids}
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        sm, smax, reasons, n = [], [], set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            uuid = parts[0].lower()
            if self.uuids and not any(uuid.endswith(u) or u.endswith(uuid) or u in uuid for u in self.uuids):
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            n += 1
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        os.unlink(self.file.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": n}


# ------------------------------------------------------------------------------------------
# inputs
# ------------------------------------------------------------------------------------------
def c2_inputs_numpy(rank: int = 0):
    """Seeded synthetic inputs: a shard `rank` of the global a, and the replicated b."""
    a = np.random.default_rng([1, rank]).uniform(-1, 1, 256 * 4096).astype(np.float32).reshape(A_SHAPE)
    b = np.random.default_rng([1, 1 << 20]).uniform(-1, 1, 512 * 4096).astype(np.float32).reshape(B_SHAPE)
    return a, b


# ------------------------------------------------------------------------------------------
# CPU baseline: the reference's own loop (or the oracle restatement), threads over row slices
# ------------------------------------------------------------------------------------------
def cpu_evaluator():
    from oracle import oracle

    ref = oracle.reference()
    if ref is not None:
        return ref, "reference"
    p = oracle.port()
    p.threads = 1
    return p, "port"


def cpu_c2_step(ev, meta_rows, a, b, out, rows: int, threads: int):
    """Evaluates `rows` leading rows of both ops, one contiguous slice of rows per thread."""
    from oracle.oracle import BINARY_OPS, DTYPES, _arr

    per = [rows * t // threads for t in range(threads + 1)]
    f = ev._f["broadcast"]
    extra = [1] if ev.threaded else []

    def work(lo, hi, op):
        if hi <= lo:
            return
        m = meta_rows(hi - lo)
        total = (hi - lo) * 512 * 4096
        rc = f(BINARY_OPS[op], DTYPES[np.dtype(np.float32)], out.ctypes.data + lo * 512 * 4096 * 4,
               a.ctypes.data + lo * 4096 * 4, b.ctypes.data, m["cdims"], _arr(m["sr"]), _arr(m["sa"]), _arr(m["sb"]),
               total, *extra)
        assert rc == 0

    for op in OPS:
        ths = [threading.Thread(target=work, args=(per[t], per[t + 1], op)) for t in range(threads)]
        for t in ths:
            t.start()
        for t in ths:
            t.join()


def cpu_c2_sampler(threads: int, target_s: float):
    """Returns (run_sample(), sample_rows, bytes_per_sample, kind)."""
    ev, kind = cpu_evaluator()
    a, b = c2_inputs_numpy(0)
    cache = {}

    def meta_rows(r):
        if r not in cache:
            cache[r] = ev.binary_meta([r, 1, 4096], [4096, 4096, 1], B_SHAPE, [2097152, 4096, 1])
        return cache[r]

    threads = max(1, min(threads, 256))
    rows = threads
    out = np.empty((256, 512, 4096), dtype=np.float32)
    t0 = time.perf_counter()
    cpu_c2_step(ev, meta_rows, a, b, out, rows, threads)
    dt = time.perf_counter() - t0
    # scale the sample to about target_s of wall time, in whole rows per thread
    rows = int(min(256, max(rows, rows * target_s / max(dt, 1e-6))))
    rows = max(threads, rows // threads * threads)
    bytes_per = 2 * (rows * 512 * 4096 + rows * 4096 + 512 * 4096) * 4

    def run():
        cpu_c2_step(ev, meta_rows, a, b, out, rows, threads)

    return run, rows, bytes_per, kind


def cpu_baseline_line(threads: int, target_s: float = 10.0):
    run, rows, bytes_per, kind = cpu_c2_sampler(threads, target_s)
    reps, dt = 0, 0.0
    while reps == 0 or dt < 0.5 * target_s:
        t0 = time.perf_counter()
        run()
        dt += time.perf_counter() - t0
        reps += 1
    return {"value": round(bytes_per * reps / dt / 1e9, 4), "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"C2 Add+Mul on the first {rows} of 256 rows of a ({rows}x512x4096 outputs per op), x{reps}, "
                      f"{'the reference CPU loop (Matrix.mm:7475-7567) compiled from its tree' if kind == 'reference' else 'oracle restatement'}, "
                      f"{threads} thread(s) over row slices, {dt:.2f} s"}


def cpu_sum_runner(ev, sample, threads: int):
    """One pass of the reference's Sum loop over the flat float32 `sample`: `threads` contiguous slices,
    each summed by the loop on its own host thread (the loop itself is single-threaded: Matrix.mm:
    15193-15205), then the slices' partial sums added in order."""
    n = sample.size
    per = [n * t // threads for t in range(threads + 1)]
    metas = {}
    parts = [np.float32(0)] * threads

    def work(t):
        lo, hi = per[t], per[t + 1]
        if hi <= lo:
            return
        m = metas.setdefault(hi - lo, ev.reduce_meta([hi - lo], [1], 0))
        parts[t] = ev.reduce_raw("sum", sample, lo, m)

    def run():
        ths = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        acc = np.float32(0)
        for v in parts:
            acc = np.float32(acc + np.float32(v))
        return acc

    return run


def cpu_c5b_sampler(threads: int, target_s: float, sample=None):
    """(run, elements, kind): a bounded sample of config 5b (a prefix of the flattened input, or seeded
    N(0,1) values when no sample is given) sized so one pass takes about target_s seconds."""
    ev, kind = cpu_evaluator()
    threads = max(1, threads)
    if sample is None:
        sample = np.random.default_rng([5, 0]).standard_normal(1 << 27, dtype=np.float32)
    n = min(sample.size, max(threads * 4096, 1 << 22))
    t0 = time.perf_counter()
    cpu_sum_runner(ev, sample[:n], threads)()
    dt = max(time.perf_counter() - t0, 1e-6)
    n = int(min(sample.size, max(threads * 4096, n * target_s / dt)))
    return cpu_sum_runner(ev, sample[:n], threads), n, kind


def cpu_c5b_line(threads: int, target_s: float, sample=None):
    run, n, kind = cpu_c5b_sampler(threads, target_s / 8, sample)
    reps, dt = 0, 0.0
    while reps == 0 or dt < 0.5 * target_s:
        t0 = time.perf_counter()
        run()
        dt += time.perf_counter() - t0
        reps += 1
    what = ("the reference CPU Sum loop (Matrix.mm:15193-15205) compiled from its tree" if kind == "reference"
            else "oracle restatement of the Sum loop")
    return {"value": round(n * 4 * reps / dt / 1e9, 4), "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"C5b: the first {n:,} of the 2^32 elements ({n * 4 / 2**20:.0f} MiB), x{reps}, {what}, "
                      f"{threads} thread(s) over contiguous slices of the flattened input, partials added in "
                      f"order, {dt:.2f} s"}


def suite_cpu_hook():
    """CPU leg of the --suite lines: the reference's own loop (oracle/_ref, else the restatement) on a
    leading-axis slice of the config's input, timed on one host core, and the GPU's result for the same
    slice compared with it (bit-exact, or the float-sum rule: within 1e-5 * sum|x| of the CPU or of the
    exact fp64 sum)."""
    import numpy as np

    from oracle import oracle

    ev = oracle.reference()
    kind = "reference"
    if ev is None:
        ev, kind = oracle.port(), "port"

    def hook(line, spec):
        import torch

        xs = spec["sample"].contiguous()
        a = xs.cpu().numpy()
        g = spec["gpu"](xs)
        torch.cuda.synchronize()
        g = g.cpu().numpy()
        t0 = time.perf_counter()
        c = spec["cpu"](ev, a)
        dt = time.perf_counter() - t0
        line["cpu_reference"] = {"GB/s": round(a.nbytes / dt / 1e9, 4), "cores": 1, "kind": kind,
                                 "sample": spec["desc"], "ms": round(dt * 1e3, 2)}
        with np.errstate(invalid="ignore"):
            if spec["kind"] == "exact":
                ok = g.shape == c.shape and bool(np.array_equal(g, c, equal_nan=True))
                verdict = "bit-exact" if ok else "MISMATCH"
            elif spec["kind"] == "softmax":
                x64 = a.astype(np.float64)
                e = np.exp(x64 - x64.max(-1, keepdims=True))
                e /= e.sum(-1, keepdims=True)
                ok = bool((np.abs(g - c) <= 1e-5 * np.abs(c) + 1e-30).all() or
                          (np.abs(g - e) <= 1e-5 * e + 1e-30).all())
                verdict = "within rel 1e-5" if ok else "MISMATCH"
            else:
                x64 = a.astype(np.float64)
                ax = spec["axis"]
                exact = x64.sum(axis=ax)
                tol = 1e-5 * np.abs(x64).sum(axis=ax) + 1e-30
                ok = bool(((np.abs(g - c) <= tol) | (np.abs(g - exact) <= tol)).all())
                verdict = "within 1e-5 * sum|x|" if ok else "MISMATCH"
        line["parity_on_sample"] = verdict

    return hook


# ------------------------------------------------------------------------------------------
# reference arm
# ------------------------------------------------------------------------------------------
def run_reference(args):
    """The reference's own CPU path for the selected workload, on rank 0 only, with every host thread."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    if args.workload == "c2":
        run, rows, bytes_per, kind = cpu_c2_sampler(threads, target_s=2.0)
        workload = {"workload": WORKLOAD, "ops": list(OPS), "sample_rows": rows,
                    "parallelism": f"{threads} host threads"}
        sample = f"{rows} of 256 rows of a per step ({rows}x512x4096 outputs per op), one row slice per thread"
        scaling, data = "weak", "synthetic (seeded U(-1,1))"
    elif args.workload == "c5b":
        # each step a bounded sample: about a minute for the whole run, at most 0.25 s per step
        per_step = min(0.25, 60.0 / max(1, args.steps + args.warmup))
        run, n, kind = cpu_c5b_sampler(threads, per_step)
        bytes_per = n * 4
        workload = {"workload": C5B_WORKLOAD, "sample_elements": n, "parallelism": f"{threads} host threads"}
        sample = (f"the first {n:,} of the 2^32 elements per step ({bytes_per / 2**20:.0f} MiB, seeded N(0,1)), one "
                  f"contiguous slice per thread, each summed by the reference loop, partials added in order")
        scaling, data = "strong", "synthetic (seeded N(0,1))"
    else:
        print(json.dumps({"impl": "reference", "unavailable": f"--impl reference covers c5b and c2, not {args.workload}"}))
        return 0
    for _ in range(args.warmup):
        run()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = bytes_per * args.steps / total / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": data,
        "config": workload,
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------
def run_c2(args):
    import torch
    import torch.distributed as dist

    from matrix_b200 import _abi, backend

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    backend.init(local)
    stream = torch.cuda.current_stream(dev)
    L = _abi.lib()

    a_shape, out_shape, op_bytes = c2_shapes(args.rows)
    a_np, b_np = c2_inputs_numpy(rank)
    a_np = np.ascontiguousarray(a_np[:args.rows])
    a = torch.from_numpy(a_np).to(dev)
    b = torch.from_numpy(b_np).to(dev)
    outs = {op: torch.empty(out_shape, dtype=torch.float32, device=dev) for op in OPS}
    meta = backend.binary_meta(a_shape, list(a.stride()), B_SHAPE, list(b.stride()))

    def step(ev_pairs=None):
        for op in OPS:
            if ev_pairs is not None:
                ev_pairs[op][0].record(stream)
            backend.binary_launch(op, a.data_ptr(), b.data_ptr(), 0, outs[op].data_ptr(), meta)
            if ev_pairs is not None:
                ev_pairs[op][1].record(stream)

    # correctness spot check (not timed): single IEEE op per element, so numpy matches exactly
    step()
    torch.cuda.synchronize()
    for op, fn in (("add", np.add), ("mul", np.multiply)):
        got = outs[op][::13].cpu().numpy()
        want = fn(a_np[::13], b_np)
        if got.tobytes() != want.tobytes():
            raise SystemExit(f"bench: {op} output differs from the reference semantics")

    sampler = None
    if rank == 0:
        uuids = []
        for i in range(torch.cuda.device_count()):
            try:
                uuids.append(str(torch.cuda.get_device_properties(i).uuid))
            except Exception:
                pass
        sampler = ClockSampler(uuids[:world] if world > 1 else uuids[local:local + 1])
        sampler.start()
        time.sleep(0.3)

    for _ in range(args.warmup):
        step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    per_launch = []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pairs = [{op: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for op in OPS}
             for _ in range(args.steps)]
    start.record(stream)
    for k in range(args.steps):
        step(pairs[k])
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed_ms = start.elapsed_time(end)
    for pr in pairs:
        for op in OPS:
            per_launch.append(pr[op][0].elapsed_time(pr[op][1]))
    clocks = sampler.stop() if sampler else None

    # e2e through the C ABI with host buffers: upload a and b from pinned memory, run both
    # ops, read both results back into pinned memory, every step
    e2e_steps = 0 if args.no_e2e else max(3, min(args.steps, 5))
    h_a = torch.from_numpy(a_np).pin_memory()
    h_b = torch.from_numpy(b_np).pin_memory()
    h_out = torch.empty(out_shape if e2e_steps else [1], dtype=torch.float32).pin_memory()
    nbytes_out = outs["add"].numel() * 4

    def e2e_step():
        _abi.check(L.mtxc_upload(a.data_ptr(), h_a.data_ptr(), a.numel() * 4))
        _abi.check(L.mtxc_upload(b.data_ptr(), h_b.data_ptr(), b.numel() * 4))
        for op in OPS:
            backend.binary_launch(op, a.data_ptr(), b.data_ptr(), 0, outs[op].data_ptr(), meta)
            _abi.check(L.mtxc_download(h_out.data_ptr(), outs[op].data_ptr(), nbytes_out))
        _abi.check(L.mtxc_sync())

    e2e_ms = 0.0
    if e2e_steps:
        e2e_step()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1)

    t = torch.tensor([elapsed_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_ms = float(t[0]), float(t[1])
    sustained = sustained_copy_gbs(dev, stream, elapsed_ms) if rank == 0 and args.rows == 256 else None

    if rank == 0:
        peak, peak_kind = measured_peak()
        avg_launch_s = statistics.mean(per_launch) / 1e3
        achieved = op_bytes / avg_launch_s / 1e9
        traffic = profile_traffic() if args.rows == 256 else None
        total_bytes = op_bytes * len(OPS) * args.steps * world
        value = total_bytes / (elapsed_ms / 1e3) / 1e9
        e2e_value = op_bytes * len(OPS) * e2e_steps * world / (e2e_ms / 1e3) / 1e9 if e2e_steps else None
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded U(-1,1))",
            "config": {"workload": WORKLOAD if args.rows == 256 else f"{WORKLOAD} ({args.rows}-row slice of a)",
                       "ops": list(OPS), "bytes_per_op": op_bytes,
                       "l2": "outputs (2 GiB per op) exceed L2; the broadcast operands a, b (12 MiB) stay L2-resident by design",
                       "parallelism": f"weak: a sharded on its leading axis over {world} GPU(s), b replicated, no collective"},
            "frac_of_hbm_peak": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "broadcast_group_kernel", "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                         if peak_kind == "measured" else "fallback 6.65 TB/s",
                         "sustained_copy_gbs": sustained,
                         "frac_of_sustained_copy": round(achieved / sustained, 4) if sustained else None,
                         "sustained_note": "a device copy of random f32 (2 GiB read + 2 GiB written per copy) back to "
                                           "back for as long as the timed region, on the same GPU right after it: the "
                                           "bandwidth a long stream keeps under the 1 kW power cap"},
            "clocks": clocks,
            "e2e": {"value": round(e2e_value, 3) if e2e_value else None, "unit": UNIT,
                    "h2d_bytes_per_step": (a.numel() + b.numel()) * 4, "d2h_bytes_per_step": nbytes_out * len(OPS),
                    "steps": e2e_steps, "path": "mtxc_upload + mtxc_broadcast_binary + mtxc_download (pinned host)"},
            "gpu_launches": len(OPS) * args.steps,
        }
        if world == 1 and not args.no_cpu and args.rows == 256:
            line["cpu_baseline"] = cpu_baseline_line(os.cpu_count() or 1, target_s=args.cpu_seconds)
            # the reference's loop is single-threaded: its own one-core speed, beside the row-sliced figure
            one = cpu_baseline_line(1, target_s=max(2.0, args.cpu_seconds / 3))
            line["cpu_baseline"]["single_thread"] = {"value": one["value"], "cores": 1, "sample": one["sample"]}
        print(json.dumps(line), flush=True)
        if args.suite:
            from matrix_b200 import suite

            cfgs = args.suite_configs.split(",") if args.suite_configs else None
            hook = None if args.no_cpu else suite_cpu_hook()
            for extra in suite.run_all(dev, stream, cfgs, args.suite_scale, cpu_hook=hook):
                print(json.dumps(extra), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_c5b(args):
    """The headline: config 5b, a full Sum of 2^32 f32 values, rows sharded over the ranks (strong
    scaling), through the C ABI: mtxc_reduce for sum(1) on the main stream, mtxc_reduce_sharded for sum(0)
    (local sum, NCCL all-gather, ordered merge) on a side stream, double-buffered so the exchange of one
    step overlaps the next step's row reduction."""
    import datetime

    import torch
    import torch.distributed as dist

    from matrix_b200 import _abi, backend
    from matrix_b200.shard import NativeComm, shard_range

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    backend.init(local)
    L = _abi.lib()
    main_s = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)
    comm = NativeComm()
    cols = args.cols
    lo, hi = shard_range(C5B_ROWS, world, rank)
    rows = hi - lo
    total_bytes = C5B_ROWS * cols * 4
    local_bytes = rows * cols * 4
    x = torch.empty((rows, cols), dtype=torch.float32, device=dev)
    fill_c5b_rows(x, lo)
    parts = [torch.empty(rows, dtype=torch.float32, device=dev) for _ in range(2)]
    outs = [torch.empty((), dtype=torch.float32, device=dev) for _ in range(2)]
    m1 = backend.reduce_meta([rows, cols], [cols, 1], 1)   # x.sum(1): this rank's rows
    m0 = backend.reduce_meta([rows], [1], 0)               # .sum(0): over the sharded axis
    f32 = backend.dtype_code(torch.float32)
    done = [torch.cuda.Event(), torch.cuda.Event()]
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    for ev in done:
        ev.record(main_s)

    def step(k, ev_pair=None):
        b = k % 2
        main_s.wait_event(done[b])                       # partial buffer b is free again
        if ev_pair is not None:
            ev_pair[0].record(main_s)
        backend.reduce_launch("sum", x.data_ptr(), f32, parts[b].data_ptr(), m1)
        if ev_pair is not None:
            ev_pair[1].record(main_s)
        ready[b].record(main_s)
        side.wait_event(ready[b])
        backend.set_stream(side)
        backend.reduce_sharded_launch("sum", parts[b].data_ptr(), f32, outs[b].data_ptr(), m0)
        backend.set_stream(main_s)
        done[b].record(side)
        return outs[b]

    result = step(0)
    torch.cuda.synchronize()
    sampler = None
    if rank == 0:
        uuids = []
        for i in range(torch.cuda.device_count()):
            try:
                uuids.append(str(torch.cuda.get_device_properties(i).uuid))
            except Exception:
                pass
        sampler = ClockSampler(uuids[:world] if world > 1 else uuids[local:local + 1])
        sampler.start()
        time.sleep(0.3)
    for k in range(args.warmup):
        step(k)
    main_s.wait_stream(side)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main_s)
    h0 = time.perf_counter()
    for k in range(args.steps):
        result = step(k, pairs[k])
    host_s = time.perf_counter() - h0
    main_s.wait_stream(side)                             # the last exchange is inside the timed region
    e1.record(main_s)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed_ms = e0.elapsed_time(e1)
    launch_ms = [a.elapsed_time(b) for a, b in pairs]
    clocks = sampler.stop() if sampler else None

    # correctness gate: the fp64 sum of the same tensor (torch, a reference value only) and the float-sum
    # rule |got - exact| <= 1e-5 * sum|x|
    exact = torch.zeros((), dtype=torch.float64, device=dev)
    absum = torch.zeros((), dtype=torch.float64, device=dev)
    for r in range(rows):
        exact += x[r].sum(dtype=torch.float64)
        absum += x[r].abs().sum(dtype=torch.float64)
    if world > 1:  # each rank holds its own rows: the whole tensor's sums
        dist.all_reduce(exact)
        dist.all_reduce(absum)
    # e2e through the C ABI with host buffers: each rank uploads its rows from pinned memory, reduces,
    # exchanges and reads the result back into pinned memory, every step
    e2e_steps = 0 if args.no_e2e else 3
    e2e_ms = 0.0
    if e2e_steps:
        hbuf = C.c_void_p()
        _abi.check(L.mtxc_host_alloc(local_bytes, C.byref(hbuf)))
        hout = C.c_void_p()
        _abi.check(L.mtxc_host_alloc(4, C.byref(hout)))
        _abi.check(L.mtxc_download(hbuf, x.data_ptr(), local_bytes))
        _abi.check(L.mtxc_sync())

        def e2e_step():
            _abi.check(L.mtxc_upload(x.data_ptr(), hbuf, local_bytes))
            backend.reduce_launch("sum", x.data_ptr(), f32, parts[0].data_ptr(), m1)
            backend.reduce_sharded_launch("sum", parts[0].data_ptr(), f32, outs[0].data_ptr(), m0)
            _abi.check(L.mtxc_download(hout, outs[0].data_ptr(), 4))
            _abi.check(L.mtxc_sync())

        e2e_step()
        if world > 1:
            dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(main_s)
        for _ in range(e2e_steps):
            e2e_step()
        a1.record(main_s)
        torch.cuda.synchronize()
        e2e_ms = a0.elapsed_time(a1)
        e2e_result = C.c_float.from_address(hout.value).value
        _abi.check(L.mtxc_host_free(hbuf))
        _abi.check(L.mtxc_host_free(hout))
    got = float(result.item())
    ok = abs(got - float(exact.item())) <= 1e-5 * float(absum.item())
    if e2e_steps:
        ok = ok and e2e_result == got  # the same kernels on the same data: the same bits
    t = torch.tensor([elapsed_ms, e2e_ms, host_s * 1e3, 0.0 if ok else 1.0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_ms, host_ms, bad = (float(v) for v in t.tolist())
    ok = bad == 0.0
    if rank == 0:
        peak, peak_kind = measured_peak()
        avg_launch_s = statistics.mean(launch_ms) / 1e3
        achieved = local_bytes / avg_launch_s / 1e9
        per_byte = profile_traffic_c5b()
        value = total_bytes * args.steps / (elapsed_ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) per row)",
            "config": {"workload": C5B_WORKLOAD if cols == C5B_COLS else f"{C5B_WORKLOAD} ([8, {cols}] case)",
                       "elements": C5B_ROWS * cols, "bytes_per_step": total_bytes,
                       "l2": "input (16 GiB; 16/N GiB per GPU) far larger than L2: every step streams it from HBM",
                       "parallelism": f"strong: {C5B_ROWS} rows over {world} GPU(s) ({rows} per GPU), sum(0) over the "
                                      f"sharded axis by mtxc_reduce_sharded (NCCL all-gather + ordered merge)"},
            "frac_of_hbm_peak": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": round(per_byte * local_bytes) if per_byte else None,
                         "kernel": "reduce_rows_kernel<SUM,float,256> (+ its split finalize)",
                         "bytes_per_launch": local_bytes,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, a read+write copy burst)"
                         if peak_kind == "measured" else "fallback 6.65 TB/s",
                         "traffic_source": "ncu DRAM read+write bytes per input byte of a [8, 2^24] launch "
                                           "(profiles/reduce_rows_c5b_traffic.txt), scaled to this launch"},
            "clocks": clocks,
            "e2e": {"value": round(total_bytes * e2e_steps / (e2e_ms / 1e3) / 1e9, 3) if e2e_steps else None,
                    "unit": UNIT, "h2d_bytes_per_step": total_bytes if e2e_steps else 0,
                    "d2h_bytes_per_step": 4 * world if e2e_steps else 0, "steps": e2e_steps,
                    "path": "per rank: mtxc_upload of its rows from pinned host memory + mtxc_reduce + "
                            "mtxc_reduce_sharded + mtxc_download of the result into pinned memory + mtxc_sync"},
            "host_enqueue_ms_per_step": round(host_ms / args.steps, 4),
            "within_tolerance_of_fp64": ok,
            "gpu_launches": 4 * args.steps,
        }
        if world == 1 and not args.no_cpu:
            sample = x[0, : 1 << 28].cpu().numpy()
            line["cpu_baseline"] = cpu_c5b_line(os.cpu_count() or 1, args.cpu_seconds, sample)
            one = cpu_c5b_line(1, max(2.0, args.cpu_seconds / 3), sample)
            line["cpu_baseline"]["single_thread"] = {"value": one["value"], "cores": 1, "sample": one["sample"]}
        print(json.dumps(line), flush=True)
        if args.suite:
            from matrix_b200 import suite

            del x
            torch.cuda.empty_cache()
            cfgs = args.suite_configs.split(",") if args.suite_configs else None
            hook = None if args.no_cpu else suite_cpu_hook()
            for extra in suite.run_all(dev, main_s, cfgs, args.suite_scale, cpu_hook=hook):
                print(json.dumps(extra), flush=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # every rank's exchanges are done before any rank releases its buffers
    comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if ok else 1


def sustained_copy_gbs(dev, stream, ms_target: float) -> float:
    """Bandwidth of a plain device copy of random f32 data (torch's copy kernel, used only as a
    reference denominator), run back to back for about `ms_target` ms: what a memory stream sustains
    once the power cap is reached, next to the burst copy figure in MEASURED_PEAKS.json."""
    import torch

    n = 1 << 29  # 2 GiB
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    src = torch.rand(n, generator=g, device=dev)
    dst = torch.empty_like(src)
    for _ in range(3):
        dst.copy_(src)
    copies = max(3, int(ms_target / 0.66))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(copies):
        dst.copy_(src)
    e1.record(stream)
    torch.cuda.synchronize()
    gbs = copies * 2 * n * 4 / (e0.elapsed_time(e1) / 1e3) / 1e9
    del src, dst
    return round(gbs, 1)


# ------------------------------------------------------------------------------------------
# sharded reductions (configs 4 and 5b): the reduced axis is the sharded one
# ------------------------------------------------------------------------------------------
def run_sharded(args):
    """A benchmark config sharded over the GPUs on its leading axis (strong scaling: the total is fixed).
    C4: Sum over axes (0, 2) of f32 [32, 4096, 2048]; the sharded axis is a reduced one, so a step is the
    local sum(2) and mtxc_reduce_sharded for sum(0) (local sum, NCCL all-gather of the per-rank partials,
    ordered merge).  C1 (Sum of the last axis), C3 (Max and ArgMax over axis 1) and C5a (fused softmax)
    shard an axis they do not reduce: no collective.  (C5b, the headline, is run_c5b.)"""
    import datetime

    import torch
    import torch.distributed as dist

    from matrix_b200 import _abi, backend
    from matrix_b200.shard import NativeComm, reduce_sharded, shard_range

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    else:  # one rank: an in-process store, nothing to rendezvous with
        dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    backend.init(local)
    stream = torch.cuda.current_stream(dev)
    wl = args.workload
    collective = wl == "c4"
    comm = NativeComm() if collective else None
    if wl == "c4":
        rows, cols = 32, 4096 * 2048
        shape = (32, 4096, 2048)
        desc = "C4: Sum over axes (0,2) of f32 [32,4096,2048] ~ N(0,1), axis 0 sharded, all-gather + ordered merge"
    elif wl == "c1":
        rows, cols = 1024, 4096
        shape = (rows, cols)
        desc = "C1: Sum(axis=-1) of f32 [1024,4096] ~ N(0,1), rows sharded, no collective (16 MiB: L2-resident after warm-up)"
    elif wl == "c3":
        rows, cols = 64, 8192 * 1024
        shape = (64, 8192, 1024)
        desc = "C3: Max and ArgMax(axis=1) of f32 [64,8192,1024] floor(U*256)/256, axis 0 sharded, no collective"
    else:
        rows, cols = 8192, 32768
        shape = (rows, cols)
        desc = "C5a: softmax over the last axis of f32 [8192,32768] ~ N(0,4), fused kernel, rows sharded, no collective"
    lo, hi = shard_range(rows, world, rank)
    x = torch.empty((hi - lo, *shape[1:]), device=dev)
    g = torch.Generator(device=dev)
    for r in range(lo, hi):  # every global row from its own seed: the tensor does not depend on N
        g.manual_seed(1000 + r)
        if wl == "c3":
            x[r - lo].uniform_(generator=g)
            x[r - lo].mul_(256).floor_().div_(256)
        else:
            x[r - lo].normal_(generator=g)
            if wl == "c5a":
                x[r - lo].mul_(2.0)
    # algorithmic bytes per step: every op reads its input once and writes its output
    if wl == "c3":
        total_bytes = 2 * (rows * cols * 4 + rows * 1024 * 4)
    elif wl == "c5a":
        total_bytes = 2 * rows * cols * 4
    elif wl == "c1":
        total_bytes = rows * cols * 4 + rows * 4
    else:
        total_bytes = rows * cols * 4

    # C4: the local reduction of step k + 1 overlaps the exchange of step k.  The local partials go to
    # one of two buffers on the main stream; the all-gather and the ordered merge of that buffer run on a
    # side stream, which waits for the partials, and the main stream does not overwrite a buffer before
    # the side stream is done with it.
    side = torch.cuda.Stream(dev)
    if collective:
        parts = [backend.reduce("sum", x, 2) for _ in range(2)]
        local_meta = backend.reduce_meta(list(x.shape), list(x.stride()), 2)
        shard_meta = backend.reduce_meta(list(parts[0].shape), list(parts[0].stride()), 0)
        merged = [torch.empty(4096, dtype=torch.float32, device=dev) for _ in range(2)]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    for ev in done:
        ev.record(stream)
    counter = [0]

    def exchange_step():
        k = counter[0] % 2
        counter[0] += 1
        stream.wait_event(done[k])                                # buffer k free again
        backend.reduce("sum", x, 2, out=parts[k], meta=local_meta)  # local axis: no collective
        ready = torch.cuda.Event()
        ready.record(stream)
        side.wait_event(ready)
        with torch.cuda.stream(side):
            backend.set_stream(side)
            try:
                r = reduce_sharded("sum", parts[k], 0, rows, comm=comm, out=merged[k], meta=shard_meta)
            finally:
                backend.set_stream(stream)
            done[k].record(side)
        return r

    def step():
        if collective:
            return exchange_step()
        if wl == "c1":
            return backend.reduce("sum", x, 1)
        if wl == "c3":
            return backend.reduce("max", x, 1), backend.reduce("argmax", x, 1)
        return backend.softmax_lastdim(x)

    result = step()
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        step()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # a bounded sleep kernel (~0.5 ms per step, outside the timed region) keeps the GPU busy while the
    # host queues the K steps, so the events time the device work rather than the host's launch rate
    # (C1's 16 MiB step is shorter than one Python launch; a C4 step on 8 GPUs is ~24 us of device work
    # behind ~130 us of Python enqueueing its reduction, NCCL all-gather and merge, measured on one B200)
    torch.cuda._sleep(1_000_000 * args.steps)
    e0.record(stream)
    for _ in range(args.steps):
        result = step()
    if collective:
        stream.wait_stream(side)  # the last exchange is inside the timed region
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = e0.elapsed_time(e1)
    # the same steps without the pre-roll: what a caller sees when the host's enqueue rate limits the device
    e0.record(stream)
    h0 = time.perf_counter()
    for _ in range(args.steps):
        result = step()
    host_ms = (time.perf_counter() - h0) * 1e3
    if collective:
        stream.wait_stream(side)
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms_visible = e0.elapsed_time(e1)
    # C4, recorded: GRAPH_STEPS exchange steps captured once into a CUDA graph (mtxc_graph_begin / end on
    # the main stream; the side stream joins through the captured events) and replayed, as a compiled trace
    # runs them; the host then enqueues one graph launch per GRAPH_STEPS steps
    graph_ms = graph_host_ms = 0.0
    graph_steps = 0
    if collective and not args.no_graph:
        L = _abi.lib()
        GRAPH_STEPS = 8
        cs = torch.cuda.Stream(dev)                              # capture needs a stream other than the default
        torch.cuda.synchronize()
        cap_done = [None, None]

        def captured_step(j):
            k = j % 2
            if cap_done[k] is not None:
                cs.wait_event(cap_done[k])                      # buffer k free again (inside the graph)
            backend.reduce("sum", x, 2, out=parts[k], meta=local_meta)
            ready = torch.cuda.Event()
            ready.record(cs)
            side.wait_event(ready)
            backend.set_stream(side)
            try:
                reduce_sharded("sum", parts[k], 0, rows, comm=comm, out=merged[k], meta=shard_meta)
            finally:
                backend.set_stream(cs)
            ev = torch.cuda.Event()
            ev.record(side)
            cap_done[k] = ev

        backend.set_stream(cs)
        g = C.c_void_p()
        try:
            _abi.check(L.mtxc_graph_begin())
            try:
                for j in range(GRAPH_STEPS):
                    captured_step(j)
                cs.wait_stream(side)                             # join: the graph ends after its last exchange
            finally:
                rc_end = L.mtxc_graph_end(C.byref(g))
            _abi.check(rc_end)
            reps = max(1, args.steps // GRAPH_STEPS)
            for _ in range(2):
                _abi.check(L.mtxc_graph_launch(g))
            torch.cuda.synchronize()
            dist.barrier()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(cs)
            h0 = time.perf_counter()
            for _ in range(reps):
                _abi.check(L.mtxc_graph_launch(g))
            graph_host_ms = (time.perf_counter() - h0) * 1e3
            g1.record(cs)
            torch.cuda.synchronize()
            dist.barrier()
            graph_ms = g0.elapsed_time(g1)
            graph_steps = reps * GRAPH_STEPS
        finally:
            if g.value:
                _abi.check(L.mtxc_graph_destroy(g))             # released before the communicator
            backend.set_stream(stream)
        result = merged[(GRAPH_STEPS - 1) % 2]
    t = torch.tensor([ms, ms_visible, host_ms, graph_ms, graph_host_ms], dtype=torch.float64,
                     device=dev if world > 1 else "cpu")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_visible, host_ms, graph_ms, graph_host_ms = (float(v) for v in t.tolist())
    # correctness against torch on the same tensor (a reference value only, never the measured path)
    if collective:
        dims = (0, 2)
        ref = x.sum(dim=dims, dtype=torch.float64)
        absum = x.abs().sum(dim=dims, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(ref)
            dist.all_reduce(absum)
        ok = bool(((result.double() - ref).abs() <= 1e-5 * absum + 1e-30).all())
    elif wl == "c1":
        ok = bool(((result.double() - x.sum(1, dtype=torch.float64)).abs()
                   <= 1e-5 * x.abs().sum(1, dtype=torch.float64)).all())
    elif wl == "c3":
        vals, idx = result
        ok = bool(torch.equal(vals, x.amax(1)) and torch.equal(idx.long(), x.argmax(1)))
    else:
        want = torch.softmax(x.double(), dim=-1)
        ok = bool(((result.double() - want).abs() <= 1e-5 * want + 1e-30).all())
    if world > 1:
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = bool(flag.item())
    if rank == 0:
        peak, _ = measured_peak()
        value = total_bytes * args.steps / (ms / 1e3) / 1e9
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) per row)",
                "config": {"workload": desc, "parallelism": f"axis 0 sharded over {world} GPU(s)",
                           "l2": "input L2-resident (16 MiB)" if wl == "c1" else "input larger than L2"},
                "frac_of_hbm_peak": round(value / world / peak, 4), "within_tolerance_of_fp64": ok,
                "host_visible": {"value": round(total_bytes * args.steps / (ms_visible / 1e3) / 1e9, 2),
                                 "ms_per_step": round(ms_visible / args.steps, 4),
                                 "host_enqueue_ms_per_step": round(host_ms / args.steps, 4),
                                 "note": "the same steps timed without the pre-roll sleep: device time including "
                                         "any gaps the host's enqueue rate leaves"}}
        if graph_steps:
            line["recorded"] = {"value": round(total_bytes * graph_steps / (graph_ms / 1e3) / 1e9, 2),
                                "ms_per_step": round(graph_ms / graph_steps, 4), "steps": graph_steps,
                                "host_enqueue_ms_per_step": round(graph_host_ms / graph_steps, 4),
                                "note": "8 exchange steps recorded once into a CUDA graph (the NCCL all-gather "
                                        "included) and replayed, no pre-roll: one graph launch per 8 steps"}
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    dist.barrier()  # every rank's exchanges are done before any rank releases its buffers
    if comm is not None:
        comm.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0 if ok else 1


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--suite", action="store_true", help="also time the other benchmark configs")
    ap.add_argument("--suite-configs", default="", help="comma-separated subset of C1,C3,C4,C5a,C5b,F2,F3,F4,F5,F6,F7,F8")
    ap.add_argument("--suite-scale", type=int, default=1, help="divide the configs' leading extent (small cases)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--rows", type=int, default=256, help="c2: leading rows of a per rank (256 = C2; smaller for ncu)")
    ap.add_argument("--cols", type=int, default=C5B_COLS, help="c5b: row length (2^29 = C5b; smaller for ncu)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end measurement")
    ap.add_argument("--no-graph", action="store_true", help="c4: skip the recorded (CUDA graph) measurement")
    ap.add_argument("--workload", choices=["c5b", "c2", "c1", "c3", "c4", "c5a"], default="c5b",
                    help="c5b (default headline: the largest config, strong scaling with the exchange), c2 (weak "
                         "scaling, no collective), or another config sharded over the GPUs: c1, c3, c5a (no "
                         "collective), c4 (all-gather + ordered merge of the reduced-axis partials)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "c5b":
        return run_c5b(args)
    if args.workload == "c2":
        return run_c2(args)
    return run_sharded(args)


if __name__ == "__main__":
    raise SystemExit(main())
