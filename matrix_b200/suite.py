"""Device-time measurements of the other benchmark configurations (bench.py --suite).

Each config is run through the same C-ABI calls a user makes (matrix_b200.backend), with
seeded synthetic inputs generated on the device, 3 warm-up repetitions and the median of 20
timed repetitions (CUDA events on the launching stream).  Each line gives the fraction of the measured
copy bandwidth (MEASURED_PEAKS.json) and of the 8 TB/s nominal HBM3e peak.  Inputs larger than L2 are streamed
as they are; C1's 16 MiB input fits in L2, so L2 is flushed (a 512 MiB write) before each
repetition (by reading a 512 MiB buffer, which leaves no dirty lines to write back) and only the
reduction is timed.
"""
from __future__ import annotations

import json
import statistics
from pathlib import Path

import torch

from . import backend

REPO = Path(__file__).resolve().parent.parent
GiB = 1 << 30


def _peak() -> float:
    try:
        return float(json.loads((REPO / "MEASURED_PEAKS.json").read_text())["hbm_gbs"])
    except Exception:
        return 6650.0


SPEC_GBS = 8000.0  # B200 HBM3e nominal peak (~8 TB/s)


def _time(fn, stream, reps=20, warmup=3, flush=None):
    """Median device time of fn.  Before each repetition the stream is kept busy (the L2 flush, or a
    bounded sleep kernel of ~50 us) so that the start event, the launch and the end event are queued
    while the GPU works: the events then measure the kernels, not the host's launch latency."""
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(reps):
        if flush is not None:
            flush()
        else:
            torch.cuda._sleep(100_000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times)


def _line(name, workload, nbytes, ms, peak, **extra):
    gbs = nbytes / (ms / 1e3) / 1e9
    d = {"suite": name, "workload": workload, "algorithmic_bytes": nbytes, "ms": round(ms, 4),
         "GB/s": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4), "frac_of_spec_8tbs": round(gbs / SPEC_GBS, 4)}
    d.update(extra)
    return d


_CPU_HOOK = None


def _cpu(line, **spec):
    """Hands a config's sample to the caller's CPU-reference hook (bench.py: the reference's own loop
    timed on a leading-axis slice of the same input, and that slice's GPU result compared with it)."""
    if _CPU_HOOK is not None:
        _CPU_HOOK(line, spec)


def run_all(dev, stream, configs=None, scale=1, cpu_hook=None):
    """configs: names to run (default all: C1 C3 C4 C5a C5b, and F2 ... F8 for the statistics, astype,
    pointwise, mixed-dtype, half-precision and 1- / 2-byte kernels, and every dtype at equal bytes); scale:
    divide each config's leading extent by this (small cases for profiling)."""
    global _CPU_HOOK
    _CPU_HOOK = cpu_hook
    peak = _peak()
    g = torch.Generator(device=dev)
    out = []
    want = set(configs) if configs else {"C1", "C3", "C4", "C5a", "C5b", "F2", "F3", "F4", "F5", "F6", "F7", "F8"}

    # C1: Sum over the last axis of f32 [1024, 4096] ~ N(0,1)
    if "C1" in want:
        _c1(out, dev, stream, g, peak)
    if "C3" in want:
        _c3(out, dev, stream, g, peak, scale)
    if "C4" in want:
        _c4(out, dev, stream, g, peak, scale)
    if "C5a" in want:
        _c5a(out, dev, stream, g, peak, scale)
    if "C5b" in want:
        _c5b(out, dev, stream, g, peak, scale)
    if "F2" in want:
        _f2(out, dev, stream, g, peak, scale)
    if "F3" in want:
        _f3(out, dev, stream, g, peak, scale)
    if "F4" in want:
        _f4(out, dev, stream, g, peak, scale)
    if "F5" in want:
        _f5(out, dev, stream, g, peak, scale)
    if "F6" in want:
        _f6(out, dev, stream, g, peak, scale)
    if "F8" in want:
        _f8(out, dev, stream, g, peak, scale)
    if "F7" in want:
        _f7(out, dev, stream, g, peak, scale)
    torch.cuda.empty_cache()
    return out


def _c1(out, dev, stream, g, peak):
    g.manual_seed(0)
    x = torch.randn(1024, 4096, generator=g, device=dev)
    y = torch.empty(1024, device=dev)
    m = backend.reduce_meta([1024, 4096], [4096, 1], -1)
    scratch = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    scratch.fill_(1)
    sink = torch.empty((), dtype=torch.int64, device=dev)
    ms = _time(lambda: backend.reduce("sum", x, -1, out=y, meta=m), stream,
               flush=lambda: torch.sum(scratch, dim=0, out=sink))
    out.append(_line("C1", "Sum(axis=-1) f32 [1024,4096] (L2 flushed before each rep)", 1024 * 4096 * 4 + 4096, ms,
                     peak))
    _cpu(out[-1], sample=x, gpu=lambda t: backend.reduce("sum", t, -1), cpu=lambda ev, a: ev.reduce("sum", a, -1),
         kind="sum", axis=-1, desc="the whole input")
    # the same launch with the 16 MiB input resident in L2 (126 MB), as it is in a loop over one tensor
    ms = _time(lambda: backend.reduce("sum", x, -1, out=y, meta=m), stream)
    out.append(_line("C1-warm", "Sum(axis=-1) f32 [1024,4096], input L2-resident (not an HBM figure)",
                     1024 * 4096 * 4 + 4096, ms, peak, l2_resident=True))
    del x, y, scratch


def _c3(out, dev, stream, g, peak, scale):
    # C3: Max and ArgMax along axis 1 of f32 [64, 8192, 1024], values k/256
    b0 = max(1, 64 // scale)
    g.manual_seed(2)
    x = torch.floor(torch.rand(b0, 8192, 1024, generator=g, device=dev) * 256) / 256
    m = backend.reduce_meta([b0, 8192, 1024], list(x.stride()), 1)
    vmax = torch.empty(b0, 1024, device=dev)
    imax = torch.empty(b0, 1024, dtype=torch.int32, device=dev)
    nbytes = b0 * 8192 * 1024 * 4 + b0 * 1024 * 4
    ms = _time(lambda: backend.reduce("max", x, 1, out=vmax, meta=m), stream)
    out.append(_line("C3-max", "Max(axis=1) f32 [64,8192,1024]", nbytes, ms, peak))
    _cpu(out[-1], sample=x[:1], gpu=lambda t: backend.reduce("max", t, 1), cpu=lambda ev, a: ev.reduce("max", a, 1),
         kind="exact", desc="x[:1] (32 MiB)")
    ms = _time(lambda: backend.reduce("argmax", x, 1, out=imax, meta=m), stream)
    out.append(_line("C3-argmax", "ArgMax(axis=1) f32 [64,8192,1024]", nbytes, ms, peak))
    _cpu(out[-1], sample=x[:1], gpu=lambda t: backend.reduce("argmax", t, 1),
         cpu=lambda ev, a: ev.reduce("argmax", a, 1), kind="exact", desc="x[:1] (32 MiB)")
    ms = _time(lambda: backend.reduce_pair("max", x, 1, meta=m), stream)
    out.append(_line("C3-max+argmax", "Max and ArgMax(axis=1) from one read (mtxc_reduce_pair)", nbytes + b0 * 1024 * 4,
                     ms, peak, ops_served=2))
    del x


def _c4(out, dev, stream, g, peak, scale):
    # C4: Sum over axes (0, 2) of [32, 4096, 2048], f32 N(0,1) and i32 U{-1000..1000}
    b0 = max(1, 32 // scale)
    g.manual_seed(3)
    for name, x in (("C4-f32", torch.randn(b0, 4096, 2048, generator=g, device=dev)),
                    ("C4-i32", torch.randint(-1000, 1001, (b0, 4096, 2048), generator=g, device=dev,
                                             dtype=torch.int32))):
        m2 = backend.reduce_meta([b0, 4096, 2048], list(x.stride()), 2)
        mid = torch.empty(b0, 4096, dtype=x.dtype, device=dev)
        m0 = backend.reduce_meta([b0, 4096], [4096, 1], 0)
        fin = torch.empty(4096, dtype=x.dtype, device=dev)

        def c4():
            backend.reduce("sum", x, 2, out=mid, meta=m2)
            backend.reduce("sum", mid, 0, out=fin, meta=m0)

        ms = _time(c4, stream)
        out.append(_line(name, "x.sum(2).sum(0) [32,4096,2048]", b0 * 4096 * 2048 * 4 + 4096 * 4, ms, peak,
                         moved_bytes=b0 * 4096 * 2048 * 4 + 2 * b0 * 4096 * 4 + 4096 * 4))
        _cpu(out[-1], sample=x[:2], gpu=lambda t: backend.reduce("sum", backend.reduce("sum", t, 2), 0),
             cpu=lambda ev, a: ev.reduce("sum", ev.reduce("sum", a, 2), 0),
             kind="sum" if name == "C4-f32" else "exact", axis=(0, 2), desc="x[:2] (64 MiB)")
        del x, mid


def _c5a(out, dev, stream, g, peak, scale):
    # C5a: softmax trace on f32 [8192, 32768] ~ N(0, 4): max, sub, exp, sum, div (5 kernels)
    rows = max(1, 8192 // scale)
    g.manual_seed(4)
    x = torch.randn(rows, 32768, generator=g, device=dev) * 2
    mx = torch.empty(rows, 1, device=dev)
    t = torch.empty_like(x)
    s = torch.empty(rows, 1, device=dev)
    mm = backend.reduce_meta([rows, 32768], [32768, 1], -1, True)
    msub = backend.binary_meta([rows, 32768], [32768, 1], [rows, 1], [1, 1])
    mexp = backend.unary_meta([rows, 32768], [32768, 1])
    mdiv = msub

    def trace():
        backend.reduce("max", x, -1, True, out=mx, meta=mm)
        backend.binary("sub", x, mx, out=t, meta=msub)
        backend.exp(t, out=t, meta=mexp)
        backend.reduce("sum", t, -1, True, out=s, meta=mm)
        backend.binary("div", t, s, out=t, meta=mdiv)

    ms = _time(trace, stream)
    n = rows * 32768 * 4
    out.append(_line("C5a-trace", "softmax trace max,sub,exp,sum,div f32 [8192,32768] (5 kernels)", 2 * n, ms, peak,
                     moved_bytes=8 * n))
    ms = _time(lambda: backend.softmax_lastdim(x, out=t), stream)
    out.append(_line("C5a-fused", "softmax trace fused (mtxc_softmax_lastdim) f32 [8192,32768]", 2 * n, ms, peak,
                     moved_bytes=2 * n))

    def cpu_trace(ev, a):
        e = ev.unary("exp", ev.binary("sub", a, ev.reduce("max", a, -1, True)))
        return ev.binary("div", e, ev.reduce("sum", e, -1, True))

    _cpu(out[-1], sample=x[:16], gpu=lambda v: backend.softmax_lastdim(v), cpu=cpu_trace, kind="softmax",
         desc="x[:16] (2 MiB), the reference's five-primitive trace on the CPU")
    del x, t


def _c5b(out, dev, stream, g, peak, scale):
    # C5b: full Sum of 2^32 f32 ~ N(0,1) as [8, 2^29] (16 GiB): sum(1) then sum(0)
    cols = (1 << 29) // scale
    g.manual_seed(5)
    x = torch.randn(8, cols, generator=g, device=dev)
    r1 = torch.empty(8, device=dev)
    r0 = torch.empty((), device=dev)
    m1 = backend.reduce_meta([8, cols], [cols, 1], 1)
    m0 = backend.reduce_meta([8], [1], 0)

    def c5b():
        backend.reduce("sum", x, 1, out=r1, meta=m1)
        backend.reduce("sum", r1, 0, out=r0, meta=m0)

    ms = _time(c5b, stream, reps=5)
    out.append(_line("C5b", "full Sum f32 2^32 as [8,2^29] (1 GPU)", 8 * cols * 4, ms, peak))
    _cpu(out[-1], sample=x[:1, : 1 << 24], gpu=lambda t: backend.reduce("sum", t, 1),
         cpu=lambda ev, a: ev.reduce("sum", a, 1), kind="sum", axis=1, desc="x[:1, :2^24] (64 MiB)")
    del x


def _f2(out, dev, stream, g, peak, scale):
    """rms over the last axis of f32 [8192, 32768]: fused (one read) and as the reference's trace."""
    rows = max(8192 // scale, 1)
    g.manual_seed(6)
    x = torch.randn(rows, 32768, generator=g, device=dev)
    n = x.numel() * 4
    ms = _time(lambda: backend.stat("rms", x, 1), stream)
    out.append(_line("F2-rms", "rms(axis=-1) f32 [8192,32768] fused (mtxc_reduce_stat)", n + rows * 4, ms, peak))
    ms = _time(lambda: backend.stat("mean", x, 1), stream)
    out.append(_line("F2-mean", "mean(axis=-1) f32 [8192,32768] fused (mtxc_reduce_stat)", n + rows * 4, ms, peak))

    def trace():
        sq = backend.binary("mul", x, x)
        s = backend.reduce("sum", sq, 1)
        nd = torch.full((), 32768.0, device=dev)
        m = backend.binary("div", s, nd)
        return backend.unary("sqrt", m)

    ms = _time(trace, stream)
    out.append(_line("F2-rms-trace", "rms as the reference's trace: mul, sum, div, sqrt (4 kernels)", n + rows * 4, ms,
                     peak, moved_bytes=3 * n))
    del x


def _f3(out, dev, stream, g, peak, scale):
    """astype: f32 -> bf16 and u8 -> f32 over [8192, 32768]."""
    rows = max(8192 // scale, 1)
    g.manual_seed(7)
    x = torch.randn(rows, 32768, generator=g, device=dev)
    ms = _time(lambda: backend.astype(x, torch.bfloat16), stream)
    out.append(_line("F3-astype-f32-bf16", "astype f32 -> bf16 [8192,32768]", x.numel() * 6, ms, peak))
    u = torch.randint(0, 256, (rows, 32768), generator=g, device=dev, dtype=torch.int32).to(torch.uint8)
    del x
    ms = _time(lambda: backend.astype(u, torch.float32), stream)
    out.append(_line("F3-astype-u8-f32", "astype u8 -> f32 [8192,32768]", u.numel() * 5, ms, peak))
    del u


def _f4(out, dev, stream, g, peak, scale):
    """The pointwise family and equal over [8192, 32768] f32 with a broadcast row operand."""
    rows = max(8192 // scale, 1)
    g.manual_seed(8)
    a = torch.randn(rows, 32768, generator=g, device=dev)
    b = torch.randn(32768, generator=g, device=dev)
    c = torch.rand(rows, 32768, generator=g, device=dev) < 0.5
    n = a.numel()
    ms = _time(lambda: backend.pointwise("where", [c, a, b]), stream)
    out.append(_line("F4-where", "where(cond bool [8192,32768], a f32 [8192,32768], b f32 [32768])",
                     n * (1 + 4 + 4) + 32768 * 4, ms, peak))
    ms = _time(lambda: backend.pointwise("greater", [a, b]), stream)
    out.append(_line("F4-greater", "greater(a f32 [8192,32768], b f32 [32768]) -> bool", n * 5 + 32768 * 4, ms, peak))
    ms = _time(lambda: backend.binary("equal", a, b), stream)
    out.append(_line("F4-equal", "equal(a f32 [8192,32768], b f32 [32768]) -> f32", n * 8 + 32768 * 4, ms, peak))
    del a, b, c


def _f5(out, dev, stream, g, peak, scale):
    """int32 [8192, 32768] + f32 [32768] -> f32: promotion fused into the op, and as the reference's
    astype + add."""
    rows = max(8192 // scale, 1)
    g.manual_seed(9)
    a = torch.randint(-1000, 1001, (rows, 32768), generator=g, device=dev, dtype=torch.int32)
    b = torch.randn(32768, generator=g, device=dev)
    n = a.numel()
    ms = _time(lambda: backend.binary("add", a, b), stream)
    out.append(_line("F5-mixed-fused", "int32 [8192,32768] + f32 [32768] -> f32, promotion fused (mtxc_broadcast_binary_mixed)",
                     n * 8 + 32768 * 4, ms, peak))

    def unfused():
        af = backend.astype(a, torch.float32, make_contig=False)
        return backend.binary("add", af, b)

    ms = _time(unfused, stream)
    out.append(_line("F5-mixed-astype-then-add", "the same as the reference runs it: astype to f32, then add (2 kernels)",
                     n * 8 + 32768 * 4, ms, peak, moved_bytes=n * 16 + 32768 * 4))
    del a, b


def _f6(out, dev, stream, g, peak, scale):
    """The half-precision kernels at the configs' shapes: bf16 broadcast Add (C2), f16 Max and ArgMax over
    axis 1 (C3), bf16 full Sum of 2^31 elements."""
    g.manual_seed(10)
    b0 = max(256 // scale, 1)
    a = (torch.rand(b0, 1, 4096, generator=g, device=dev) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand(1, 512, 4096, generator=g, device=dev) * 2 - 1).to(torch.bfloat16)
    outb = torch.empty(b0, 512, 4096, dtype=torch.bfloat16, device=dev)
    meta = backend.binary_meta(list(a.shape), list(a.stride()), list(b.shape), list(b.stride()))
    ms = _time(lambda: backend.binary("add", a, b, out=outb, meta=meta), stream)
    out.append(_line("F6-bf16-add-C2", "broadcast Add bf16 a[256,1,4096] + b[1,512,4096]", outb.numel() * 2 +
                     (a.numel() + b.numel()) * 2, ms, peak))
    del a, b, outb
    c0 = max(64 // scale, 1)
    x = (torch.floor(torch.rand(c0, 8192, 1024, generator=g, device=dev) * 256) / 256).to(torch.float16)
    ms = _time(lambda: backend.reduce("max", x, 1), stream)
    out.append(_line("F6-f16-max-C3", "Max(axis=1) f16 [64,8192,1024]", x.numel() * 2 + c0 * 1024 * 2, ms, peak))
    ms = _time(lambda: backend.reduce("argmax", x, 1), stream)
    out.append(_line("F6-f16-argmax-C3", "ArgMax(axis=1) f16 [64,8192,1024]", x.numel() * 2 + c0 * 1024 * 4, ms, peak))
    del x
    y = torch.randn(8, (1 << 28) // scale, generator=g, device=dev).to(torch.bfloat16)
    ms = _time(lambda: backend.reduce("sum", y, 1), stream)
    out.append(_line("F6-bf16-sum", "Sum(axis=1) bf16 [8, 2^28] (4 GiB)", y.numel() * 2, ms, peak))
    del y


def _f7(out, dev, stream, g, peak, scale):
    """The packed (value, index) folds of the 1- and 2-byte integer types, 512 MiB of int8 or 1 GiB of
    int16 each (values 0..99): ArgMax over a strided axis at C3's layout (int8 first, so a profile that
    skips two column-kernel launches lands on it), int8 ArgMax over rows of 32,768, int16 ArgMax over a
    strided axis."""
    g.manual_seed(11)
    c0 = max(64 // scale, 1)
    x = torch.randint(0, 100, (c0, 8192, 1024), generator=g, device=dev, dtype=torch.int32).to(torch.int8)
    ms = _time(lambda: backend.reduce("argmax", x, 1), stream)
    out.append(_line("F7-i8-argmax-cols", "ArgMax(axis=1) int8 [64,8192,1024]", x.numel() + c0 * 1024 * 4, ms, peak))
    del x
    r0 = max(16384 // scale, 1)
    y = torch.randint(0, 100, (r0, 32768), generator=g, device=dev, dtype=torch.int32).to(torch.int8)
    ms = _time(lambda: backend.reduce("argmax", y, 1), stream)
    out.append(_line("F7-i8-argmax-rows", "ArgMax(axis=-1) int8 [16384,32768]", y.numel() + r0 * 4, ms, peak))
    del y
    z = torch.randint(0, 100, (c0, 8192, 1024), generator=g, device=dev, dtype=torch.int32).to(torch.int16)
    ms = _time(lambda: backend.reduce("argmax", z, 1), stream)
    out.append(_line("F7-i16-argmax-cols", "ArgMax(axis=1) int16 [64,8192,1024]", z.numel() * 2 + c0 * 1024 * 4, ms,
                     peak))
    del z


F8_DTYPES = [torch.float32, torch.float16, torch.bfloat16, torch.int32, torch.uint32, torch.int64, torch.uint64,
             torch.int16, torch.uint16, torch.int8, torch.uint8, torch.bool]


def _f8(out, dev, stream, g, peak, scale):
    """Every dtype at equal bytes (512 MiB inputs for the 1- to 4-byte types, 1 GiB for the 8-byte ones):
    broadcast Add a[64f,1,4096] + b[1,512,4096], Sum / Max / ArgMax over the last axis of [4096f, 32768], and
    Max / ArgMax / Sum over axis 1 of [16f, 8192, 1024], with f = 4 / element size for the narrow types (1
    otherwise); values 0..99, Bool 0 / 1."""
    g.manual_seed(12)
    for dt in F8_DTYPES:
        es = torch.tensor([], dtype=dt).element_size()
        f = max(1, 4 // es)
        name = str(dt).replace("torch.", "")

        def make(shape):
            if dt == torch.bool:
                return torch.randint(0, 2, shape, generator=g, device=dev, dtype=torch.int32).to(dt)
            return torch.randint(0, 100, shape, generator=g, device=dev, dtype=torch.int32).to(dt)

        a0 = max(64 * f // scale, 1)
        a, b = make((a0, 1, 4096)), make((1, 512, 4096))
        ob = torch.empty(a0, 512, 4096, dtype=dt, device=dev)
        meta = backend.binary_meta(list(a.shape), list(a.stride()), list(b.shape), list(b.stride()))
        ms = _time(lambda: backend.binary("add", a, b, out=ob, meta=meta), stream)
        out.append(_line(f"F8-{name}-add", f"broadcast Add {name} a[{a0},1,4096] + b[1,512,4096]",
                         (ob.numel() + a.numel() + b.numel()) * es, ms, peak))
        del a, b, ob
        r0 = max(4096 * f // scale, 1)
        x = make((r0, 32768))
        for op in ("sum", "max", "argmax"):
            m = backend.reduce_meta(list(x.shape), list(x.stride()), 1)
            o = backend.reduce(op, x, 1, meta=m)
            ms = _time(lambda: backend.reduce(op, x, 1, out=o, meta=m), stream)
            out.append(_line(f"F8-{name}-{op}-rows", f"{op}(axis=-1) {name} [{r0},32768]",
                             x.numel() * es + o.numel() * o.element_size(), ms, peak))
        del x
        c0 = max(16 * f // scale, 1)
        x = make((c0, 8192, 1024))
        for op in ("max", "argmax", "sum"):
            m = backend.reduce_meta(list(x.shape), list(x.stride()), 1)
            o = backend.reduce(op, x, 1, meta=m)
            ms = _time(lambda: backend.reduce(op, x, 1, out=o, meta=m), stream)
            out.append(_line(f"F8-{name}-{op}-cols", f"{op}(axis=1) {name} [{c0},8192,1024]",
                             x.numel() * es + o.numel() * o.element_size(), ms, peak))
        del x
