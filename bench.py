"""Benchmark of the tensor.cx hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (BASELINE.json metric, configs[1] at its largest size): float32 matmul
C = A @ B at M = N = K = 8192, A, B ~ U(-1, 1) (seeded per rank), in TFLOP/s
(2*M*N*K flops per step, whole job). A step is one tcx_sm100_matmul call: the
3xTF32 split pre-pass plus the tcgen05 GEMM. Inputs (256 MiB each) exceed the
126 MB L2, so no flush is needed between steps.

N > 1 (torchrun, one rank per GPU, NCCL): every rank multiplies its own 8192^3 pair
(weak scaling, no communication); the timed region is bracketed by barrier +
synchronize, and the time is the max over ranks.

Also measured in the same run, device-resident, and reported under "workloads"
(each with its own roofline fraction): row softmax / rmsnorm / layernorm on
[16384, 4096] (rows sharded over ranks) and softmax on [4096, 32768]; full
reductions over 2^28 float32 (sum, argmax) and int32 (sum), sharded over ranks and
combined by an NCCL all-gather of 16-byte partial records; batched matmul
[64, 2048, 2048]^2 with the fused bias + SiLU epilogue, batch sharded over ranks.

`--impl reference` times the reference's own CPU matmul (cpu::matmul, compiled from
the tensor.cx sources into oracle/_ref) on row slices of the same 8192^3 product,
on all host threads, rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
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
sys.path.insert(0, ROOT)

SIZE = 8192
METRIC = "fp32 matmul TFLOP/s (M=N=K=8192)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--size", type=int, default=SIZE)
    p.add_argument("--no-workloads", action="store_true", help="headline only")
    # --case: one workload alone on cuda:0, for profilers (ncu) and quick timing
    p.add_argument("--case", default=None,
                   help="matmul | bmm | softmax | rmsnorm | layernorm | sum | max | min | argmax | mean | "
                        "sum_axis0 | sum_axes02 | attention")
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--rows", type=int, default=16384)
    p.add_argument("--cols", type=int, default=4096)
    p.add_argument("--n", type=int, default=1 << 28)
    p.add_argument("--int32", action="store_true")
    p.add_argument("--path", default="auto")
    p.add_argument("--repeat", type=int, default=3)
    p.add_argument("--causal", action="store_true")
    p.add_argument("--kernels", action="store_true", help="with --case: device time per kernel as well")
    return p.parse_args()


def run_case(a):
    """One hot-path workload called `--repeat` times on cuda:0 after one untimed call;
    prints the mean device time per call (CUDA events on the current stream).

        python bench.py --case matmul --size 4096 [--path tensor|ffma] [--repeat 3] [--kernels]
        python bench.py --case bmm --batch 64 --size 2048
        python bench.py --case softmax|rmsnorm|layernorm --rows 16384 --cols 4096
        python bench.py --case sum|max|min|argmax|mean --n 268435456 [--int32]
        python bench.py --case attention --batch 32 --rows 2048 --cols 2048 --size 128 [--causal]
        python bench.py --case sum_axis0 --rows 65536 --cols 4096
        python bench.py --case sum_axes02 --batch 64 --rows 4096 --cols 1024
        python bench.py --case randn|rand --n 268435456
    """
    import torch
    from tensorcx_b200 import ops
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    w = a.case
    if w == "matmul":
        x = torch.rand(a.size, a.size, device="cuda", generator=g) * 2 - 1
        y = torch.rand(a.size, a.size, device="cuda", generator=g) * 2 - 1
        fn = lambda: ops.matmul(x, y, path=a.path)  # noqa: E731
    elif w == "bmm":
        x = torch.rand(a.batch, a.size, a.size, device="cuda", generator=g) * 2 - 1
        y = torch.rand(a.batch, a.size, a.size, device="cuda", generator=g) * 2 - 1
        bias = torch.randn(a.size, device="cuda", generator=g)
        fn = lambda: ops.matmul(x, y, bias=bias, act="silu", path=a.path)  # noqa: E731
    elif w in ("softmax", "rmsnorm", "layernorm"):
        x = torch.randn(a.rows, a.cols, device="cuda", generator=g) * 3
        f = getattr(ops, w)
        fn = lambda: f(x, axis=-1)  # noqa: E731
    elif w in ("sum", "max", "min", "argmax", "mean"):
        if a.int32:
            x = torch.randint(-1000, 1001, (a.n,), device="cuda", generator=g, dtype=torch.int32)
        else:
            x = torch.randn(a.n, device="cuda", generator=g)
        f = getattr(ops, w)
        fn = lambda: f(x)  # noqa: E731
    elif w == "sum_axis0":
        x = torch.randn(a.rows, a.cols, device="cuda", generator=g)
        fn = lambda: ops.sum(x, axis=0)  # noqa: E731
    elif w == "sum_axes02":
        x = torch.randn(a.batch, a.rows, a.cols, device="cuda", generator=g)
        fn = lambda: ops.sum(x, axis=(0, 2))  # noqa: E731
    elif w in ("randn", "rand"):
        gen = ops.randn if w == "randn" else ops.rand_uniform
        fn = lambda: gen((a.n,), seed=2024)  # noqa: E731
    elif w == "attention":  # batch = heads, rows = queries, cols = keys, size = features
        q = torch.randn(a.batch, a.rows, a.size, device="cuda", generator=g)
        k = torch.randn(a.batch, a.cols, a.size, device="cuda", generator=g)
        v = torch.randn(a.batch, a.cols, a.size, device="cuda", generator=g)
        fn = lambda: ops.attention(q, k, v, is_causal=a.causal)  # noqa: E731
    else:
        raise SystemExit(f"unknown workload {w}")
    fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.repeat):
        fn()
    e.record()
    torch.cuda.synchronize()
    print(f"{w}: {s.elapsed_time(e) / a.repeat:.4f} ms per call")
    if a.kernels:  # device time per kernel, the calls queued behind a device spin
        from tensorcx_b200 import _abi
        lib = _abi.lib()
        step = queued(torch, fn)
        hooks_on(lib)
        for _ in range(a.repeat):
            step()
        torch.cuda.synchronize()
        lib.tcx_sm100_timer_enable(0)
        for name, (count, total) in read_timer(lib).items():
            print(f"  {name}: {count} launches, {total / max(count, 1) * 1e3:.2f} us per launch")


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# ------------------------------------------------------------------ CPU legs
# Rows of the size^3 product each host thread computes per CPU step: the same sample
# in the reference arm and in the GPU arm's cpu_baseline leg, so the two agree.
CPU_ROWS_PER_THREAD = 2


def cpu_matmul_rate(size: int, threads: int, rows_per_thread: int, a, b, ref=None):
    """Reference cpu::matmul on `threads` disjoint row slices of the size^3 product
    (identical per-element arithmetic to the full product), B bound once beforehand
    (Reference.matmul_bind_rhs) so a step is the rows' arithmetic alone. Returns
    (flops/s, rows, seconds, rows of C)."""
    from oracle.oracle import Reference
    ref = ref or Reference()
    outs = [None] * threads

    def work(t):
        r0 = t * rows_per_thread
        outs[t] = ref.matmul_rows(a, b, r0, r0 + rows_per_thread)

    t0 = time.perf_counter()
    pool = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
    for th in pool:
        th.start()
    for th in pool:
        th.join()
    dt = time.perf_counter() - t0
    rows = threads * rows_per_thread
    return 2.0 * rows * size * size / dt, rows, dt, np.concatenate(outs)


def cpu_sample_text(size, threads, rows_per_thread):
    return (f"cpu::matmul (reference sources, -O3) on {threads * rows_per_thread} disjoint rows of the {size}^3 "
            f"product per step ({rows_per_thread} per thread, {threads} threads), B bound once outside the timing")


def headline_config(size, world):
    return {"workload": f"fp32 matmul M=N=K={size} (BASELINE configs[1], largest size)",
            "per_gpu": f"{size}^3", "parallelism": f"independent products, {world} GPU(s)",
            "l2": "inputs (256 MiB each) larger than the 126 MB L2; no flush"}


def host_threads() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return os.cpu_count() or 1


def reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle.oracle import Reference
    if not Reference.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libtcx_ref.so was not built"}))
        return
    threads = host_threads()
    size = args.size
    per = CPU_ROWS_PER_THREAD
    rng = np.random.default_rng(0)
    a = rng.random((threads * per, size), dtype=np.float32) * 2 - 1
    b = rng.random((size, size), dtype=np.float32) * 2 - 1
    ref = Reference()
    ref.matmul_bind_rhs(b)
    for _ in range(args.warmup):
        cpu_matmul_rate(size, threads, per, a, b, ref)
    times = []
    for _ in range(args.steps):
        _, _, dt, _ = cpu_matmul_rate(size, threads, per, a, b, ref)
        times.append(dt)
    mean_dt = sum(times) / len(times)
    value = 2.0 * threads * per * size * size / mean_dt / 1e12
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean_dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": headline_config(size, args.gpus),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "reference",
                         "sample": cpu_sample_text(size, threads, per)},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (every 50 ms) of SM clock and throttle reasons."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines = []
        self.windows = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu=timestamp,{self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self, t0, t1):
        self.windows.append((t0, t1))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        for ts, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            inside = any(a - 0.05 <= ts <= b + 0.05 for a, b in self.windows)
            rows.append((inside, parts))
        use = [p for inside, p in rows if inside] or [p for _, p in rows]
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(p[2]) for p in use if p[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for p in use for i in range(4) if "Active" in p[6 + i] and "Not" not in p[6 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(use[0][3]) if use[0][3].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(use),
                "power_w_max": max((float(p[4]) for p in use if p[4].replace(".", "").isdigit()), default=None)}


def smi_index(torch, local):
    """nvidia-smi's index of CUDA device `local`, matched by UUID (CUDA's enumeration
    order and CUDA_VISIBLE_DEVICES need not follow nvidia-smi's); falls back to the
    CUDA_VISIBLE_DEVICES entry, then to the CUDA index."""
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
        r = subprocess.run(["nvidia-smi", "-i", uuid, "--query-gpu=index", "--format=csv,noheader"],
                           capture_output=True, text=True, timeout=20)
        if r.returncode == 0 and r.stdout.strip().isdigit():
            return r.stdout.strip()
    except (OSError, subprocess.SubprocessError, RuntimeError):
        pass
    visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    return visible[local] if local < len(visible) else str(local)


# ------------------------------------------------------------------ GPU arm
class Timer:
    """CUDA-event timing on the current stream, max over ranks."""

    def __init__(self, torch, dist, world):
        self.torch, self.dist, self.world = torch, dist, world

    # idle time before each workload's warm-up: a workload measured right after a
    # power-capped one (the GEMMs draw the 1 kW limit) otherwise starts at the lowered SM
    # clock the power limiter is still holding (measured: the fused attention kernel 0.22
    # -> 0.30 ms right after the bmm, back to 0.22 ms after 3 s idle). The warm-up comes
    # after the pause: a timed region that starts straight out of an idle pause is slow
    # too (measured: softmax [16384, 4096] 84 -> 96 us, 2048^3 matmul 83 -> 88-98 us;
    # three warm-up calls restore 84 / 83 us).
    rest_s = 0.5

    def run(self, step, steps, warmup, sampler=None, before_timing=None):
        torch = self.torch
        torch.cuda.synchronize()
        time.sleep(self.rest_s)
        for _ in range(max(warmup, 3)):
            step()
        self.barrier()
        torch.cuda.synchronize()
        if before_timing:
            before_timing()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.time()
        start.record()
        for _ in range(steps):
            step()
        end.record()
        torch.cuda.synchronize()
        t1 = time.time()
        self.barrier()
        if sampler:
            sampler.mark(t0, t1)
        ms = start.elapsed_time(end)
        return self.max_over_ranks(ms)

    def run_hbm(self, step, steps, warmup, sampler, working_bytes, before_timing=None):
        """Timing of an HBM-bound step: back to back (`run`) when the step's data is at
        least twice L2, so every step streams from HBM and pays the write-back of the
        previous step's output (the steady state); otherwise `run_flushed`."""
        l2 = self.torch.cuda.get_device_properties(self.torch.cuda.current_device()).L2_cache_size
        if working_bytes >= 2 * l2:
            return self.run(step, steps, warmup, sampler, before_timing)
        return self.run_flushed(step, steps, warmup, sampler, before_timing)

    def run_flushed(self, step, steps, warmup, sampler=None, before_timing=None):
        """Device time of `steps` calls of `step` with L2 emptied before each: a 256 MiB
        memset then a read of a second 256 MiB buffer (L2 ends up holding clean lines of
        the flush, so the step neither hits its own data nor pays the flush's
        write-back; the flush also keeps the GPU busy while the host enqueues the step).
        Each step has its own CUDA event pair; the step times are summed, max over ranks."""
        torch = self.torch
        if getattr(self, "flush", None) is None:
            self.flush = (torch.empty(256 << 20, dtype=torch.uint8, device="cuda"),
                          torch.ones(64 << 20, dtype=torch.float32, device="cuda"))
        torch.cuda.synchronize()
        time.sleep(self.rest_s)
        for _ in range(max(warmup, 3)):
            step()
        self.barrier()
        torch.cuda.synchronize()
        if before_timing:
            before_timing()
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        t0 = time.time()
        for start, end in events:
            self.flush[0].zero_()
            self.flush_sink = self.flush[1].sum()
            start.record()
            step()
            end.record()
        torch.cuda.synchronize()
        t1 = time.time()
        self.barrier()
        if sampler:
            sampler.mark(t0, t1)
        return self.max_over_ranks(sum(start.elapsed_time(end) for start, end in events))

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, value):
        if self.world == 1:
            return value
        t = self.torch.tensor([value], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())


def read_timer(lib):
    names = ctypes.create_string_buffer(64 * 64)
    launches = (ctypes.c_int64 * 64)()
    total = (ctypes.c_double * 64)()
    n = ctypes.c_int32(0)
    lib.tcx_sm100_timer_read(names, len(names), launches, total, 64, ctypes.byref(n))
    out = {}
    raw = names.raw.split(b"\0")
    for i in range(n.value):
        out[raw[i].decode()] = (int(launches[i]), float(total[i]))
    return out


def hooks_on(lib):
    """Clears the per-kernel device timing records and turns the hooks on (called right
    before a timed region, after its warm-up)."""
    read_timer(lib)
    lib.tcx_sm100_timer_enable(1)


# ~0.1 ms of device spin at the B200's clocks
SPIN_CYCLES = 200_000


def queued(torch, step):
    """`step` behind a short device spin on the current stream. The timing hooks record an
    event before and after each launch; on an idle GPU the start event completes at once
    and the pair then also spans the host's own launch of the kernel (a few microseconds,
    the whole duration of a small product's kernels). Behind the spin the host enqueues
    the step's events and launches while the GPU is still busy, so each pair brackets the
    kernel's device time."""
    def run():
        torch.cuda._sleep(SPIN_CYCLES)
        step()
    return run


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "of measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "of fallback"


# The bench's one JSON line goes to the process's original stdout; everything else that
# writes to file descriptor 1 during the run (NCCL's version banner at communicator
# creation, library messages) is sent to stderr, so stdout holds exactly that line.
JSON_FD = 1


def quiet_stdout():
    global JSON_FD
    sys.stdout.flush()
    JSON_FD = os.dup(1)
    os.dup2(2, 1)


def gpu_arm(args):
    quiet_stdout()
    import torch
    import torch.distributed as dist
    from tensorcx_b200 import _abi, ops

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    lib = _abi.lib()
    assert lib.tcx_sm100_device_supported(local) == 0, lib.tcx_sm100_last_error()
    timer = Timer(torch, dist, world)
    pk, pk_note = peaks()
    hbm_peak = float(pk["hbm_gbs"])
    sampler = ClockSampler(smi_index(torch, local))
    sampler.start()
    size = args.size
    flops = 2.0 * size ** 3

    # cuBLAS TF32 rate on this GPU now: the denominator of the 3xTF32 roofline
    torch.backends.cuda.matmul.allow_tf32 = True
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    ta = torch.rand(size, size, device="cuda", generator=g)
    tb = torch.rand(size, size, device="cuda", generator=g)
    tf32_ms = timer.run(lambda: torch.matmul(ta, tb), 10, 3)
    tf32_tflops = flops * 10 / (tf32_ms * 1e-3) / 1e12
    torch.backends.cuda.matmul.allow_tf32 = False
    sgemm_ms = timer.run(lambda: torch.matmul(ta, tb), 3, 1)
    sgemm_tflops = flops * 3 / (sgemm_ms * 1e-3) / 1e12
    del ta, tb
    torch.cuda.empty_cache()

    # headline inputs (host-generated, seeded per rank, then resident in HBM)
    rng = np.random.default_rng(rank)
    a_host = torch.from_numpy(rng.random((size, size), dtype=np.float32) * 2 - 1).pin_memory()
    b_host = torch.from_numpy(rng.random((size, size), dtype=np.float32) * 2 - 1).pin_memory()
    c_host = torch.empty((size, size), dtype=torch.float32).pin_memory()
    a = a_host.cuda()
    b = b_host.cuda()
    c = torch.empty((size, size), dtype=torch.float32, device="cuda")
    ws_bytes = lib.tcx_sm100_matmul_workspace_bytes(size, size, size, 1, 1, 0)
    ws_buf = torch.empty(ws_bytes + 1024, dtype=torch.uint8, device="cuda")
    ws = ctypes.c_void_p((ws_buf.data_ptr() + 1023) // 1024 * 1024)
    one = _abi.i64_array([])

    def step():
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        _abi.check(lib.tcx_sm100_matmul(s, ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                                        ctypes.c_void_p(c.data_ptr()), size, size, size, 1, one, one, one, 0,
                                        None, 0, 0, ws, ws_bytes))

    step()
    torch.cuda.synchronize()

    # the per-kernel device timing covers the timed steps only
    ms = timer.run(step, args.steps, args.warmup, sampler, before_timing=lambda: hooks_on(lib))
    lib.tcx_sm100_timer_enable(0)
    kernels = read_timer(lib)
    ms_per_step = ms / args.steps
    value = world * flops / (ms_per_step * 1e-3) / 1e12
    gemm_launches, gemm_ms = kernels.get("gemm_tf32x3", (0, 0.0))
    gemm_avg_ms = gemm_ms / max(gemm_launches, 1)
    gemm_avg_ms = timer.max_over_ranks(gemm_avg_ms)
    achieved = flops / (gemm_avg_ms * 1e-3) / 1e12
    peak_3x = tf32_tflops / 3.0
    launches = sum(v[0] for v in kernels.values())

    # e2e: pinned host buffers in, host result out, through the C ABI's host-buffer
    # matmul (uploads, 3xTF32 GEMMs and downloads pipelined in row chunks)
    e2e_ws_bytes = lib.tcx_sm100_matmul_host_workspace_bytes(size, size, size)
    del ws_buf
    torch.cuda.empty_cache()
    e2e_buf = torch.empty(e2e_ws_bytes + 1024, dtype=torch.uint8, device="cuda")
    e2e_ws = ctypes.c_void_p((e2e_buf.data_ptr() + 1023) // 1024 * 1024)
    torch.cuda.synchronize()

    # the transfer floor of one step: A and B uploaded over PCIe from page-locked memory
    # while C comes back on another stream (full duplex; the download slows the uploads)
    up = e2e_buf[:3 * size * size * 4].view(torch.float32)
    s_up, s_down = torch.cuda.Stream(), torch.cuda.Stream()
    h2d_s = duplex_s = float("inf")
    for duplex in (False, True):
        for _ in range(3):
            torch.cuda.synchronize()
            t1 = time.perf_counter()
            with torch.cuda.stream(s_up):
                up[:size * size].copy_(a_host.view(-1), non_blocking=True)
                up[size * size:2 * size * size].copy_(b_host.view(-1), non_blocking=True)
            if duplex:
                with torch.cuda.stream(s_down):
                    c_host.view(-1).copy_(up[2 * size * size:], non_blocking=True)
            torch.cuda.synchronize()
            dt = time.perf_counter() - t1
            if duplex:
                duplex_s = min(duplex_s, dt)
            else:
                h2d_s = min(h2d_s, dt)
    h2d_gbs = 2 * size * size * 4 / h2d_s / 1e9
    del up

    def e2e_step():
        _abi.check(lib.tcx_sm100_matmul_host(ctypes.c_void_p(a_host.data_ptr()), ctypes.c_void_p(b_host.data_ptr()),
                                             ctypes.c_void_p(c_host.data_ptr()), size, size, size, e2e_ws,
                                             e2e_ws_bytes))

    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(2):
        e2e_step()
    timer.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()  # synchronous: returns with C in host memory
    e2e_ms = timer.max_over_ranks((time.perf_counter() - t0) * 1e3 / e2e_steps)
    e2e_value = world * flops / (e2e_ms * 1e-3) / 1e12
    del e2e_buf

    # CPU baseline (rank 0, N = 1): the reference's cpu::matmul on the reference arm's
    # row sample (CPU_ROWS_PER_THREAD rows per host thread), one warm-up step, mean of 3
    cpu = None
    if rank == 0 and world == 1:
        from oracle.oracle import Reference
        if Reference.available():
            threads = host_threads()
            per = CPU_ROWS_PER_THREAD
            a_np = a_host.numpy()
            b_np = b_host.numpy()
            ref = Reference()
            ref.matmul_bind_rhs(b_np)
            cpu_matmul_rate(size, threads, per, a_np, b_np, ref)
            dts = []
            for _ in range(3):
                _, rows, dt, got_rows = cpu_matmul_rate(size, threads, per, a_np, b_np, ref)
                dts.append(dt)
            dt = sum(dts) / len(dts)
            gpu_rows = c_host[:rows].numpy()  # C of the last e2e step (same A, B)
            rel = float(np.linalg.norm(gpu_rows.astype(np.float64) - got_rows) / np.linalg.norm(got_rows))
            cpu = {"value": 2.0 * rows * size * size / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
                   "kind": "reference",
                   "sample": cpu_sample_text(size, threads, per) + f", mean of 3 steps ({dt:.2f} s each)",
                   "gpu_rows_rel_frobenius_error": rel,
                   "tolerance": 1e-4 * math.sqrt(size / 1024)}
    del a_host, b_host, c_host

    workloads = {} if args.no_workloads else secondary(args, torch, dist, lib, ops, timer, world, rank,
                                                       hbm_peak, peak_3x, sampler)
    del a, b, c
    sampler.stop()
    clocks = sampler.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (3xTF32 split on tf32 tensor cores, f32 accumulate)",
            "data": "synthetic (seeded U(-1,1), per-rank seed)",
            "config": headline_config(size, world),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_3x, "unit": "TFLOP/s",
                         "frac": achieved / peak_3x,
                         # DRAM bytes read + written by one gemm_tf32x3 launch (raw mode) at
                         # 8192^3: dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture
                         "traffic": 8685800960 if size == 8192 else None,
                         "traffic_unit": "B per launch",
                         "kernel": "gemm_tf32x3 (tcgen05.mma kind::tf32 x3 per k-step)",
                         "kernel_ms": gemm_avg_ms,
                         "peak_note": f"cuBLAS TF32 GEMM {size}^3 measured in this run = {tf32_tflops:.1f} TFLOP/s, "
                                      f"/3 for 3xTF32 (MEASURED_PEAKS bf16 {pk.get('bf16_tflops')} TFLOP/s "
                                      f"{pk_note}; bf16/6 = {float(pk.get('bf16_tflops', 0)) / 6:.1f})"},
            "context": {"cublas_tf32_tflops": tf32_tflops, "cublas_fp32_sgemm_tflops": sgemm_tflops,
                        "split_prepass_ms": sum(kernels.get(name, (0, 0.0))[1] for name in ("split_lo", "split_pair"))
                        / max(args.steps, 1)},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": 2 * size * size * 4,
                    "d2h_bytes_per_step": size * size * 4, "ms_per_step": e2e_ms,
                    "api": "tcx_sm100_matmul_host (pinned host A, B in; C out; synchronous)",
                    "pcie_h2d_gbs": h2d_gbs, "upload_floor_ms": h2d_s * 1e3,
                    "transfer_floor_ms": duplex_s * 1e3,
                    "frac_of_transfer_floor": duplex_s * 1e3 / e2e_ms},
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "kernels_in_timed_region": {k: {"launches": v[0], "total_ms": v[1]} for k, v in kernels.items()},
            "clocks": clocks,
            "workloads": workloads,
            "strong_scaling": {k: v["strong_scaling"]["efficiency_vs_n1"] for k, v in workloads.items()
                               if isinstance(v, dict) and "strong_scaling" in v} or None,
        }
        os.write(JSON_FD, (json.dumps(line) + "\n").encode())
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def secondary(args, torch, dist, lib, ops, timer, world, rank, hbm_peak, peak_3x, sampler):
    """The other hot-path workloads of BASELINE configs[2..4], device-resident."""
    from tensorcx_b200 import _abi
    out = {}
    steps = max(5, args.steps)
    g = torch.Generator(device="cuda").manual_seed(77 + rank)

    def hbm_entry(name, bytes_per_step, ms_step, kernel, kernels, extra=None):
        if kernel not in kernels and kernels:  # the width decides which row kernel runs
            kernel = max(kernels, key=lambda k: kernels[k][1])
        k_launches, k_ms = kernels.get(kernel, (0, 0.0))
        k_avg = timer.max_over_ranks(k_ms / max(k_launches, 1))
        achieved = bytes_per_step / (k_avg * 1e-3) / 1e9 if k_avg else None
        d = {"value": world * bytes_per_step / (ms_step * 1e-3) / 1e9, "unit": "GB/s",
             "ms_per_step": ms_step,
             "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                          "frac": achieved / hbm_peak if achieved else None, "kernel": kernel,
                          "kernel_ms": k_avg}}
        if extra:
            d.update(extra)
        out[name] = d

    def measure_hbm(st, working_bytes):
        """(ms per step, per-kernel times): the step time with the library's timing hooks
        off (their events between launches would block the programmatic-launch overlap
        of back-to-back kernels), then the per-kernel times from a shorter pass with the
        hooks on."""
        ms_ = timer.run_hbm(st, steps, 2, sampler, working_bytes) / steps
        timer.run_hbm(st, max(3, steps // 2), 1, None, working_bytes, before_timing=lambda: hooks_on(lib))
        lib.tcx_sm100_timer_enable(0)
        return ms_, read_timer(lib)

    # Strong scaling (N > 1): the same whole workload timed on rank 0's GPU alone in
    # this run (the other ranks wait at a barrier), so each sharded workload carries its
    # own speedup and efficiency against one GPU on the same box.
    solo = Timer(torch, dist, 1)
    gs = torch.Generator(device="cuda").manual_seed(4242)

    def strong(name, solo_value):
        if world == 1:
            return
        v1 = solo_value() if rank == 0 else None
        timer.barrier()
        if rank == 0 and v1:
            vn = out[name]["value"]
            out[name]["strong_scaling"] = {
                "n1_value": v1, "speedup_vs_n1": vn / v1, "efficiency_vs_n1": vn / (world * v1),
                "n1_measured": "the whole workload on rank 0's GPU alone, same run, same timing rule"}
        torch.cuda.empty_cache()

    # row ops, [16384, 4096] and [4096, 32768]: rows sharded over ranks
    for name, (rows, cols), op in [("softmax_16384x4096", (16384, 4096), "softmax"),
                                   ("rmsnorm_16384x4096", (16384, 4096), "rmsnorm"),
                                   ("layernorm_16384x4096", (16384, 4096), "layernorm"),
                                   ("softmax_4096x32768", (4096, 32768), "softmax")]:
        r = rows // world
        x = torch.randn(r, cols, device="cuda", generator=g) * 3
        y = torch.empty_like(x)
        fn = getattr(ops, op)
        kw = {} if op == "softmax" else {"eps": 1e-5}

        def st(x=x, fn=fn, kw=kw):
            return fn(x, axis=-1, **kw)
        st()
        ms, kern = measure_hbm(st, 8 * r * cols)
        hbm_entry(name, 8.0 * r * cols, ms, "row_kernel", kern,
                  {"config": f"[{rows},{cols}] float32, rows sharded {world} way(s), 8 B/element; "
                            "back to back when the data is >= 2x L2, else L2 flushed before each step"})
        del x, y

        def solo_rows(rows=rows, cols=cols, fn=fn, kw=kw):
            xs = torch.randn(rows, cols, device="cuda", generator=gs) * 3
            ms1 = solo.run_hbm(lambda: fn(xs, axis=-1, **kw), steps, 2, None, 8 * rows * cols) / steps
            return 8.0 * rows * cols / (ms1 * 1e-3) / 1e9
        strong(name, solo_rows)

    # full reductions over 2^28 elements: shard + per-rank record + NCCL all-gather
    from tensorcx_b200 import shard as sharding
    total = 1 << 28
    base, stop = sharding.shard_range(total, rank, world)
    shard = stop - base
    xf = torch.randn(shard, device="cuda", generator=g)
    xi = torch.randint(-1000, 1001, (shard,), device="cuda", generator=g, dtype=torch.int32)
    gathered = torch.empty((world, 16), dtype=torch.uint8, device="cuda")
    # N > 1: the records cross GPUs inside the reduction kernel (peer-memory mailboxes,
    # tensorcx_b200.collective); NCCL all_gather of the records only without peer access
    peer = None
    here = torch.cuda.current_device()
    if world > 1 and all(torch.cuda.can_device_access_peer(here, d)
                         for d in range(torch.cuda.device_count()) if d != here):
        from tensorcx_b200.collective import PeerReduction
        peer = PeerReduction()
    combine = ("in the reduction kernel over NVLink peer memory" if peer else
               "by NCCL all_gather + the combine kernel" if world > 1 else "by the combine kernel")
    for name, x, op in [("sum_f32_2^28", xf, "sum"), ("mean_f32_2^28", xf, "mean"), ("max_f32_2^28", xf, "max"),
                        ("min_f32_2^28", xf, "min"), ("argmax_f32_2^28", xf, "argmax"),
                        ("sum_i32_2^28", xi, "sum"), ("max_i32_2^28", xi, "max")]:
        def st(x=x, op=op):
            if peer is not None:
                return peer.reduce(x, op, base, total)
            rec = ops.reduce_partial(x, op, index_base=base)
            if world > 1:
                dist.all_gather_into_tensor(gathered, rec)
                recs = gathered
            else:
                recs = rec.view(1, 16)
            return ops.reduce_combine(recs, op, x.dtype, total)
        st()
        ms, kern = measure_hbm(st, 4 * shard)
        stage1 = kern.get("reduce_stage1", (0, 0.0))
        fold = kern.get("reduce_exchange", kern.get("reduce_combine", (0, 0.0)))
        hbm_entry(name, 4.0 * shard, ms, "reduce_stage1", kern,
                  {"config": f"2^28 elements total, {world} shard(s), partials combined {combine} "
                             "in rank order; back to back when the data is >= 2x L2, else L2 flushed before each step",
                   "split_ms": {"stage1": timer.max_over_ranks(stage1[1] / max(stage1[0], 1)),
                                "exchange" if world > 1 and peer is not None else "combine":
                                    timer.max_over_ranks(fold[1] / max(fold[0], 1)),
                                "note": "per call, max over ranks; the exchange includes the wait for the "
                                        "slowest peer's record"}})

        def solo_reduce(x=x, op=op):
            full = (torch.randn(total, device="cuda", generator=gs) if x.dtype == torch.float32 else
                    torch.randint(-1000, 1001, (total,), device="cuda", generator=gs, dtype=torch.int32))

            def one():
                rec = ops.reduce_partial(full, op, index_base=0)
                return ops.reduce_combine(rec.view(1, 16), op, full.dtype, total)
            ms1 = solo.run_hbm(one, steps, 2, None, 4 * total) / steps
            return 4.0 * total / (ms1 * 1e-3) / 1e9
        strong(name, solo_reduce)
    if peer is not None:
        peer.close()
    if world == 1:
        # which side of the float32 sum bar holds at 2^28: relative error of the CPU's
        # sequential sum and of the GPU's tree against the float64 sum of the same data
        from oracle.oracle import Oracle
        o = Oracle()
        host = xf.cpu().numpy()
        exact = o.sum_f64(host)
        cpu_sum = float(o.sum(host))
        gpu_sum = float(ops.reduce_combine(ops.reduce_partial(xf, "sum", index_base=0).view(1, 16), "sum",
                                           xf.dtype, total).item())
        out["sum_f32_2^28"]["error_vs_float64"] = {
            "gpu_rel": abs(gpu_sum - exact) / abs(exact), "cpu_reference_rel": abs(cpu_sum - exact) / abs(exact),
            "gpu_vs_cpu_rel": abs(gpu_sum - cpu_sum) / abs(cpu_sum),
            "bar": "within 1e-5 of the CPU result, or closer to the float64 sum than the CPU"}
        del host
    del xf, xi

    # device-side seeded generation of 2^28 standard normals (each rank its slice of one
    # stream, at its global offset): HBM-bound, 4 B written per element
    gen_n = total // world
    gen_out = torch.empty(gen_n, device="cuda")

    def st_gen():
        _abi.check(lib.tcx_sm100_random(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), 0,
                                        ctypes.c_void_p(gen_out.data_ptr()), gen_n, 2024, rank * gen_n, 0.0, 1.0))
    st_gen()
    ms, kern = measure_hbm(st_gen, 4 * gen_n)
    hbm_entry("randn_2^28", 4.0 * gen_n, ms, "random", kern,
              {"config": f"2^28 float32 N(0,1) from the Philox4x32-10 stream of one seed, {world} slice(s) at "
                         "their global offsets, 4 B written per element"})
    del gen_out

    def solo_gen():
        full = torch.empty(total, device="cuda")

        def one():
            _abi.check(lib.tcx_sm100_random(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), 0,
                                            ctypes.c_void_p(full.data_ptr()), total, 2024, 0, 0.0, 1.0))
        ms1 = solo.run_hbm(one, steps, 2, None, 4 * total) / steps
        return 4.0 * total / (ms1 * 1e-3) / 1e9
    strong("randn_2^28", solo_gen)

    # strided and multi-axis reductions (1 GiB each): axis 0 of [65536, 4096], and
    # axes (0, 2) of [64, 4096, 1024]; outer rows sharded
    for name, shape, axis in [("sum_axis0_65536x4096", (65536 // world, 4096), 0),
                              ("sum_axes02_64x4096x1024", (64 // world, 4096, 1024), (0, 2))]:
        x = torch.randn(*shape, device="cuda", generator=g)

        def st(x=x, axis=axis):
            return ops.sum(x, axis=axis)
        st()
        ms, kern = measure_hbm(st, 4 * x.numel())
        hbm_entry(name, 4.0 * x.numel(), ms, "axis_chunks" if axis == 0 else "axes_chunks", kern,
                  {"config": f"float32 {list(shape)} sum over axis {axis} per rank (leading axis sharded "
                             f"{world} way(s)), 4 B/element; partials per rank are not combined across ranks; "
                             "back to back when the data is >= 2x L2, else L2 flushed before each step"})
        del x

    # host <-> device transfers of 1 GiB pageable host memory (from_cpu / to_cpu): the
    # pinned two-slot staging of tcx_sm100_copy_to_* against the driver's pageable path
    import numpy as np
    nbytes = 1 << 30
    host_buf = np.ones(nbytes // 4, np.float32)
    back_buf = np.empty_like(host_buf)
    dev_buf = torch.empty(nbytes // 4, device="cuda")
    cs = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    hp, bp, dp = (ctypes.c_void_p(host_buf.ctypes.data), ctypes.c_void_p(back_buf.ctypes.data),
                  ctypes.c_void_p(dev_buf.data_ptr()))

    def wall(fn, reps=3):
        fn()
        best = float("inf")
        for _ in range(reps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            fn()
            torch.cuda.synchronize()
            best = min(best, time.perf_counter() - t0)
        return nbytes / best / 1e9
    host_t, back_t = torch.from_numpy(host_buf), torch.from_numpy(back_buf)
    out["transfer_pageable_1GiB"] = {
        "value": wall(lambda: lib.tcx_sm100_copy_to_device(cs, dp, hp, nbytes)), "unit": "GB/s",
        "d2h_gbs": wall(lambda: lib.tcx_sm100_copy_to_host(cs, bp, dp, nbytes)),
        "driver_pageable_h2d_gbs": wall(lambda: dev_buf.copy_(host_t)),
        "driver_pageable_d2h_gbs": wall(lambda: back_t.copy_(dev_buf)),
        "config": "1 GiB pageable numpy buffer <-> device, synchronous, wall clock (best of 3); value = "
                  "host-to-device through tcx_sm100_copy_to_device"}
    del host_buf, back_buf, dev_buf, host_t, back_t

    # the rest of the square matmul sweep (512 ... 4096; 8192 is
    # the headline): per-rank replicas, device-resident, pre-pass included
    for size in (512, 1024, 2048, 4096):
        a = torch.rand(size, size, device="cuda", generator=g) * 2 - 1
        b = torch.rand(size, size, device="cuda", generator=g) * 2 - 1

        def st(a=a, b=b):
            return ops.matmul(a, b)
        st()
        reps = max(5, steps) if size >= 2048 else 50
        ms = timer.run(st, reps, 3, sampler) / reps  # timing hooks off: no event records per launch
        # per-kernel device times, with the host's launches queued ahead of the GPU
        timer.run(queued(torch, st), max(3, reps // 2), 1, before_timing=lambda: hooks_on(lib))
        lib.tcx_sm100_timer_enable(0)
        kern = read_timer(lib)
        fl = 2.0 * size ** 3
        k_launches, k_ms = kern.get("gemm_tf32x3", (0, 0.0))
        k_avg = timer.max_over_ranks(k_ms / max(k_launches, 1))
        graph_ms = None
        if size <= 1024:  # latency-bound sizes: the same call replayed from a CUDA graph
            from tensorcx_b200.graphs import CapturedSequence
            seq = CapturedSequence(st)
            graph_ms = timer.run(seq, 200, 5, sampler) / 200
            seq.release()
        out[f"matmul_{size}^3"] = {
            "value": world * fl / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "graph_replay": None if graph_ms is None else {
                "ms_per_step": graph_ms, "value": world * fl / (graph_ms * 1e-3) / 1e12},
            "config": f"fp32 [{size},{size}] x [{size},{size}], U(-1,1), per-rank replica, split pre-pass + GEMM "
                      "(+ split-K reduce when the tiles fill few SMs) per step, called from Python "
                      "(graph_replay: the same call captured as a CUDA graph; kernels_ms: event pairs per "
                      "launch with the calls queued behind a 0.1 ms device spin, i.e. device time)",
            "kernels_ms": {name: round(t / max(c, 1), 4) for name, (c, t) in kern.items()},
            "roofline": {"bound": "tensor", "achieved": fl / (k_avg * 1e-3) / 1e12 if k_avg else None,
                         "peak": peak_3x, "unit": "TFLOP/s",
                         "frac": (fl / (k_avg * 1e-3) / 1e12) / peak_3x if k_avg else None,
                         "kernel": "gemm_tf32x3", "kernel_ms": k_avg}}
        del a, b

    # batched matmul + fused bias + SiLU: [64, 2048, 2048]^2, batch sharded
    nb = 64 // world
    a = torch.rand(nb, 2048, 2048, device="cuda", generator=g) * 2 - 1
    b = torch.rand(nb, 2048, 2048, device="cuda", generator=g) * 2 - 1
    bias = torch.randn(2048, device="cuda", generator=g)

    def st():
        return ops.matmul(a, b, bias=bias, act="silu")
    st()
    ms = timer.run(st, max(3, steps // 2), 1, sampler) / max(3, steps // 2)  # timing hooks off
    timer.run(st, max(3, steps // 2), 1, before_timing=lambda: hooks_on(lib))
    lib.tcx_sm100_timer_enable(0)
    kern = read_timer(lib)
    fl = 2.0 * nb * 2048 ** 3
    k_launches, k_ms = kern.get("gemm_tf32x3", (0, 0.0))
    k_avg = timer.max_over_ranks(k_ms / max(k_launches, 1))
    out["bmm_bias_silu_64x2048^3"] = {
        "value": world * fl / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
        "config": f"[64,2048,2048]^2 + bias[2048] + SiLU fused in the GEMM epilogue, batch sharded {world} way(s)",
        "roofline": {"bound": "tensor", "achieved": fl / (k_avg * 1e-3) / 1e12 if k_avg else None,
                     "peak": peak_3x, "unit": "TFLOP/s",
                     "frac": (fl / (k_avg * 1e-3) / 1e12) / peak_3x if k_avg else None,
                     "kernel": "gemm_tf32x3", "kernel_ms": k_avg}}
    del a, b

    def solo_bmm():
        a1 = torch.rand(64, 2048, 2048, device="cuda", generator=gs) * 2 - 1
        b1 = torch.rand(64, 2048, 2048, device="cuda", generator=gs) * 2 - 1
        n_b = max(3, steps // 2)
        ms1 = solo.run(lambda: ops.matmul(a1, b1, bias=bias, act="silu"), n_b, 1) / n_b
        return 2.0 * 64 * 2048 ** 3 / (ms1 * 1e-3) / 1e12
    strong("bmm_bias_silu_64x2048^3", solo_bmm)

    # attention, [32 heads, 2048 queries, 2048 keys, 128 features]: heads sharded
    heads = max(1, 32 // world)
    q = torch.randn(heads, 2048, 128, device="cuda", generator=g)
    k = torch.randn(heads, 2048, 128, device="cuda", generator=g)
    v = torch.randn(heads, 2048, 128, device="cuda", generator=g)

    def st():
        return ops.attention(q, k, v, is_causal=True)
    st()
    n_att = max(3, steps // 2)
    ms = timer.run(st, n_att, 1, sampler) / n_att  # step time with the timing hooks off
    timer.run(st, n_att, 1, before_timing=lambda: hooks_on(lib))
    lib.tcx_sm100_timer_enable(0)
    kern = read_timer(lib)
    fl = 4.0 * heads * 2048 * 2048 * 128
    # work the fused kernel executes: causal key blocks of 128 up to the diagonal only
    qtiles = 2048 // 128
    executed = heads * sum(min(qtiles, t + 1) for t in range(qtiles)) * 2.0 * 128 * 128 * (128 + 128)
    k_launches, k_ms = kern.get("flash_tf32x3", (0, 0.0))
    k_avg = timer.max_over_ranks(k_ms / max(k_launches, 1))
    out["attention_causal_32x2048x2048x128"] = {
        "value": world * fl / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
        "config": f"q,k,v [32,2048,128] float32, causal, heads sharded {world} way(s); value counts "
                  "4*H*L*S*D flops (both products, masked half included)",
        "kernels_ms": {name: round(t / max(c, 1), 4) for name, (c, t) in kern.items()},
        "roofline": {"bound": "tensor", "achieved": executed / (k_avg * 1e-3) / 1e12 if k_avg else None,
                     "peak": peak_3x, "unit": "TFLOP/s",
                     "frac": (executed / (k_avg * 1e-3) / 1e12) / peak_3x if k_avg else None,
                     "kernel": "flash_tf32x3", "kernel_ms": k_avg,
                     "note": "achieved = flops of the key blocks executed (up to the causal diagonal)"}}

    # the same product with a float additive mask [2048, 2048] (-inf entries mask keys),
    # broadcast over the heads: read inside the fused kernel
    mgen = torch.Generator(device="cuda").manual_seed(99)
    amask = torch.randn(2048, 2048, device="cuda", generator=mgen)
    amask[torch.rand(2048, 2048, device="cuda", generator=mgen) < 0.1] = float("-inf")

    def st_masked():
        return ops.attention(q, k, v, amask)
    st_masked()
    ms_m = timer.run(st_masked, n_att, 1, sampler) / n_att
    timer.run(st_masked, max(3, n_att // 2), 1, before_timing=lambda: hooks_on(lib))
    lib.tcx_sm100_timer_enable(0)
    kern_m = read_timer(lib)
    fl_m = 4.0 * heads * 2048 * 2048 * 128
    km_launches, km_ms = kern_m.get("flash_tf32x3", (0, 0.0))
    km_avg = timer.max_over_ranks(km_ms / max(km_launches, 1))
    out["attention_masked_32x2048x2048x128"] = {
        "value": world * fl_m / (ms_m * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms_m,
        "config": f"q,k,v [32,2048,128] float32, float32 additive mask [2048,2048] (10 % -inf) broadcast over "
                  f"heads, not causal, heads sharded {world} way(s); 4*H*L*S*D flops",
        "kernels_ms": {name: round(t / max(c, 1), 4) for name, (c, t) in kern_m.items()},
        "roofline": {"bound": "tensor", "achieved": fl_m / (km_avg * 1e-3) / 1e12 if km_avg else None,
                     "peak": peak_3x, "unit": "TFLOP/s",
                     "frac": (fl_m / (km_avg * 1e-3) / 1e12) / peak_3x if km_avg else None,
                     "kernel": "flash_tf32x3", "kernel_ms": km_avg}}
    del amask, q, k, v

    def solo_attention():
        q1, k1, v1 = (torch.randn(32, 2048, 128, device="cuda", generator=gs) for _ in range(3))
        ms1 = solo.run(lambda: ops.attention(q1, k1, v1, is_causal=True), n_att, 1) / n_att
        return 4.0 * 32 * 2048 * 2048 * 128 / (ms1 * 1e-3) / 1e12
    if heads * world == 32:
        strong("attention_causal_32x2048x2048x128", solo_attention)

    # MLP latency (configs[0]: x[256,784] -> linear 512 + ReLU -> linear 10 -> softmax)
    x = torch.randn(256, 784, device="cuda", generator=g)
    w1 = (torch.rand(784, 512, device="cuda", generator=g) * 2 - 1) / 784 ** 0.5
    w2 = (torch.rand(512, 10, device="cuda", generator=g) * 2 - 1) / 512 ** 0.5
    b1 = torch.zeros(512, device="cuda")
    b2 = torch.zeros(10, device="cuda")

    def mlp():
        h = ops.matmul(x, w1, bias=b1, act="relu")
        return ops.softmax(ops.matmul(h, w2, bias=b2), axis=-1)
    mlp()
    eager_ms = timer.run(mlp, 50, 1, sampler) / 50  # timing hooks off
    timer.run(mlp, 20, 1, before_timing=lambda: hooks_on(lib))
    lib.tcx_sm100_timer_enable(0)
    kern = read_timer(lib)
    # the same forward replayed as one CUDA graph (no host work per op)
    from tensorcx_b200.graphs import CapturedSequence
    seq = CapturedSequence(mlp)
    ms = timer.run(seq, 200, 5, sampler) / 200
    seq.release()
    out["mlp_256x784x512x10_latency"] = {
        "value": ms, "unit": "ms", "higher_is_better": False, "ms_per_step": ms,
        "eager_ms": eager_ms,
        "config": "x[256,784] @ W1[784,512] + b1 -> ReLU (fused epilogue) -> @ W2[512,10] + b2 -> softmax; "
                  "per-rank replica; value: the forward captured once as a CUDA graph "
                  "(tensorcx_b200.graphs.CapturedSequence) and replayed back to back; eager_ms: the same ops "
                  "called from Python, stream-ordered, no host sync inside",
        "gpu_launches_per_step": sum(c for c, _ in kern.values()) / 20,
        "kernels_ms": {name: round(t / max(c, 1), 4) for name, (c, t) in kern.items()}}
    return out


def main():
    args = parse()
    if args.case:
        run_case(args)
        return
    if args.impl == "reference":
        reference_arm(args)
        return
    gpu_arm(args)


if __name__ == "__main__":
    main()
