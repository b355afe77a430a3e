"""Benchmark driver for tosa_b200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

Workloads (synthetic seeded inputs of the stated
shapes and distributions):
  matmul  config 2: batched int8 MATMUL A[8,1024,1024] x B[8,1024,1024], a/b zero
          points in [-8,8], fused RESCALE (single multiplier, shift 35,
          single_round) to int8. Metric: int8 TOPS (2*8*1024^3 ops per step).
  conv    config 1: int8 CONV2D [1,56,56,64] x [64,3,3,64] pad 1, input_zp -3,
          per-channel double-round RESCALE to int8 (output_zp 5).

Multi-GPU (torchrun, one process per GPU): every rank runs its own copy of the
workload (weak scaling; the batch shards are independent, no collective on the
data path). Timing: W untimed warm-up steps; K timed steps, each bracketed by
CUDA events on the launching stream with the L2 flushed (a 256 MiB write)
between steps; barrier + synchronize around the timed region; the max over
ranks of the summed step time. `e2e` repeats the measurement through the same
C-ABI entry point with the step's inputs copied from pinned host memory and
its output copied back inside the timed region.

`--impl reference` times the reference's arithmetic on the host CPU cores
instead: the C restatement of the reference loops (oracle/, the reference is
Rust and cannot be built here), multi-threaded over output rows, each step a
bounded sample of the workload.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "int8 conv/matmul TOPS; ResNet-50-shape int8 graph img/s at 1/2/4/8 B200"
L2_FLUSH_BYTES = 256 << 20


# ---------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------


class MatmulWorkload:
    """BASELINE config 2."""

    name = "matmul"
    unit = "TOPS"
    N, H, C, W = 8, 1024, 1024, 1024
    seed = 2

    def __init__(self):
        rng = np.random.default_rng(self.seed)
        self.a = rng.integers(-128, 128, (self.N, self.H, self.C), dtype=np.int8)
        self.b = rng.integers(-128, 128, (self.N, self.C, self.W), dtype=np.int8)
        self.za = int(rng.integers(-8, 9))
        self.zb = int(rng.integers(-8, 9))
        self.mult = int(rng.integers(1 << 30, 1 << 31))
        self.shift = 35
        self.ops = 2 * self.N * self.H * self.C * self.W

    def config(self):
        return {"workload": "config2: batched int8 MATMUL [8,1024,1024]x[8,1024,1024] + RESCALE(single_round, "
                            "shift 35) -> int8",
                "global_batch": self.N, "a_zp": self.za, "b_zp": self.zb,
                "l2": "flushed between timed steps (256 MiB write)"}

    # -- GPU
    def setup(self, L, ctx, torch):
        self.L, self.torch = L, torch
        d = L.MatmulDesc(n=self.N, h=self.H, c=self.C, w=self.W, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8,
                         out_dtype=L.DT_INT32, a_zp=self.za, b_zp=self.zb)
        self.attr = L.rescale_attr([self.mult], [self.shift], rounding=L.ROUND_SINGLE, out_dtype=L.DT_INT8)
        h = ctypes.c_void_p()
        L.check(L.load().tb_matmul_plan_create(ctx.h, d, self.attr, ctypes.byref(h)))
        self.plan = h
        self.da = torch.from_numpy(self.a).cuda()
        self.db = torch.from_numpy(self.b).cuda()
        self.dout = torch.empty((self.N, self.H, self.W), dtype=torch.int8, device="cuda")
        self.ha = torch.from_numpy(self.a).pin_memory()
        self.hb = torch.from_numpy(self.b).pin_memory()
        self.hout = torch.empty((self.N, self.H, self.W), dtype=torch.int8).pin_memory()
        self.h2d = self.a.nbytes + self.b.nbytes
        self.d2h = self.N * self.H * self.W

    def step(self, stream):
        L = self.L
        L.check(L.load().tb_matmul_plan_run(self.plan, L.ptr(self.da), L.ptr(self.db), L.ptr(self.dout),
                                            L.stream_ptr(stream)))

    def step_e2e(self, stream):
        self.da.copy_(self.ha, non_blocking=True)
        self.db.copy_(self.hb, non_blocking=True)
        self.step(stream)
        self.hout.copy_(self.dout, non_blocking=True)

    def check(self, rows=16):
        """Bit-exact spot check of the device result against the oracle."""
        from tests import helpers as H
        got = self.dout.cpu().numpy()
        a = self.a[:1, :rows].astype(np.int64)
        acc = H.oracle_matmul_int(a, self.b[:1].astype(np.int64), self.za, self.zb)
        rc, exp = H.oracle_rescale(acc, 5, 3, [self.mult], [self.shift], 0, 0, 1, 1, 0)
        return rc == 0 and np.array_equal(got[:1, :rows].reshape(-1).astype(np.int64), exp)

    def close(self):
        self.L.load().tb_matmul_plan_destroy(self.plan)

    # -- roofline of the dominant kernel
    kernel_regex = "tc_gemm_kernel"

    # -- CPU (oracle restatement)
    def cpu_run(self, rows, threads):
        """MATMUL + RESCALE of the first `rows` rows of A (row-major over [N*H], so a
        sample may span batches) against their batch's B; returns ops done."""
        from oracle import oracle as O
        L = O.lib()
        p = lambda x: x.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        mult = np.array([self.mult], np.int64)
        shift = np.array([self.shift], np.int64)
        done = 0
        while done < rows:
            bi, r0 = divmod(done, self.H)
            nr = min(rows - done, self.H - r0)
            a = np.ascontiguousarray(self.a[bi, r0:r0 + nr], dtype=np.int64)
            b = np.ascontiguousarray(self.b[bi], dtype=np.int64)
            out = np.zeros(nr * self.W, dtype=np.int64)
            if threads > 1:
                L.orc_matmul_int_mt(ctypes.c_int64(1), ctypes.c_int64(nr), ctypes.c_int64(self.C),
                                    ctypes.c_int64(self.W), p(a), p(b), ctypes.c_int64(self.za),
                                    ctypes.c_int64(self.zb), p(out), ctypes.c_int(threads))
            else:
                L.orc_matmul_int(ctypes.c_int64(1), ctypes.c_int64(nr), ctypes.c_int64(self.C),
                                 ctypes.c_int64(self.W), p(a), p(b), ctypes.c_int64(self.za),
                                 ctypes.c_int64(self.zb), ctypes.c_int(0), p(out))
            res = np.zeros_like(out)
            L.orc_rescale(p(out), ctypes.c_int64(out.size), ctypes.c_int(5), ctypes.c_int(3), p(mult), p(shift),
                          ctypes.c_int64(1), ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_int(1), ctypes.c_int(1),
                          ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0), p(res))
            done += nr
        return 2 * rows * self.C * self.W

    def cpu_sample_desc(self, rows, threads):
        return (f"first {rows} of the {self.N * self.H} rows of A[8,1024,1024] (row-major over batch) x their "
                f"batch's B + RESCALE ({rows}x1024x1024 MACs), {threads} thread(s), C restatement of the "
                f"reference loops")


WORKLOADS = {"matmul": MatmulWorkload}


# ---------------------------------------------------------------------------
# Measurement helpers
# ---------------------------------------------------------------------------


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def measure_int8_peak(torch):
    """Dense int8 tensor throughput of cuBLASLt (torch._int_mm, 8192^3), best of 10:
    the roofline denominator for the int8 kernels (no int8 figure is
    provided by the pool's measured peaks)."""
    try:
        n = 8192
        a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda").t().contiguous().t()
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = 0.0
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch._int_mm(a, b)
            e.record()
            e.synchronize()
            best = max(best, 2 * n ** 3 / (s.elapsed_time(e) * 1e-3) / 1e12)
        del a, b
        return best, "measured in this run: torch._int_mm (cuBLASLt) int8 8192^3, best of 10"
    except Exception as ex:  # pragma: no cover
        return 4500.0, f"nominal dense int8 4.5 POPS (measurement failed: {ex})"


def load_traffic(kernel_workload):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(kernel_workload)
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------------------
# Arms
# ---------------------------------------------------------------------------


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_reference(args, wl):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    rows = args.ref_rows
    for _ in range(args.warmup):
        wl.cpu_run(rows, threads)
    t0 = time.perf_counter()
    ops = 0
    for _ in range(args.steps):
        ops += wl.cpu_run(rows, threads)
    dt = time.perf_counter() - t0
    value = ops / dt / 1e12
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": wl.unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "config": wl.config(),
            "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
                             "sample": wl.cpu_sample_desc(rows, threads)},
            "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_gpu(args, wl):
    import torch

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    from tosa_b200 import _lib as L

    ctx = L.Context(local)
    wl.setup(L, ctx, torch)
    stream = torch.cuda.current_stream()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def barrier():
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        wl.step(stream)
    ctx.synchronize(stream)
    ok = wl.check()

    def timed(fn):
        evs = []
        barrier()
        for _ in range(args.steps):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn(stream)
            e.record(stream)
            evs.append((s, e))
        barrier()
        ms = sum(s.elapsed_time(e) for s, e in evs)
        if ws > 1:
            t = torch.tensor([ms], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def soak(seconds):
        # keeps the GPU busy with the same step so the clock samples see load
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            for _ in range(50):
                wl.step(stream)
            torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    soak(0.6)
    launches0 = ctx.launches
    ms = timed(wl.step)
    launches = ctx.launches - launches0
    soak(0.6)
    clk = clocks.stop()
    ctx.synchronize(stream)
    for _ in range(args.warmup):
        wl.step_e2e(stream)
    ms_e2e = timed(wl.step_e2e)
    ctx.synchronize(stream)

    # roofline: the dominant kernel timed alone (same launch as a step)
    peak, peak_src = (None, None)
    kernel_ms = None
    if rank == 0:
        evs = []
        for _ in range(args.steps):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            wl.step(stream)
            e.record(stream)
            evs.append((s, e))
        torch.cuda.synchronize()
        kernel_ms = statistics.mean(s.elapsed_time(e) for s, e in evs)
        del flush
        peak, peak_src = measure_int8_peak(torch)

    value = ws * wl.ops * args.steps / (ms * 1e-3) / 1e12
    e2e = ws * wl.ops * args.steps / (ms_e2e * 1e-3) / 1e12
    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu:
            rows = args.cpu_rows
            t0 = time.perf_counter()
            ops = wl.cpu_run(rows, 1)  # ~10 s of single-thread work at the default size
            dt = time.perf_counter() - t0
            cpu = {"value": ops / dt / 1e12, "unit": wl.unit, "cores": 1, "kind": "port",
                   "sample": wl.cpu_sample_desc(rows, 1)}
        achieved = wl.ops / (kernel_ms * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": wl.unit, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "config": wl.config(),
            "parity_spot_check": bool(ok),
            "e2e": {"value": e2e, "unit": wl.unit, "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOPS (int8)",
                         "frac": achieved / peak if peak else None, "traffic": load_traffic(wl.name),
                         "peak_source": peak_src,
                         "note": "achieved = 2*M*N*K of one step / mean CUDA-event time of the step "
                                 "(one GEMM launch with the zero-point column sums and RESCALE fused), "
                                 "L2 flushed; clocks sampled during a 1.2 s soak of the same step around "
                                 "the timed region"},
            "cpu_baseline": cpu,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    wl.close()
    ctx.close()
    if ws > 1:
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="matmul", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="tosa_b200", choices=["tosa_b200", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=1536, help="rows of the single-thread CPU baseline sample")
    ap.add_argument("--ref-rows", type=int, default=1024, help="rows per step of the --impl reference arm")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl = WORKLOADS[args.workload]()
    if args.impl == "reference":
        return run_reference(args, wl)
    return run_gpu(args, wl)


if __name__ == "__main__":
    sys.exit(main())
