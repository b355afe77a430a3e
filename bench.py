"""Benchmark driver for tosa_b200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

Workloads (synthetic seeded inputs of the stated shapes
and distributions, random-init weights):
  resnet50     (default) config 4: the ResNet-50-shaped int8 TOSA graph
               (tosa_b200/graphs.py), 64 images per GPU, run by the graph runner
               (one CUDA graph per step). Metric: images/s; the roofline line
               reports the int8 TOPS of its tensor-core convolutions.
  matmul       config 2: batched int8 MATMUL A[8,1024,1024] x B[8,1024,1024], a/b
               zero points in [-8,8], fused RESCALE (single multiplier, shift 35,
               single_round) to int8. Metric: int8 TOPS (2*8*1024^3 ops per step).
  mobilenetv2  config 3: the MobileNetV2-shaped int8 graph, batch 64 per GPU.
  conv1        config 1: one int8 CONV2D [1,56,56,64] x [64,3,3,64] + per-channel RESCALE to
               int8 (the CPU-runnable case), one image per step; the roofline line times the
               same layer over 64 images. Metric: int8 TOPS.
  bf16         config 5: the five bf16 x bf16 -> fp32 MATMULs of one transformer block (QKV,
               attention scores, P.V, MLP up and down). Metric: TFLOP/s; roofline against the
               pool's measured sustained bf16 peak.

Multi-GPU (torchrun, one process per GPU): every rank runs its own shard of the
workload (weak scaling: 64 images per GPU, the global batch 64 x N; the shards
are independent, no collective on the data path). Timing: W untimed warm-up steps; K timed steps, each bracketed by
CUDA events on the launching stream with the L2 flushed (a 256 MiB write)
between steps; barrier + synchronize around the timed region; the max over
ranks of the summed step time. `e2e` repeats the measurement through the same
public entry point with every step's inputs copied from pinned host memory and
its output copied back, double-buffered as a server would run it: step i+1's
inputs upload on a copy stream into device staging buffers while step i computes,
and move to the bound input buffers (a device-to-device copy) when step i+1
starts; the time runs from the first upload to the last result download (the L2
flushes between steps subtracted), so every copy lies inside it.

`--impl reference` times the reference's arithmetic on the host CPU cores
instead: the C restatement of the reference loops (oracle/; the reference is
Rust and cannot be built here) on all host threads, each step a bounded sample
of the workload.
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
    kernel = "tc_gemm_kernel"

    def __init__(self, args):
        rng = np.random.default_rng(self.seed)
        self.a = rng.integers(-128, 128, (self.N, self.H, self.C), dtype=np.int8)
        self.b = rng.integers(-128, 128, (self.N, self.C, self.W), dtype=np.int8)
        self.za = int(rng.integers(-8, 9))
        self.zb = int(rng.integers(-8, 9))
        self.mult = int(rng.integers(1 << 30, 1 << 31))
        self.shift = 35
        self.ops = 2 * self.N * self.H * self.C * self.W
        self.units_per_step = self.ops / 1e12  # TOPS

    def config(self):
        return {"workload": "config2: batched int8 MATMUL [8,1024,1024]x[8,1024,1024] + RESCALE(single_round, "
                            "shift 35) -> int8",
                "global_batch": self.N, "a_zp": self.za, "b_zp": self.zb,
                "l2": "flushed between timed steps (256 MiB write)"}

    # -- GPU
    def setup(self, L, ctx, torch, stream):
        self.L, self.torch, self.ctx = L, torch, ctx
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
        n0 = self.ctx.launches
        L.check(L.load().tb_matmul_plan_run(self.plan, L.ptr(self.da), L.ptr(self.db), L.ptr(self.dout),
                                            L.stream_ptr(stream)))
        return self.ctx.launches - n0  # the column-term kernel (a_zp != 0) and the GEMM

    def e2e_inputs(self):
        return [(self.ha, self.da), (self.hb, self.db)]

    def e2e_output(self, stream):
        self.hout.copy_(self.dout, non_blocking=True)

    def check(self, rows=16):
        """Bit-exact spot check against the oracle: the first rows of the first batch and
        the last rows of the last batch."""
        from tests import helpers as H
        got = self.dout.cpu().numpy()
        for bi, r0 in ((0, 0), (self.N - 1, self.H - rows)):
            a = self.a[bi:bi + 1, r0:r0 + rows].astype(np.int64)
            acc = H.oracle_matmul_int(a, self.b[bi:bi + 1].astype(np.int64), self.za, self.zb)
            rc, exp = H.oracle_rescale(acc, 5, 3, [self.mult], [self.shift], 0, 0, 1, 1, 0)
            if rc != 0 or not np.array_equal(got[bi, r0:r0 + rows].reshape(-1).astype(np.int64), exp):
                return False
        return True

    def kernel_time(self, stream, flush, steps):
        """Mean CUDA-event time of the step: the GEMM, and before it the column-term kernel
        of the A zero point, which the GEMM overlaps (both counted as the GEMM's time)."""
        torch = self.torch
        evs = []
        for _ in range(steps):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            self.step(stream)
            e.record(stream)
            evs.append((s, e))
        torch.cuda.synchronize()
        ms = statistics.mean(s.elapsed_time(e) for s, e in evs)
        return self.ops / (ms * 1e-3) / 1e12, "TOPS (int8)", ms, 1

    def close(self):
        if getattr(self, "plan", None) is not None:
            self.L.load().tb_matmul_plan_destroy(self.plan)
            self.plan = None

    # -- CPU (oracle restatement)
    def cpu_run(self, rows, threads):
        """MATMUL + RESCALE of the first `rows` rows of A (row-major over [N*H], so a
        sample may span batches) against their batch's B; returns work done in units."""
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
        return 2 * rows * self.C * self.W / 1e12

    def cpu_default(self, args):
        return args.cpu_rows

    def ref_default(self, args):
        return args.ref_rows

    def cpu_sample_desc(self, rows, threads):
        return (f"first {rows} of the {self.N * self.H} rows of A[8,1024,1024] (row-major over batch) x their "
                f"batch's B + RESCALE ({rows}x1024x1024 MACs), {threads} thread(s), C restatement of the "
                f"reference loops")


def _oracle_image(data, image):
    """Run one image through the oracle (a worker of the CPU baseline)."""
    from oracle import oracle as O
    block = O.read_graph(data).main_block
    name = block.inputs[0]
    return O.run_block(block, {name: O.T(3, list(image.shape), image.astype(np.int64).reshape(-1))})


class GraphWorkload:
    """A synthetic int8 TOSA graph run by the graph runner (configs 3 and 4)."""

    unit = "img/s"
    kernel = "tc_gemm_kernel"
    batch = 64
    seed = 21

    def __init__(self, args):
        from tosa_b200 import graphs
        self.graphs = graphs
        self.batch = args.batch or self.batch
        self.data, self.info = self.builder(self.batch)
        self.units_per_step = self.batch
        rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        rng = np.random.default_rng(self.seed + rank)  # this rank's shard of the global batch
        self.images = rng.integers(-128, 128, (self.batch, 224, 224, 3), dtype=np.int8)

    def config(self):
        return {"workload": self.desc, "global_batch": self.batch * self.world, "batch_per_gpu": self.batch,
                "parallelism": f"dp{self.world} (batch sharded, no collective on the data path)",
                "int_ops_per_image": self.info["ops_per_image"],
                "l2": "flushed between timed steps (256 MiB write); activations exceed L2"}

    def setup(self, L, ctx, torch, stream):
        from tosa_b200 import interpreter as I
        self.L, self.torch, self.I = L, torch, I
        self.ctx = ctx
        self.dimg = torch.from_numpy(self.images).cuda()
        self.himg = torch.from_numpy(self.images).pin_memory()
        self.it = I.Interpreter(self.data, context=ctx, cuda_graph=True)
        self.it.bind_device(self.info["input"], L.DT_INT8, list(self.images.shape), self.dimg.data_ptr())
        self.out_name = self.info["output"]
        self.h2d = self.images.nbytes
        self.it.execute(stream=stream)  # compile + capture
        info = L.TensorInfo()
        L.check(L.load().tb_graph_get_output(self.it._h, self.out_name.encode(), ctypes.byref(info)))
        self.out_ptr = info.data
        self.out_bytes = int(np.prod([info.shape[i] for i in range(info.rank)])) * 4
        self.hout = torch.empty(self.out_bytes, dtype=torch.uint8).pin_memory()
        self.d2h = self.out_bytes

    def step(self, stream):
        self.it.execute(stream=stream)
        return self.it.last_launches

    def e2e_inputs(self):
        return [(self.himg, self.dimg)]

    def e2e_output(self, stream):
        L = self.L
        L.check(L.load().tb_memcpy_d2h(self.ctx.h, ctypes.c_void_p(self.hout.data_ptr()),
                                       ctypes.c_void_p(self.out_ptr), self.out_bytes, L.stream_ptr(stream)))

    def check(self):
        """The first and the last image's logits bit-exact against the oracle."""
        got = self.it.output(self.out_name).data.reshape(self.batch, -1).astype(np.int64)
        d1, _ = self.builder(1)
        for i in sorted({0, self.batch - 1}):
            want = _oracle_image(d1, self.images[i:i + 1])
            if not np.array_equal(next(iter(want.values())).values, got[i]):
                return False
        return True

    def kernel_time(self, stream, flush, steps):
        """Per-operator CUDA-event times of an eager run; the dominant kernel is the
        tensor-core implicit-GEMM convolution: achieved = its 2*MACs / its time."""
        I = self.I
        it = I.Interpreter(self.data, context=self.ctx, time_ops=True)
        it.bind_device(self.info["input"], self.L.DT_INT8, list(self.images.shape), self.dimg.data_ptr())
        it.execute(stream=stream)  # compile
        block = self.graphs.TG.read_graph(self.data).main_block
        conv_ops = [i for i, o in enumerate(block.operators) if o.name == "CONV2D"]
        tc_ops = [i for i in conv_ops if block.tensor(block.operators[i].inputs[0]).shape[3] % 16 == 0]
        tot_ms, tot_macs, all_ms, n = 0.0, 0, 0.0, 0
        for _ in range(steps):
            flush.fill_(1)
            it.execute(stream=stream)
            for i in range(len(block.operators)):
                t = it.op_time_ms(i)
                if t > 0:
                    all_ms += t
            for i in tc_ops:
                tot_ms += it.op_time_ms(i)
                tot_macs += self.info["op_macs"][i]
            n += len(tc_ops)
        it.close()
        self.kernel_share = tot_ms / all_ms if all_ms else None
        return 2 * tot_macs / (tot_ms * 1e-3) / 1e12, "TOPS (int8)", tot_ms / n, len(tc_ops)

    def close(self):
        if getattr(self, "it", None) is not None:
            self.it.close()
        if getattr(self, "_pool", None) is not None:
            self._pool.close()
            self._pool.join()
            self._pool = None

    # -- CPU (oracle restatement): whole images through the graph
    def cpu_run(self, images, threads):
        if not hasattr(self, "_d1"):
            self._d1, _ = self.builder(1)
        imgs = [self.images[i % self.batch][None] for i in range(images)]
        if threads > 1:
            if getattr(self, "_pool", None) is None:
                import multiprocessing as mp
                self._pool = mp.get_context("spawn").Pool(threads)  # kept for every step of the run
            self._pool.starmap(_oracle_image, [(self._d1, im) for im in imgs])
        else:
            for im in imgs:
                _oracle_image(self._d1, im)
        return images

    def cpu_default(self, args):
        return 3  # about 15 s of single-core work

    def ref_default(self, args):
        return os.cpu_count() or 1

    def cpu_sample_desc(self, images, threads):
        return (f"{images} image(s) through the whole {self.name} graph at batch 1 on {threads} "
                f"process(es), C restatement of the reference loops")


class ResNet50Workload(GraphWorkload):
    name = "resnet50"
    desc = ("config4: ResNet-50-shaped int8 TOSA graph (stem 7x7/s2, stages [3,4,6,3], RESCALE+CLAMP after "
            "every conv, residual ADD via RESCALE to int32, AVG_POOL2D, 2048->1000 MATMUL), 224x224x3 int8")

    def builder(self, batch):
        return self.graphs.resnet50_int8(batch)


class MobileNetV2Workload(GraphWorkload):
    name = "mobilenetv2"
    desc = ("config3: MobileNetV2-shaped int8 TOSA graph (17 inverted-residual blocks, expand x6, depthwise "
            "3x3, RESCALE+CLAMP[0,127], residual ADD via RESCALE to int32, AVG_POOL2D, 1280->1000 MATMUL)")

    def builder(self, batch):
        return self.graphs.mobilenetv2_int8(batch)


class Conv1Workload:
    """one int8 CONV2D [1,56,56,64] x [64,3,3,64] (pad 1, input zero point -3)
    with its per-channel double-rounding RESCALE to int8 fused (output zero point 5). The step
    is that one image; the roofline line times the same layer over 64 images, where the
    tensor cores have enough tiles to be measured."""

    name = "conv1"
    unit = "TOPS"
    kernel = "tc_gemm_kernel"
    dtype = "int8"
    seed = 1
    roof_batch = 64

    def __init__(self, args):
        rng = np.random.default_rng(self.seed)
        self.x = rng.integers(-128, 128, (1, 56, 56, 64), dtype=np.int8)
        self.w = rng.integers(-127, 128, (64, 3, 3, 64), dtype=np.int8)
        self.bias = rng.integers(-32768, 32768, 64).astype(np.int32)
        self.mult = rng.integers(1 << 30, (1 << 31) - 1, 64, endpoint=True)
        self.shift = rng.integers(30, 39, 64)
        self.macs = 56 * 56 * 64 * 3 * 3 * 64
        self.ops = 2 * self.macs
        self.units_per_step = self.ops / 1e12

    def config(self):
        return {"workload": "config1: int8 CONV2D [1,56,56,64] x [64,3,3,64], pad 1, input_zp -3, weight_zp 0, "
                            "+ per-channel RESCALE (double_round, shift 30-38, output_zp 5) -> int8, one image",
                "global_batch": 1, "roofline_batch": self.roof_batch,
                "l2": "flushed between timed steps (256 MiB write)"}

    def _plan(self, L, ctx, n):
        d = L.conv_desc(n, 56, 56, 64, 64, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), L.DT_INT8, L.DT_INT8, L.DT_INT32,
                        L.DT_INT32, -3, 0, 64)
        h = ctypes.c_void_p()
        L.check(L.load().tb_conv2d_plan_create(ctx.h, d, L.ptr(self.dw), L.ptr(self.db), self.attr, ctypes.byref(h)))
        return h

    def setup(self, L, ctx, torch, stream):
        self.L, self.torch = L, torch
        self.attr = L.rescale_attr(self.mult, self.shift, rounding=L.ROUND_DOUBLE, output_zp=5, out_dtype=L.DT_INT8)
        self.dw = torch.from_numpy(self.w).cuda()
        self.db = torch.from_numpy(self.bias).cuda()
        self.plan = self._plan(L, ctx, 1)
        self.ctx = ctx
        self.dx = torch.from_numpy(self.x).cuda()
        self.dout = torch.empty((1, 56, 56, 64), dtype=torch.int8, device="cuda")
        self.hx = torch.from_numpy(self.x).pin_memory()
        self.hout = torch.empty((1, 56, 56, 64), dtype=torch.int8).pin_memory()
        self.h2d = self.x.nbytes
        self.d2h = self.hout.numel()

    def step(self, stream):
        L = self.L
        L.check(L.load().tb_conv2d_plan_run(self.plan, L.ptr(self.dx), L.ptr(self.dout), L.stream_ptr(stream)))
        return 1

    def e2e_inputs(self):
        return [(self.hx, self.dx)]

    def e2e_output(self, stream):
        self.hout.copy_(self.dout, non_blocking=True)

    def _oracle(self, x):
        from tests import helpers as H
        acc = H.oracle_conv_int(x.astype(np.int64), self.w.astype(np.int64), self.bias.astype(np.int64), -3, 0,
                                (1, 1, 1, 1), (1, 1), (1, 1))
        rc, q = H.oracle_rescale(acc, 5, 3, self.mult, self.shift, 0, 5, 1, 3, 1)
        return rc, q.reshape(acc.shape)

    def check(self):
        """The whole output bit-exact against the oracle."""
        rc, want = self._oracle(self.x)
        return rc == 0 and np.array_equal(self.dout.cpu().numpy().astype(np.int64), want)

    def kernel_time(self, stream, flush, steps):
        """CUDA-event time of the same layer over 64 images (one launch of the GEMM)."""
        torch, L = self.torch, self.L
        plan = self._plan(L, self.ctx, self.roof_batch)
        x = torch.randint(-128, 128, (self.roof_batch, 56, 56, 64), dtype=torch.int8, device="cuda")
        out = torch.empty((self.roof_batch, 56, 56, 64), dtype=torch.int8, device="cuda")
        run = lambda: L.check(L.load().tb_conv2d_plan_run(plan, L.ptr(x), L.ptr(out), L.stream_ptr(stream)))  # noqa
        run()
        evs = []
        for _ in range(steps):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            run()
            e.record(stream)
            evs.append((s, e))
        torch.cuda.synchronize()
        L.load().tb_conv2d_plan_destroy(plan)
        ms = statistics.mean(s.elapsed_time(e) for s, e in evs)
        return self.roof_batch * self.ops / (ms * 1e-3) / 1e12, "TOPS (int8)", ms, 1

    def close(self):
        if getattr(self, "plan", None) is not None:
            self.L.load().tb_conv2d_plan_destroy(self.plan)
            self.plan = None

    def cpu_run(self, images, threads):
        """`images` config-1 convolutions (+ RESCALE) through the oracle's C loops."""
        from oracle import oracle as O
        from tests import helpers as H
        if threads > 1:
            x = np.ascontiguousarray(np.repeat(self.x, images, axis=0), np.int64)
            g = H.conv_geom(x.shape, self.w.shape, (1, 1, 1, 1), (1, 1), (1, 1))
            acc = np.zeros(images * 56 * 56 * 64, dtype=np.int64)
            p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
            O.lib().orc_conv2d_int_mt(ctypes.byref(g), p(x), p(np.ascontiguousarray(self.w, np.int64)),
                                      p(np.ascontiguousarray(self.bias, np.int64)), ctypes.c_int64(64),
                                      ctypes.c_int64(-3), ctypes.c_int64(0), p(acc), ctypes.c_int(threads))
            H.oracle_rescale(acc, 5, 3, self.mult, self.shift, 0, 5, 1, 3, 1)
        else:
            for _ in range(images):
                self._oracle(self.x)
        return images * self.units_per_step

    def cpu_default(self, args):
        return 100  # about 12 s of single-core work

    def ref_default(self, args):
        return 2 * (os.cpu_count() or 1)

    def cpu_sample_desc(self, images, threads):
        return (f"{images} config-1 convolution(s) + RESCALE (115.6 M MAC each) on {threads} thread(s), "
                f"C restatement of the reference loops")


class Bf16Workload:
    """the bf16 contractions of one transformer block (batch 32, sequence 512,
    hidden 4096, 32 heads), MATMUL with fp32 results: QKV [1,16384,4096] x [1,4096,12288],
    attention scores [1024,512,128] x [1024,128,512] and P.V [1024,512,512] x [1024,512,128],
    MLP [1,16384,4096] x [1,4096,11008] and [1,16384,11008] x [1,11008,4096]. Activations
    N(0,1), weights N(0,0.02), cast to bf16. A step runs the five; the metric is TFLOP/s."""

    name = "bf16"
    unit = "TFLOP/s"
    kernel = "tc_gemm_kernel"
    dtype = "bf16"
    seed = 5
    # (name, n, h, c, w, B is a weight)
    SHAPES = [("qkv", 1, 16384, 4096, 12288, True), ("scores", 1024, 512, 128, 512, False),
              ("pv", 1024, 512, 512, 128, False), ("mlp_up", 1, 16384, 4096, 11008, True),
              ("mlp_down", 1, 16384, 11008, 4096, True)]

    def __init__(self, args):
        self.flops = sum(2 * n * h * c * w for _, n, h, c, w, _ in self.SHAPES)
        self.units_per_step = self.flops / 1e12

    def config(self):
        return {"workload": "config5: bf16 transformer-block contractions (batch 32, seq 512, hidden 4096, 32 heads): "
                            "QKV [16384,4096]x[4096,12288], scores [1024,512,128]x[1024,128,512], "
                            "P.V [1024,512,512]x[1024,512,128], MLP 4096->11008->4096; MATMUL bf16 x bf16 -> fp32",
                "global_batch": 32, "seq_len": 512, "flop_per_step": self.flops,
                "l2": "operands larger than L2; flushed between timed steps (256 MiB write)",
                "e2e_copies": "every activation operand uploaded, the MLP output downloaded"}

    def setup(self, L, ctx, torch, stream):
        self.L, self.torch, self.ctx = L, torch, ctx
        g = torch.Generator(device="cuda")
        g.manual_seed(self.seed)
        self.ops = []
        for name, n, h, c, w, weight in self.SHAPES:
            a = torch.randn((n, h, c), generator=g, device="cuda").to(torch.bfloat16)
            b = (torch.randn((n, c, w), generator=g, device="cuda") * (0.02 if weight else 1.0)).to(torch.bfloat16)
            out = torch.empty((n, h, w), dtype=torch.float32, device="cuda")
            d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_BF16, b_dtype=L.DT_BF16, out_dtype=L.DT_FP32,
                             a_zp=0, b_zp=0)
            plan = ctypes.c_void_p()
            L.check(L.load().tb_matmul_plan_create(ctx.h, d, None, ctypes.byref(plan)))
            self.ops.append({"name": name, "shape": (n, h, c, w), "a": a, "b": b, "out": out, "plan": plan,
                             "weight": weight})
        uploads = []
        for op in self.ops:
            uploads.append(op["a"])
            if not op["weight"]:
                uploads.append(op["b"])
        self.pairs = [(t.cpu().pin_memory(), t) for t in uploads]
        last = self.ops[-1]["out"]
        self.hout = torch.empty(last.shape, dtype=torch.float32).pin_memory()
        self.h2d = sum(t.numel() * 2 for t in uploads)
        self.d2h = last.numel() * 4

    def _run(self, op, stream):
        L = self.L
        L.check(L.load().tb_matmul_plan_run(op["plan"], L.ptr(op["a"]), L.ptr(op["b"]), L.ptr(op["out"]),
                                            L.stream_ptr(stream)))

    def step(self, stream):
        for op in self.ops:
            self._run(op, stream)
        return len(self.ops)

    def e2e_inputs(self):
        return self.pairs

    def e2e_output(self, stream):
        self.hout.copy_(self.ops[-1]["out"], non_blocking=True)

    def check(self):
        """Sampled rows of every product (the first two rows of the first batch, the last row of
        the last batch) against the oracle's AccF32 loop, within 2 bf16 ULP of the expected value
        plus 2^-16 of the row's sum of |a*b| (the accumulation order differs)."""
        from tests import helpers as H
        from oracle import oracle as O
        for op in self.ops:
            n, h, c, w = op["shape"]
            for bi, r0, nr in ((0, 0, 2), (n - 1, h - 1, 1)):
                a = op["a"][bi:bi + 1, r0:r0 + nr].float().cpu().numpy()
                b = op["b"][bi:bi + 1].float().cpu().numpy()
                want = H.oracle_matmul_float(a, b, O.D["FP32"])
                got = op["out"][bi:bi + 1, r0:r0 + nr].cpu().numpy()
                ok, _ = H.float_matmul_within_tolerance(got, want, a, b)
                if not ok:
                    return False
        return True

    def kernel_time(self, stream, flush, steps):
        """CUDA-event time of every GEMM launch of the step (the step is five launches of the
        tensor-core kernel): achieved = the step's FLOPs / their summed time."""
        torch = self.torch
        evs = []
        for _ in range(steps):
            flush.fill_(1)
            for op in self.ops:
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                self._run(op, stream)
                e.record(stream)
                evs.append((s, e))
        torch.cuda.synchronize()
        tot = sum(s.elapsed_time(e) for s, e in evs)
        return self.flops * steps / (tot * 1e-3) / 1e12, "TFLOP/s (bf16)", tot / len(evs), len(self.ops)

    def peak(self, torch):
        peaks = _measured_peaks()
        if peaks.get("bf16_tflops_sustained"):
            return float(peaks["bf16_tflops_sustained"]), "MEASURED_PEAKS.json bf16_tflops_sustained (of measured)"
        return 1400.0, "fallback 1.4 PFLOP/s sustained bf16 (of fallback)"

    def close(self):
        for op in getattr(self, "ops", []):
            if op["plan"] is not None:
                self.L.load().tb_matmul_plan_destroy(op["plan"])
                op["plan"] = None

    # -- CPU (oracle restatement): rows of the QKV product
    def cpu_prepare(self):
        """Seeded operands of the QKV product on the host (outside the timed CPU region)."""
        if not hasattr(self, "_cpu_ab"):
            from tests import helpers as H
            g = np.random.default_rng(self.seed)
            a = g.standard_normal((1, 512, 4096), dtype=np.float32)
            b = g.standard_normal((1, 4096, 12288), dtype=np.float32) * np.float32(0.02)
            self._cpu_ab = (H.bf16_round(a), H.bf16_round(b))

    def cpu_run(self, rows, threads):
        from oracle import oracle as O
        self.cpu_prepare()
        a, b = self._cpu_ab
        rows = min(rows, a.shape[1])
        a = np.ascontiguousarray(a[:, :rows])
        out = np.zeros(rows * 12288, dtype=np.float32)
        p = lambda x: x.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        if threads > 1:
            O.lib().orc_matmul_float_mt(ctypes.c_int64(1), ctypes.c_int64(rows), ctypes.c_int64(4096),
                                        ctypes.c_int64(12288), p(a), p(b), ctypes.c_int(O.D["FP32"]), p(out),
                                        ctypes.c_int(threads))
        else:
            O.lib().orc_matmul_float(ctypes.c_int64(1), ctypes.c_int64(rows), ctypes.c_int64(4096),
                                     ctypes.c_int64(12288), p(a), p(b), ctypes.c_int(O.D["FP32"]), p(out))
        return 2 * rows * 4096 * 12288 / 1e12

    def cpu_default(self, args):
        return 32  # about 16 s of single-core work

    def ref_default(self, args):
        return 2 * (os.cpu_count() or 1)

    def cpu_sample_desc(self, rows, threads):
        return (f"{rows} row(s) of the QKV product [rows,4096] x [4096,12288] (bf16 operands, AccF32), "
                f"{threads} thread(s), C restatement of the reference loops")


def _measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


WORKLOADS = {"matmul": MatmulWorkload, "resnet50": ResNet50Workload, "mobilenetv2": MobileNetV2Workload,
             "conv1": Conv1Workload, "bf16": Bf16Workload}


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


def load_traffic(workload):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload)
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
    sample = args.ref_sample or wl.ref_default(args)
    if hasattr(wl, "cpu_prepare"):
        wl.cpu_prepare()
    for _ in range(args.warmup):
        wl.cpu_run(sample, threads)
    t0 = time.perf_counter()
    units = 0.0
    for _ in range(args.steps):
        units += wl.cpu_run(sample, threads)
    dt = time.perf_counter() - t0
    value = units / dt
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": wl.unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": getattr(wl, "dtype", "int8"),
            "data": "synthetic", "config": wl.config(),
            "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
                             "sample": wl.cpu_sample_desc(sample, threads)},
            "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    if hasattr(wl, "close"):
        wl.close()
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
    from tosa_b200 import parallel as P

    ctx = L.Context(local)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    wl.setup(L, ctx, torch, stream)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def barrier():
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        wl.step(stream)
    ctx.synchronize(stream)
    ok = wl.check()
    if not ok:
        # a throughput of wrong results is no result: report the mismatch and stop
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": None, "unit": wl.unit, "n_gpus": ws,
                              "parity_spot_check": False, "config": wl.config(),
                              "error": "device results differ from the oracle on the spot-checked outputs"}),
                  flush=True)
        wl.close()
        ctx.close()
        if ws > 1:
            torch.distributed.destroy_process_group()
        return 1

    def timed(fn):
        evs = []
        launches = 0
        barrier()
        for _ in range(args.steps):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            launches += fn(stream) or 0
            e.record(stream)
            evs.append((s, e))
        barrier()
        ms = P.max_over_ranks(sum(s.elapsed_time(e) for s, e in evs))
        return ms, launches

    def soak(seconds):
        # keeps the GPU busy with the same step so the clock samples see load
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            for _ in range(10):
                wl.step(stream)
            torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    soak(0.6)
    ms, launches = timed(wl.step)
    soak(0.6)
    clk = clocks.stop()
    ctx.synchronize(stream)

    def timed_e2e(steps):
        # double-buffered uploads: step i+1's inputs copy on copy_stream into stage[(i+1) % 2]
        # while step i computes; each step starts by moving its staged inputs to the bound
        # device buffers on the compute stream
        pairs = wl.e2e_inputs()
        copy_stream = torch.cuda.Stream()
        stage = [[torch.empty_like(d) for _, d in pairs] for _ in range(2)]
        copied = [torch.cuda.Event() for _ in range(2)]
        moved = [torch.cuda.Event() for _ in range(2)]

        def upload(i):
            k = i % 2
            copy_stream.wait_event(moved[k])  # stage k's previous inputs have been moved
            with torch.cuda.stream(copy_stream):
                for (h, _), sb in zip(pairs, stage[k]):
                    sb.copy_(h, non_blocking=True)
            copied[k].record(copy_stream)

        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        flushes = []
        start.record(stream)
        copy_stream.wait_event(start)
        upload(0)
        for i in range(steps):
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            flush.fill_(1)
            f1.record(stream)
            flushes.append((f0, f1))
            k = i % 2
            stream.wait_event(copied[k])
            for (_, d), sb in zip(pairs, stage[k]):
                d.copy_(sb, non_blocking=True)
            moved[k].record(stream)
            if i + 1 < steps:
                upload(i + 1)
            wl.step(stream)
            wl.e2e_output(stream)
        end.record(stream)
        barrier()
        return P.max_over_ranks(start.elapsed_time(end) - sum(a.elapsed_time(b) for a, b in flushes))

    timed_e2e(args.warmup)
    ms_e2e = timed_e2e(args.steps)
    ctx.synchronize(stream)

    # roofline: the dominant kernel timed on its own stream with CUDA events
    peak = peak_src = achieved = kunit = kms = None
    if rank == 0:
        achieved, kunit, kms, _ = wl.kernel_time(stream, flush, max(3, min(args.steps, 10)))
        del flush
        peak, peak_src = wl.peak(torch) if hasattr(wl, "peak") else measure_int8_peak(torch)

    value = ws * wl.units_per_step * args.steps / (ms * 1e-3)
    e2e = ws * wl.units_per_step * args.steps / (ms_e2e * 1e-3)
    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu:
            sample = args.cpu_sample or wl.cpu_default(args)
            if hasattr(wl, "cpu_prepare"):
                wl.cpu_prepare()
            t0 = time.perf_counter()
            done = wl.cpu_run(sample, 1)
            dt = time.perf_counter() - t0
            cpu = {"value": done / dt, "unit": wl.unit, "cores": 1, "kind": "port",
                   "sample": wl.cpu_sample_desc(sample, 1)}
        line = {
            "metric": METRIC, "value": value, "unit": wl.unit, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": getattr(wl, "dtype", "int8"), "data": "synthetic", "config": wl.config(),
            "parity_spot_check": bool(ok),
            "e2e": {"value": e2e, "unit": wl.unit, "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h,
                    "overlap": "step i+1's host-to-device upload (copy stream) during step i's compute"},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": kunit,
                         "frac": achieved / peak if peak else None, "traffic": load_traffic(wl.name),
                         "kernel": wl.kernel, "kernel_ms_per_launch": kms, "peak_source": peak_src,
                         "note": "achieved = algorithmic ops (2*MACs) of the dominant kernel's launches / "
                                 "their CUDA-event time in an eager run (kernel launches, not the CUDA-graph "
                                 "replay that `value` times), L2 flushed; clocks sampled during a 1.2 s soak of "
                                 "the same step around the timed region"},
            "cpu_baseline": cpu,
            "clocks": clk,
        }
        share = getattr(wl, "kernel_share", None)
        if share is not None:
            line["roofline"]["kernel_share_of_step"] = share
        print(json.dumps(line), flush=True)
    wl.close()
    ctx.close()
    if ws > 1:
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="resnet50", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="tosa_b200", choices=["tosa_b200", "reference"])
    ap.add_argument("--batch", type=int, default=0, help="images per GPU for the graph workloads (default 64)")
    ap.add_argument("--cpu-rows", type=int, default=1536, help="rows of the single-thread CPU baseline sample")
    ap.add_argument("--ref-rows", type=int, default=1024, help="rows per step of the --impl reference arm")
    ap.add_argument("--cpu-sample", type=int, default=0, help="override the CPU baseline sample size")
    ap.add_argument("--ref-sample", type=int, default=0, help="override the reference arm's per-step sample")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl = WORKLOADS[args.workload](args)
    if args.impl == "reference":
        return run_reference(args, wl)
    return run_gpu(args, wl)


if __name__ == "__main__":
    sys.exit(main())
