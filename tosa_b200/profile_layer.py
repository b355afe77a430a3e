"""Run one layer of the hot path a few times with nothing else around it: a target for a
profiler (and a quick timing with CUDA events).

    python -m tosa_b200.profile_layer conv N HW IC OC K [--runs 5]
    python -m tosa_b200.profile_layer depthwise N HW C K STRIDE [--runs 5]
    python -m tosa_b200.profile_layer residual N HW C [--runs 5]
    python -m tosa_b200.profile_layer matmul_t N H C W D [--runs 5]

conv: int8 CONV2D (square HW x HW input, K x K window, stride 1 or --stride, "same" padding,
input zero point -3 or --zx) with a fused per-channel RESCALE (double rounding) + CLAMP to int8,
planned once with tb_conv2d_plan_create and run through tb_conv2d_plan_run.
depthwise: the same for DEPTHWISE_CONV2D (channel multiplier 1, weight zero point 2,
stride 1 or 2) through tb_depthwise_conv2d_plan_create.
residual: one residual chain (two int8 inputs [N, HW, HW, C] -> RESCALE to int32 each,
ADD, RESCALE to int8, CLAMP) built with graphs.GraphBuilder and run by the graph runner.
matmul_t: int8 MATMUL_T a [N,H,C] x b [D,W,C] (D = N, or 1 shared by every batch), zero points
-3 / 2, through tb_matmul_t_plan_create and tb_matmul_plan_run; also prints int8 TOPS (2*N*H*W*C).
Inputs are seeded uniform int8. The mean time of the runs after the first two is printed.
"""

from __future__ import annotations

import argparse
import ctypes

import numpy as np


def _time(run, runs, torch):
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for i in range(runs):
        if i == min(2, runs - 1):
            ev[0].record()
        run()
    ev[1].record()
    torch.cuda.synchronize()
    timed = runs - min(2, runs - 1)
    return ev[0].elapsed_time(ev[1]) / timed * 1000.0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("kind", choices=["conv", "depthwise", "residual", "matmul_t"])
    ap.add_argument("dims", type=int, nargs="+")
    ap.add_argument("--runs", type=int, default=5)
    ap.add_argument("--zx", type=int, default=-3, help="input zero point of conv (default -3)")
    ap.add_argument("--stride", type=int, default=1, help="stride of conv (default 1)")
    args = ap.parse_args(argv)

    import torch

    from . import _lib as L

    lib = L.load()
    ctx = L.Context(0)
    rng = np.random.default_rng(2)
    if args.kind == "conv":
        n, hw, ic, oc, k = args.dims
        st = args.stride
        # "same" padding (the graphs' rule: the extra row and column at the bottom and right)
        tot = max((-(-hw // st) - 1) * st + k - hw, 0)
        pad = (tot // 2, tot - tot // 2) * 2
        pad = (pad[0], pad[1], pad[0], pad[1])
        d = L.conv_desc(n, hw, hw, ic, oc, k, k, pad, (st, st), (1, 1), L.DT_INT8, L.DT_INT8, L.DT_INT32,
                        L.DT_INT32, input_zp=args.zx)
        w = torch.from_numpy(rng.integers(-127, 128, (oc, k, k, ic), dtype=np.int8)).cuda()
        bias = torch.from_numpy(rng.integers(-30000, 30000, oc).astype(np.int32)).cuda()
        at = L.rescale_attr(rng.integers(1 << 30, (1 << 31) - 1, oc), rng.integers(36, 40, oc),
                            rounding=L.ROUND_DOUBLE, per_channel=True, output_zp=3, out_dtype=L.DT_INT8,
                            clamp=(3, 127))
        h = ctypes.c_void_p()
        L.check(lib.tb_conv2d_plan_create(ctx.h, d, L.ptr(w), L.ptr(bias), at, ctypes.byref(h)))
        oh, ow = L.conv_out_hw(hw, hw, k, k, pad, (st, st), (1, 1))
        x = torch.from_numpy(rng.integers(-128, 128, (n, hw, hw, ic), dtype=np.int8)).cuda()
        o = torch.empty((n, oh, ow, oc), dtype=torch.int8, device="cuda")
        us = _time(lambda: L.check(lib.tb_conv2d_plan_run(h, L.ptr(x), L.ptr(o), L.stream_ptr())), args.runs, torch)
        lib.tb_conv2d_plan_destroy(h)
        print(f"conv {n}x{hw}x{hw}x{ic}->{oc} k{k}" + (f" s{st}" if st > 1 else "") + f": {us:.1f} us")
    elif args.kind == "depthwise":
        n, hw, c, k, st = args.dims
        p = k // 2
        pads = (p, p, p, p) if st == 1 else (p - 1, p, p - 1, p)
        d = L.conv_desc(n, hw, hw, c, c, k, k, pads, (st, st), (1, 1), L.DT_INT8, L.DT_INT8, L.DT_INT32,
                        L.DT_INT32, -3, 2, c, 1)
        oh, ow = L.conv_out_hw(hw, hw, k, k, pads, (st, st), (1, 1))
        w = torch.from_numpy(rng.integers(-127, 128, (k, k, c, 1), dtype=np.int8)).cuda()
        bias = torch.from_numpy(rng.integers(-30000, 30000, c).astype(np.int32)).cuda()
        at = L.rescale_attr(rng.integers(1 << 30, (1 << 31) - 1, c), rng.integers(36, 40, c),
                            rounding=L.ROUND_DOUBLE, per_channel=True, output_zp=3, out_dtype=L.DT_INT8,
                            clamp=(3, 127))
        h = ctypes.c_void_p()
        L.check(lib.tb_depthwise_conv2d_plan_create(ctx.h, d, L.ptr(w), L.ptr(bias), at, ctypes.byref(h)))
        x = torch.from_numpy(rng.integers(-128, 128, (n, hw, hw, c), dtype=np.int8)).cuda()
        o = torch.empty((n, oh, ow, c), dtype=torch.int8, device="cuda")
        us = _time(lambda: L.check(lib.tb_conv2d_plan_run(h, L.ptr(x), L.ptr(o), L.stream_ptr())), args.runs, torch)
        lib.tb_conv2d_plan_destroy(h)
        print(f"depthwise {n}x{hw}x{hw}x{c} k{k} s{st}: {us:.1f} us")
    elif args.kind == "matmul_t":
        n, h, c, w, dd = args.dims
        desc = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32,
                            a_zp=-3, b_zp=2)
        h_ = ctypes.c_void_p()
        L.check(lib.tb_matmul_t_plan_create(ctx.h, desc, dd, None, ctypes.byref(h_)))
        a = torch.from_numpy(rng.integers(-128, 128, (n, h, c), dtype=np.int8)).cuda()
        b = torch.from_numpy(rng.integers(-128, 128, (dd, w, c), dtype=np.int8)).cuda()
        o = torch.empty((n, h, w), dtype=torch.int32, device="cuda")
        us = _time(lambda: L.check(lib.tb_matmul_plan_run(h_, L.ptr(a), L.ptr(b), L.ptr(o), L.stream_ptr())),
                   args.runs, torch)
        lib.tb_matmul_plan_destroy(h_)
        print(f"matmul_t [{n},{h},{c}]x[{dd},{w},{c}]: {us:.1f} us, {2.0 * n * h * w * c / us / 1e6:.1f} TOPS")
    else:
        from . import graphs
        from . import interpreter as I

        n, hw, c = args.dims
        shape = [n, hw, hw, c]
        g = graphs.GraphBuilder(5, n)
        a = g.input("x", shape)
        b = g.input("y", shape)
        q, _ = g.residual(a, -3, b, 6, relu=True)
        g.outputs.append(q)
        it = I.Interpreter(g.build(), context=ctx)
        keep = []
        for nm in ("x", "y"):
            t = torch.from_numpy(rng.integers(-128, 128, shape).astype(np.int8)).cuda()
            it.bind_device(nm, L.DT_INT8, shape, t.data_ptr())
            keep.append(t)
        stream = torch.cuda.current_stream()
        us = _time(lambda: it.execute(stream=stream), args.runs, torch)
        it.close()
        print(f"residual {shape}: {us:.1f} us per graph run")
    ctx.synchronize()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
