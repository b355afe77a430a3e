"""Run a benchmark workload's step a few times with nothing else around it
(no timing, no clock sampling, no CPU checks): the target for a profiler.

    python -m tosa_b200.profile_step [--workload resnet50|mobilenetv2] [--batch 64] [--steps 2]

Every step is one eager run of the graph runner over the synthetic graph
(tosa_b200/graphs.py) on cuda:0, so each kernel appears as its own launch in
the graph's operator order.
"""

from __future__ import annotations

import argparse

import numpy as np


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="resnet50", choices=["resnet50", "mobilenetv2"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--steps", type=int, default=2)
    args = ap.parse_args(argv)

    import torch

    from . import _lib as L
    from . import graphs
    from . import interpreter as I

    build = graphs.resnet50_int8 if args.workload == "resnet50" else graphs.mobilenetv2_int8
    data, info = build(args.batch)
    ctx = L.Context(0)
    it = I.Interpreter(data, context=ctx)
    images = np.random.default_rng(21).integers(-128, 128, (args.batch, 224, 224, 3), dtype=np.int8)
    dimg = torch.from_numpy(images).cuda()
    it.bind_device(info["input"], L.DT_INT8, list(images.shape), dimg.data_ptr())
    stream = torch.cuda.Stream()
    for _ in range(args.steps):
        it.execute(stream=stream)
    torch.cuda.synchronize()
    print(f"{args.workload} batch {args.batch}: {args.steps} step(s), {it.last_launches} launches per step")
    it.close()
    ctx.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
