"""Synthetic quantized TOSA graphs of the benchmark configurations.

The reference ships no model files; these builders write seeded `.tosa`
graphs with the shapes of BASELINE configs 3 (MobileNetV2-shaped, int8) and 4
(ResNet-50-shaped, int8), plus small residual graphs for the tests. Weights
are uniform int8 in [-127, 127], biases calibrated int32, zero points uniform
in [-8, 8] (the ResNet-50 graph keeps weight zero points at 0). Every contraction is followed by a per-channel RESCALE (scale32,
double rounding) to int8 and a CLAMP; residual additions follow the quantized
pattern RESCALE(int8 -> int32) of both branches, ADD (int32), RESCALE
(int32 -> int8), CLAMP.

Multipliers, shifts and biases are calibrated on one seeded image so the
int8 activations stay in range rather than saturating: the builder carries a
float64 shadow of every activation for that image (numpy convolutions of the
same weights); for each output channel the bias cancels the accumulator's
mean over the image (plus uniform noise of +-1024) and the RESCALE scale maps
its standard deviation to 24 int8 steps, written as a multiplier in
[2^30, 2^31) and the matching shift. The shadow only picks constants; the
graph itself is exact integer TOSA.
"""

from __future__ import annotations

import math

import numpy as np

from . import tosa_graph as TG

D = TG.DTYPE


class GraphBuilder:
    def __init__(self, seed: int, batch: int, weight_zp: bool = True):
        self.rng = np.random.default_rng(seed)
        self.weight_zp = weight_zp  # draw weight zero points (else symmetric weights, zero point 0)
        self.batch = batch
        self.ops: list = []
        self.tensors: dict = {}
        self.inputs: list = []
        self.outputs: list = []
        self.n = 0
        self.macs = 0           # contraction multiply-accumulates of the whole graph
        self.dw_macs = 0        # of which depthwise
        self.cal_rng = np.random.default_rng(seed + 1000)
        self.sh = {}            # tensor -> float64 shadow [H, W, C] of the calibration image
        self.op_macs = {}       # operator index -> multiply-accumulates (contractions)

    # -- tensors -------------------------------------------------------------------------
    def _name(self, p):
        self.n += 1
        return f"{p}_{self.n}"

    def _tensor(self, name, shape, dtype, data=None):
        self.tensors[name] = TG.TensorDef(name, list(shape), dtype, data)
        return name

    def input(self, name, shape, dtype=D["INT8"]):
        self._tensor(name, shape, dtype)
        self.inputs.append(name)
        self.sh[name] = self.cal_rng.integers(-128, 128, shape[1:]).astype(np.float64)
        return name

    def const(self, arr, dtype, prefix="c"):
        name = self._name(prefix)
        a = np.ascontiguousarray(arr)
        if dtype == D["SHAPE"]:
            data = a.astype("<i8").tobytes()
            self.tensors[name] = TG.TensorDef(name, [a.size], dtype, data)
            self.ops.append(TG.Operator(op=TG.OP["CONST_SHAPE"], inputs=[], outputs=[name]))
            return name
        store = {D["INT8"]: "<i1", D["INT16"]: "<i2", D["INT32"]: "<i4", D["FP32"]: "<f4"}[dtype]
        self._tensor(name, a.shape, dtype, a.astype(store).tobytes())
        self.ops.append(TG.Operator(op=TG.OP["CONST"], inputs=[], outputs=[name]))
        return name

    def scalar(self, v, dtype):
        return self.const(np.array([v]), dtype, "zp")

    def shape(self, name):
        return self.tensors[name].shape

    def zp(self):
        return int(self.rng.integers(-8, 9))

    # -- operators -----------------------------------------------------------------------
    @staticmethod
    def same_pads(size, k, stride):
        """TF 'SAME' padding: out = ceil(size / stride); the extra row/column goes
        after, which also makes (size - 1 + pads - (k - 1)) divide exactly, as
        the TOSA extent rule requires."""
        out = -(-size // stride)
        total = max((out - 1) * stride + k - size, 0)
        return total // 2, total - total // 2, out

    def conv(self, x, x_zp, oc, k, stride=1, depthwise=False):
        n, ih, iw, ic = self.shape(x)
        pt, pb, oh = self.same_pads(ih, k, stride)
        pl, pr, ow = self.same_pads(iw, k, stride)
        assert (ih - 1 + pt + pb - (k - 1)) % stride == 0 and (iw - 1 + pl + pr - (k - 1)) % stride == 0
        w_zp = self.zp() if self.weight_zp else 0
        if depthwise:
            w = self.rng.integers(-127, 128, (k, k, ic, 1), dtype=np.int8)
            oc = ic
            kk = k * k
        else:
            w = self.rng.integers(-127, 128, (oc, k, k, ic), dtype=np.int8)
            kk = k * k * ic
        acc = self._shadow_conv(self.sh[x] - x_zp, w.astype(np.float64) - w_zp, (pt, pb, pl, pr), stride, depthwise)
        noise = self.rng.integers(-1024, 1025, oc)
        bias = np.clip(np.round(-acc.mean(axis=(0, 1))) + noise, -2 ** 31, 2 ** 31 - 1).astype(np.int32)
        acc = acc + bias
        out = self._name("acc")
        self._tensor(out, [n, oh, ow, oc], D["INT32"])
        op = "DEPTHWISE_CONV2D" if depthwise else "CONV2D"
        self.ops.append(TG.Operator(op=TG.OP[op], inputs=[
            x, self.const(w, D["INT8"], "w"), self.const(bias, D["INT32"], "b"), self.scalar(x_zp, D["INT8"]),
            self.scalar(w_zp, D["INT8"])], outputs=[out],
            attr={"pad": [pt, pb, pl, pr], "stride": [stride] * 2, "dilation": [1, 1], "local_bound": False,
                  "acc_type": D["INT32"]}))
        macs = n * oh * ow * oc * kk
        self.op_macs[len(self.ops) - 1] = macs
        self.macs += macs
        if depthwise:
            self.dw_macs += macs
        self.sh[out] = acc
        return out

    @staticmethod
    def _shadow_conv(x, w, pads, stride, depthwise):
        """float64 convolution of one HWC image (OHWI or [KH,KW,C,1] weights)."""
        pt, pb, pl, pr = pads
        xp = np.pad(x, ((pt, pb), (pl, pr), (0, 0)))
        k = w.shape[0] if depthwise else w.shape[1]
        win = np.lib.stride_tricks.sliding_window_view(xp, (k, k), axis=(0, 1))[::stride, ::stride]
        # win: [OH, OW, C, KH, KW]
        if depthwise:
            return np.einsum("hwcij,ijc->hwc", win, w[..., 0], optimize=True)
        oh, ow = win.shape[:2]
        cols = win.transpose(0, 1, 3, 4, 2).reshape(oh * ow, -1)       # (ky, kx, c) order
        return (cols @ w.reshape(w.shape[0], -1).T).reshape(oh, ow, -1)

    def matmul(self, a, a_zp, b_arr):
        n, h, c = self.shape(a)
        w = b_arr.shape[2]
        b_zp = self.zp() if self.weight_zp else 0
        out = self._name("mm")
        self._tensor(out, [n, h, w], D["INT32"])
        self.ops.append(TG.Operator(op=TG.OP["MATMUL"], inputs=[
            a, self.const(b_arr, D["INT8"], "fc"), self.scalar(a_zp, D["INT8"]), self.scalar(b_zp, D["INT8"])],
            outputs=[out]))
        self.op_macs[len(self.ops) - 1] = n * h * w * c
        self.macs += n * h * w * c
        return out

    def _mult_shift(self, scale, channels):
        m, s = [], []
        for sc in np.broadcast_to(np.asarray(scale, np.float64), (channels,)):
            e = math.frexp(sc)[1]          # sc = f * 2^e with f in [0.5, 1)
            shift = 31 - e                 # m = sc * 2^shift in [2^30, 2^31)
            mult = int(round(sc * 2.0 ** shift))
            if mult >= 1 << 31:
                mult >>= 1
                shift -= 1
            m.append(mult)
            s.append(shift)
        return np.array(m, np.int64), np.array(s, np.int64)

    def rescale(self, x, in_zp, out_dtype, out_zp, scale, per_channel=True, rounding="DOUBLE_ROUND"):
        shape = self.shape(x)
        in_dt = self.tensors[x].dtype
        ch = shape[-1] if per_channel else 1
        m, s = self._mult_shift(scale, ch)
        lo, hi = {D["INT8"]: (-128, 127), D["INT16"]: (-32768, 32767), D["INT32"]: (-2 ** 31, 2 ** 31 - 1)}[out_dtype]
        eff = m.astype(np.float64) * np.exp2(-s.astype(np.float64))
        out = self._name("q")
        self._tensor(out, shape, out_dtype)
        self.ops.append(TG.Operator(op=TG.OP["RESCALE"], inputs=[
            x, self.const(m, D["INT32"], "mult"), self.const(s.astype(np.int8), D["INT8"], "shift"),
            self.scalar(in_zp, in_dt), self.scalar(out_zp, out_dtype)], outputs=[out],
            attr={"scale32": True, "rounding_mode": TG.ROUNDING[rounding], "per_channel": per_channel,
                  "input_unsigned": False, "output_unsigned": False}))
        if x in self.sh:
            self.sh[out] = np.clip(np.round((self.sh[x] - in_zp) * eff) + out_zp, lo, hi)
        return out

    def clamp(self, x, lo, hi):
        out = self._name("act")
        self._tensor(out, self.shape(x), self.tensors[x].dtype)
        self.ops.append(TG.Operator(op=TG.OP["CLAMP"], inputs=[x], outputs=[out], attr={
            "min_val": np.array([lo], np.int8).tobytes(), "max_val": np.array([hi], np.int8).tobytes(),
            "nan_mode": TG.NAN_MODE["PROPAGATE"]}))
        if x in self.sh:
            self.sh[out] = np.clip(self.sh[x], lo, hi)
        return out

    def conv_block(self, x, x_zp, oc, k, stride=1, depthwise=False, relu=True, clamp=None):
        """CONV2D -> per-channel RESCALE -> int8 [-> CLAMP]; returns (tensor, zero point)."""
        acc = self.conv(x, x_zp, oc, k, stride, depthwise=depthwise)
        out_zp = self.zp()
        std = np.maximum(self.sh[acc].std(axis=(0, 1)), 1.0)
        q = self.rescale(acc, 0, D["INT8"], out_zp, 24.0 / std)
        if relu or clamp is not None:
            lo, hi = clamp if clamp is not None else (out_zp, 127)
            q = self.clamp(q, lo, hi)
        return q, out_zp

    def residual(self, a, a_zp, b, b_zp, relu=True, clamp=None, rounding="DOUBLE_ROUND"):
        """RESCALE(a), RESCALE(b) to int32 -> ADD -> RESCALE to int8 [-> CLAMP]."""
        ra = self.rescale(a, a_zp, D["INT32"], 0, 2.0 ** 10, per_channel=False, rounding="SINGLE_ROUND")
        rb = self.rescale(b, b_zp, D["INT32"], 0, 2.0 ** 10 * 0.9, per_channel=False, rounding="SINGLE_ROUND")
        s = self._name("sum")
        self._tensor(s, self.shape(a), D["INT32"])
        self.ops.append(TG.Operator(op=TG.OP["ADD"], inputs=[ra, rb], outputs=[s]))
        self.sh[s] = self.sh[ra] + self.sh[rb]
        out_zp = self.zp()
        centre = self.sh[s].mean(axis=(0, 1))
        spread = max(float(np.sqrt(((self.sh[s] - centre) ** 2).mean() + (centre ** 2).mean())), 1.0)
        q = self.rescale(s, 0, D["INT8"], out_zp, 24.0 / spread, per_channel=False, rounding=rounding)
        if relu or clamp is not None:
            lo, hi = clamp if clamp is not None else (out_zp, 127)
            q = self.clamp(q, lo, hi)
        return q, out_zp

    def max_pool(self, x, k, stride):
        n, ih, iw, c = self.shape(x)
        pt, pb, oh = self.same_pads(ih, k, stride)
        pl, pr, ow = self.same_pads(iw, k, stride)
        out = self._name("pool")
        self._tensor(out, [n, oh, ow, c], self.tensors[x].dtype)
        self.ops.append(TG.Operator(op=TG.OP["MAX_POOL2D"], inputs=[x], outputs=[out], attr={
            "kernel": [k, k], "stride": [stride, stride], "pad": [pt, pb, pl, pr],
            "nan_mode": TG.NAN_MODE["PROPAGATE"]}))
        xp = np.pad(self.sh[x], ((pt, pb), (pl, pr), (0, 0)), constant_values=-np.inf)
        win = np.lib.stride_tricks.sliding_window_view(xp, (k, k), axis=(0, 1))[::stride, ::stride]
        self.sh[out] = win.max(axis=(3, 4))
        return out

    def avg_pool(self, x, x_zp, k, stride=1):
        n, ih, iw, c = self.shape(x)
        out_zp = x_zp
        out = self._name("gap")
        self._tensor(out, [n, (ih - k) // stride + 1, (iw - k) // stride + 1, c], self.tensors[x].dtype)
        self.ops.append(TG.Operator(op=TG.OP["AVG_POOL2D"], inputs=[
            x, self.scalar(x_zp, D["INT8"]), self.scalar(out_zp, D["INT8"])], outputs=[out], attr={
            "kernel": [k, k], "stride": [stride, stride], "pad": [0, 0, 0, 0], "acc_type": D["INT32"]}))
        win = np.lib.stride_tricks.sliding_window_view(self.sh[x], (k, k), axis=(0, 1))[::stride, ::stride]
        self.sh[out] = np.round(win.mean(axis=(3, 4)))
        return out, out_zp

    def reshape(self, x, shape):
        out = self._name("flat")
        self._tensor(out, shape, self.tensors[x].dtype)
        self.ops.append(TG.Operator(op=TG.OP["RESHAPE"], inputs=[x, self.const(np.array(shape), D["SHAPE"], "shape")],
                                    outputs=[out]))
        return out

    def build(self) -> bytes:
        blk = TG.Block(name="main", operators=self.ops, tensors=list(self.tensors.values()), inputs=self.inputs,
                       outputs=self.outputs)
        return TG.write_graph(TG.Graph(regions=[("main", [blk])]))


def resnet50_int8(batch: int, seed: int = 4, image: int = 224, classes: int = 1000):
    """stem CONV2D 7x7/s2, MAX_POOL2D 3x3/s2, bottleneck stages
    [3, 4, 6, 3] with widths 64/128/256/512 (x4 out), RESCALE+CLAMP after every
    conv, residual ADD, AVG_POOL2D 7x7, 2048 -> 1000 MATMUL (int32 logits).
    Padding is TF 'SAME'; the strided projection shortcut is AVG_POOL2D 2x2/s2
    followed by a 1x1 CONV2D. Weights are symmetric (zero point 0, as int8
    classifiers quantize them); activation zero points are drawn from [-8, 8].
    Returns (graph bytes, info dict)."""
    g = GraphBuilder(seed, batch, weight_zp=False)
    x = g.input("images", [batch, image, image, 3])
    x_zp = g.zp()
    # the stem conv has 3 input channels: pad 3
    y, zp = g.conv_block(x, x_zp, 64, 7, stride=2)
    y = g.max_pool(y, 3, 2)
    in_c = 64
    for stage, (blocks, width) in enumerate(zip([3, 4, 6, 3], [64, 128, 256, 512])):
        for i in range(blocks):
            stride = 2 if (i == 0 and stage > 0) else 1
            a, za = g.conv_block(y, zp, width, 1)
            a, za = g.conv_block(a, za, width, 3, stride=stride)
            a, za = g.conv_block(a, za, width * 4, 1, relu=False)
            if i == 0:
                # projection; strided as AVG_POOL2D 2x2/s2 + 1x1 CONV2D (a 1x1 stride-2 CONV2D of an
                # even extent breaks TOSA's exact-extent rule), the same MACs as a strided 1x1
                src, sz = (g.avg_pool(y, zp, 2, 2) if stride == 2 else (y, zp))
                skip, zs = g.conv_block(src, sz, width * 4, 1, relu=False)
            else:
                skip, zs = y, zp
            y, zp = g.residual(a, za, skip, zs)
            in_c = width * 4
    p, pz = g.avg_pool(y, zp, g.shape(y)[1])
    f = g.reshape(p, [1, batch, in_c])
    fc = g.rng.integers(-127, 128, (1, in_c, classes), dtype=np.int8)
    logits = g.matmul(f, pz, fc)
    g.outputs.append(logits)
    return g.build(), {"macs": g.macs, "ops_per_image": 2 * g.macs / batch, "batch": batch, "input": "images",
                       "output": logits, "n_ops": len(g.ops), "op_macs": g.op_macs}


def mobilenetv2_int8(batch: int, seed: int = 3, image: int = 224, classes: int = 1000):
    """stem CONV2D 3x3/s2 (3 -> 32), 17 inverted-residual blocks
    (1x1 CONV2D expand x6, 3x3 DEPTHWISE_CONV2D stride 1/2, 1x1 CONV2D project,
    each followed by per-channel RESCALE and CLAMP[0,127]; residual ADD via
    RESCALE to int32 where stride is 1 and channels match), 1x1 CONV2D to 1280,
    AVG_POOL2D 7x7, 1280 -> 1000 MATMUL. Returns (graph bytes, info dict)."""
    g = GraphBuilder(seed, batch)
    x = g.input("images", [batch, image, image, 3])
    x_zp = g.zp()
    y, zp = g.conv_block(x, x_zp, 32, 3, stride=2, clamp=(0, 127))
    c = 32
    for t, cout, n, s in [(6, 16, 1, 1), (6, 24, 2, 2), (6, 32, 3, 2), (6, 64, 4, 2), (6, 96, 3, 1),
                          (6, 160, 3, 2), (6, 320, 1, 1)]:
        for i in range(n):
            stride = s if i == 0 else 1
            e, ze = g.conv_block(y, zp, c * t, 1, clamp=(0, 127))
            d, zd = g.conv_block(e, ze, c * t, 3, stride=stride, depthwise=True, clamp=(0, 127))
            p, zpj = g.conv_block(d, zd, cout, 1, clamp=(0, 127))
            if stride == 1 and c == cout:
                y, zp = g.residual(p, zpj, y, zp, clamp=(0, 127))
            else:
                y, zp = p, zpj
            c = cout
    y, zp = g.conv_block(y, zp, 1280, 1, clamp=(0, 127))
    p, pz = g.avg_pool(y, zp, g.shape(y)[1])
    f = g.reshape(p, [1, batch, 1280])
    fc = g.rng.integers(-127, 128, (1, 1280, classes), dtype=np.int8)
    logits = g.matmul(f, pz, fc)
    g.outputs.append(logits)
    return g.build(), {"macs": g.macs, "dw_macs": g.dw_macs, "ops_per_image": 2 * g.macs / batch, "batch": batch,
                       "input": "images", "output": logits, "n_ops": len(g.ops), "op_macs": g.op_macs}


def residual_block_int8(batch: int = 2, hw: int = 14, c: int = 64, seed: int = 7):
    """A small graph with every fusion pattern: CONV2D+RESCALE+CLAMP, the
    residual chain with and without CLAMP, DEPTHWISE, MAX_POOL2D, AVG_POOL2D,
    RESHAPE and an int8 MATMUL with both zero points."""
    g = GraphBuilder(seed, batch)
    x = g.input("x", [batch, hw, hw, c])
    xz = g.zp()
    a, za = g.conv_block(x, xz, c, 3)
    b, zb = g.conv_block(a, za, c, 1, relu=False)
    y, zy = g.residual(b, zb, x, xz)
    d, zd = g.conv_block(y, zy, c, 3, depthwise=True)
    y2, zy2 = g.residual(d, zd, y, zy, relu=False)
    m = g.max_pool(y2, 3, 2)
    p, pz = g.avg_pool(m, zy2, g.shape(m)[1])
    f = g.reshape(p, [1, batch, c])
    fc = g.rng.integers(-127, 128, (1, c, 16), dtype=np.int8)
    out = g.matmul(f, pz, fc)
    g.outputs.append(out)
    g.outputs.append(y)
    return g.build(), {"macs": g.macs, "input": "x", "outputs": [out, y]}
