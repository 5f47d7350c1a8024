"""The rec-latin recognizer with random weights: its layer shapes, the FP32 and
INT8 (Q/DQ) ONNX files the reference's executor reads, and a float forward pass
(numpy) used for calibration and for the FP16 tolerance checks.

Layer shapes follow the reference's model card (docs/MODELS.md:186-212, the
rec-latin table): a 3x3/2 stem to 32 channels; stages of 3x3 convolutions to 48
(stride 2), 96 (stride 2) and 160 (stride (2, 1)) channels, two a stage; a 2x3
collapse of the last two rows to 256 channels; two mixing blocks (depthwise 1x9,
1x1 to 512 with ReLU, 1x1 back to 256 plus the block's input) with a nearest 2x
upsample of the width between them; a 1x1 head to 800 classes, class 0 the CTC
blank.  Every block is a plain (folded) convolution with a bias, ReLU after the
backbone's and the collapse's and the mixing blocks' first 1x1.

The INT8 file mirrors the reference's own miniature Q/DQ fixture
(tests/data/native-rec.int8.onnx): per-output-channel symmetric int8 weights
(axis 0, zero points 0), uint8 activations with a per-tensor scale and zero point
(MinMax calibration on synthetic crops), a Q/DQ after every convolution, the
residual Add and the Resize (the Resize with its input's parameters), and the head's
output quantized before and after its Squeeze.
"""
from __future__ import annotations

import numpy as np

from . import netdef
from . import onnx_pb as pb

# (name, cin, cout, kh, kw, sh, sw, pads (t, l, b, r), relu)
BACKBONE = [
    ("stem", 1, 32, 3, 3, 2, 2, (1, 1, 1, 1), True),
    ("s1a", 32, 48, 3, 3, 2, 2, (1, 1, 1, 1), True),
    ("s1b", 48, 48, 3, 3, 1, 1, (1, 1, 1, 1), True),
    ("s2a", 48, 96, 3, 3, 2, 2, (1, 1, 1, 1), True),
    ("s2b", 96, 96, 3, 3, 1, 1, (1, 1, 1, 1), True),
    ("s3a", 96, 160, 3, 3, 2, 1, (1, 1, 1, 1), True),
    ("s3b", 160, 160, 3, 3, 1, 1, (1, 1, 1, 1), True),
    ("collapse", 160, 256, 2, 3, 1, 1, (0, 1, 0, 1), True),
]
MIX_C, MIX_HIDDEN, CLASSES, HEIGHT = 256, 512, 800, 32
BLANK_BIAS = 4.75  # class 0's bias: about four frames in five blank, as a trained CTC recognizer gives them


def make_weights(seed: int = 0, classes: int = CLASSES) -> dict[str, np.ndarray]:
    """He-normal weights (std sqrt(2 / fan_in)), small normal biases; the mixing blocks'
    last 1x1 at half gain so the residual stream stays bounded; the head wide enough
    that a frame's best class is well clear of the next (a trained head's margins)."""
    rng = np.random.default_rng(seed)
    w: dict[str, np.ndarray] = {}

    def conv(name, cin, cout, kh, kw, gain=1.0, groups=1, bias_std=0.05):
        fan_in = cin // groups * kh * kw
        w[name + ".w"] = (rng.standard_normal((cout, cin // groups, kh, kw)) * gain * np.sqrt(2.0 / fan_in)).astype(np.float32)
        w[name + ".b"] = (rng.standard_normal(cout) * bias_std).astype(np.float32)

    for name, cin, cout, kh, kw, *_ in BACKBONE:
        conv(name, cin, cout, kh, kw)
    for m in ("mix1", "mix2"):
        conv(m + ".dw", MIX_C, MIX_C, 1, 9, groups=MIX_C, gain=0.7)
        conv(m + ".up", MIX_C, MIX_HIDDEN, 1, 1)
        conv(m + ".down", MIX_HIDDEN, MIX_C, 1, 1, gain=0.5)
    conv("head", MIX_C, classes, 1, 1, gain=2.5, bias_std=0.5)
    w["head.b"][0] += BLANK_BIAS
    return w


# ----------------------------------------------------------------------------- graph building

class _Builder:
    def __init__(self, quant: dict[str, tuple[float, int]] | None, weights: dict[str, np.ndarray]):
        self.g = pb.Graph(name="rec-latin")
        self.quant = quant  # tensor name -> (scale, zero): INT8 Q/DQ file; None: FP32
        self.w = weights

    def init(self, name, a):
        self.g.initializers[name] = a
        return name

    def node(self, op, ins, outs, **attrs):
        self.g.nodes.append(pb.Node(op, ins, outs, outs[0], attrs))
        return outs[0]

    def qdq(self, t: str, params_of: str | None = None) -> str:
        """A Q then DQ on tensor t (its own calibrated parameters, or those of params_of)."""
        if self.quant is None:
            return t
        key = params_of or t
        s, z = self.quant[key]
        sn, zn = key + "_scale", key + "_zero_point"
        if sn not in self.g.initializers:
            self.init(sn, np.array(s, np.float32))
            self.init(zn, np.array(z, np.uint8))
        q = self.node("QuantizeLinear", [t, sn, zn], [t + "_QuantizeLinear_Output"])
        return self.node("DequantizeLinear", [q, sn, zn], [t + "_DequantizeLinear_Output"])

    def weight(self, name: str) -> str:
        w = self.w[name + ".w"]
        if self.quant is None:
            return self.init(name + ".w", w)
        amax = np.abs(w).reshape(w.shape[0], -1).max(axis=1)
        scale = (np.maximum(amax, 1e-12) / 127.0).astype(np.float32)
        q = np.clip(np.rint(w / scale[:, None, None, None]), -127, 127).astype(np.int8)
        self.init(name + ".w_quantized", q)
        self.init(name + ".w_scale", scale)
        self.init(name + ".w_zero_point", np.zeros(w.shape[0], np.int8))
        return self.node("DequantizeLinear", [name + ".w_quantized", name + ".w_scale", name + ".w_zero_point"],
                         [name + ".w_DequantizeLinear_Output"], axis=0)

    def conv(self, name, x, kh, kw, sh, sw, pads, relu, group=1, out=None):
        wn = self.weight(name)
        bn = self.init(name + ".b", self.w[name + ".b"])
        y = self.node("Conv", [x, wn, bn], [out or (name + (".relu" if relu else ".out"))],
                      dilations=[1, 1], group=group, kernel_shape=[kh, kw], pads=list(pads), strides=[sh, sw])
        if relu:
            # the Relu as a node of its own (the reference joins it to the convolution)
            pre = y
            self.g.nodes[-1].outputs = [name + ".conv"]
            self.g.nodes[-1].name = name + ".conv"
            y = self.node("Relu", [name + ".conv"], [pre])
        return y


def build_onnx(weights: dict[str, np.ndarray], quant: dict[str, tuple[float, int]] | None = None) -> pb.Model:
    """rec-latin as an ONNX model: FP32 (quant None) or INT8 Q/DQ with the given per-tensor parameters."""
    b = _Builder(quant, weights)
    classes = weights["head.w"].shape[0]
    x = b.qdq("x")
    for name, cin, cout, kh, kw, sh, sw, pads, relu in BACKBONE:
        x = b.qdq(b.conv(name, x, kh, kw, sh, sw, pads, relu))
    b.init("resize.scales", np.array([1, 1, 1, 2], np.float32))
    for m in ("mix1", "mix2"):
        inp = x
        d = b.qdq(b.conv(m + ".dw", inp, 1, 9, 1, 1, (0, 4, 0, 4), False, group=MIX_C))
        u = b.qdq(b.conv(m + ".up", d, 1, 1, 1, 1, (0, 0, 0, 0), True))
        dn = b.qdq(b.conv(m + ".down", u, 1, 1, 1, 1, (0, 0, 0, 0), False))
        s = b.node("Add", [dn, inp], [m + ".add"])
        x = b.qdq(s)
        if m == "mix1":
            r = b.node("Resize", [x, "", "resize.scales"], ["resize"], coordinate_transformation_mode="asymmetric",
                       mode="nearest", nearest_mode="floor")
            x = b.qdq(r, params_of=m + ".add")
    h = b.qdq(b.conv("head", x, 1, 1, 1, 1, (0, 0, 0, 0), False))
    b.init("axes", np.array([2], np.int64))
    sq = b.node("Squeeze", [h, "axes"], ["logits_pre" if quant else "logits"])
    if quant is not None:
        s, z = quant["head.out"]
        b.init("logits_scale", np.array(s, np.float32))
        b.init("logits_zero_point", np.array(z, np.uint8))
        q = b.node("QuantizeLinear", [sq, "logits_scale", "logits_zero_point"], ["logits_QuantizeLinear_Output"])
        b.node("DequantizeLinear", [q, "logits_scale", "logits_zero_point"], ["logits"])
    b.g.inputs = [pb.ValueInfo("x", pb.FLOAT, ["N", 1, HEIGHT, "W"])]
    b.g.outputs = [pb.ValueInfo("logits", pb.FLOAT, ["N", classes, "T"])]
    meta = {"carbon.crop.height": str(HEIGHT), "carbon.crop.pad_v": "0.2", "carbon.crop.pad_h": "0.3"}
    return pb.Model(b.g, 17, meta)


# ----------------------------------------------------------------------------- float forward

def _to_half(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float16).astype(np.float32)


def forward_float(net: netdef.RecNet, x: np.ndarray, half: bool = False, keep: bool = False):
    """A float forward pass of a compiled float network on x [N, 1, H, W] (ink values).
    half: weights and every tensor between layers rounded to FP16 (sums in FP32), as an
    FP16 engine keeps them.  Returns the output [N, classes, T] (and every value's
    tensor, NCHW float32, when keep)."""
    vals: dict[int, np.ndarray] = {net.inp: _to_half(x) if half else x.astype(np.float32)}
    for l in net.layers:
        a = vals[l.inp]
        if l.kind == netdef.KIND_RESIZE:
            y = np.repeat(np.repeat(a, l.fh, axis=2), l.fw, axis=3)
        else:
            w = _to_half(l.wf) if half else l.wf
            n, c, h, wd = a.shape
            ap = np.pad(a, ((0, 0), (0, 0), (l.pt, l.pb), (l.pl, l.pr)))
            oh = (h + l.pt + l.pb - l.kh) // l.sh + 1
            ow = (wd + l.pl + l.pr - l.kw) // l.sw + 1
            if l.kind == netdef.KIND_DW:
                y = np.zeros((n, c, oh, ow), np.float32)
                for ky in range(l.kh):
                    for kx in range(l.kw):
                        y += ap[:, :, ky:ky + l.sh * (oh - 1) + 1:l.sh, kx:kx + l.sw * (ow - 1) + 1:l.sw] * w[:, 0, ky, kx][None, :, None, None]
            else:
                cols = np.empty((n, oh, ow, c, l.kh, l.kw), np.float32)
                for ky in range(l.kh):
                    for kx in range(l.kw):
                        cols[:, :, :, :, ky, kx] = ap[:, :, ky:ky + l.sh * (oh - 1) + 1:l.sh,
                                                      kx:kx + l.sw * (ow - 1) + 1:l.sw].transpose(0, 2, 3, 1)
                y = cols.reshape(n * oh * ow, -1) @ w.reshape(l.cout, -1).T
                y = y.reshape(n, oh, ow, l.cout).transpose(0, 3, 1, 2)
            y = y + l.bias[None, :, None, None]
            if l.residual >= 0:
                r = vals[l.residual]
                if l.res_shift or l.res_fh > 1:
                    r = np.repeat(np.repeat(r, l.res_fh, axis=2), 1 << l.res_shift, axis=3)
                y = y + r
            if l.relu:
                y = np.maximum(y, 0)
        y = y.astype(np.float32)
        vals[l.out] = _to_half(y) if half and l.out != net.out else y
    out = vals[net.out]
    out = out.reshape(out.shape[0], out.shape[1], -1)
    return (out, vals) if keep else out


# ----------------------------------------------------------------------------- calibration

def calibrate(weights: dict[str, np.ndarray], crops: np.ndarray) -> dict[str, tuple[float, int]]:
    """MinMax uint8 parameters for every tensor the INT8 file quantizes, from a float run on
    crops [N, 32, W] uint8 (ink = 1 - p / 255): range widened to hold 0, scale = range / 255,
    zero point = round(-min / scale)."""
    fp = build_onnx(weights, None)
    net = netdef.compile_model(fp)
    x = (np.float32(1.0) - crops.astype(np.float32) / np.float32(255.0))[:, None]
    _, vals = forward_float(net, x, keep=True)
    # the float file's tensors by name, before fusion: rebuild from the compiled values by `last` names
    ranges: dict[str, tuple[float, float]] = {}
    for i, v in enumerate(net.values):
        a = vals[i]
        ranges[v.name] = (float(a.min()), float(a.max()))
        ranges[v.last] = ranges[v.name]
    # the pre-add 1x1s are fused away in the float graph: their own output ranges from their layer
    q: dict[str, tuple[float, int]] = {}

    def params(lo, hi):
        lo, hi = min(lo, 0.0), max(hi, 0.0)
        s = np.float32((hi - lo) / 255.0) if hi > lo else np.float32(1.0)
        z = int(np.clip(np.rint(-lo / float(s)), 0, 255))
        return float(s), z

    q["x"] = params(0.0, 1.0)
    for name, *_rest in BACKBONE:
        q[name + ".relu"] = params(*ranges[name + ".relu"])
    for m in ("mix1", "mix2"):
        q[m + ".dw.out"] = params(*ranges[m + ".dw.out"])
        q[m + ".up.relu"] = params(*ranges[m + ".up.relu"])
        q[m + ".add"] = params(*ranges[m + ".add"])
        q[m + ".down.out"] = q[m + ".add"]  # fused into the Add: never read
    q["head.out"] = params(*ranges["head.out"])
    return q


def synthetic_crops(rng: np.random.Generator, n: int, wmin: int = 96, wmax: int = 640, height: int = HEIGHT):
    """Config 1's crops: widths uniform in [wmin, wmax] rounded to 8, background ~N(230, 10),
    3-6 px dark strokes ~N(40, 15) at random positions.  Returns (list of [32, w] uint8)."""
    out = []
    for _ in range(n):
        w = int(np.clip(int(round(rng.uniform(wmin, wmax) / 8.0)) * 8, 8, None))
        c = rng.normal(230, 10, (height, w))
        for _ in range(int(w / 6)):
            sw = int(rng.integers(3, 7))
            x0 = int(rng.integers(0, max(1, w - sw)))
            y0 = int(rng.integers(4, height // 2))
            y1 = int(rng.integers(height // 2, height - 4))
            if rng.random() < 0.5:  # a vertical stroke
                c[y0:y1, x0:x0 + sw] = rng.normal(40, 15, (y1 - y0, min(sw, w - x0)))
            else:  # a horizontal one
                yy = int(rng.integers(6, height - 6))
                x1 = min(w, x0 + int(rng.integers(4, 14)))
                c[yy:yy + sw // 2 + 1, x0:x1] = rng.normal(40, 15, (sw // 2 + 1, x1 - x0))
        out.append(np.clip(np.rint(c), 0, 255).astype(np.uint8))
    return out


MINI_BACKBONE = [
    ("stem", 1, 8, 3, 3, 2, 2, (1, 1, 1, 1), True),
    ("s1a", 8, 12, 3, 3, 2, 2, (1, 1, 1, 1), True),
    ("s1b", 12, 12, 3, 3, 1, 1, (1, 1, 1, 1), True),
    ("s2a", 12, 16, 3, 3, 2, 2, (1, 1, 1, 1), True),
    ("s3a", 16, 20, 3, 3, 2, 1, (1, 1, 1, 1), True),
    ("collapse", 20, 24, 2, 3, 1, 1, (0, 1, 0, 1), True),
]


def make_mini(seed: int = 4, calib_lines: int = 16):
    """A miniature recognizer of the same family with channel counts that are not multiples of
    16 (8, 12, 16, 20, 24; mixing 24 -> 48 -> 24; 11 classes): (weights, quant, fp32, int8)."""
    global BACKBONE, MIX_C, MIX_HIDDEN
    saved = BACKBONE, MIX_C, MIX_HIDDEN
    BACKBONE, MIX_C, MIX_HIDDEN = MINI_BACKBONE, 24, 48
    try:
        w = make_weights(seed, classes=11)
        rng = np.random.default_rng(2000 + seed)
        crops = synthetic_crops(rng, calib_lines, 128, 128)
        quant = calibrate(w, np.stack(crops))
        return w, quant, build_onnx(w, None), build_onnx(w, quant)
    finally:
        BACKBONE, MIX_C, MIX_HIDDEN = saved


def make_rec_latin(seed: int = 0, calib_lines: int = 24):
    """(weights, quant params, fp32 ONNX model, int8 ONNX model) of rec-latin at `seed`."""
    w = make_weights(seed)
    rng = np.random.default_rng(1000 + seed)
    crops = synthetic_crops(rng, calib_lines, 256, 256)
    quant = calibrate(w, np.stack(crops))
    return w, quant, build_onnx(w, None), build_onnx(w, quant)


# ----------------------------------------------------------------------------- kernel sweep layers

def make_conv(c_in: int, c_out: int, height: int, seed: int = 0, stride: int = 1, relu: bool = False,
              calib_width: int = 64):
    """BASELINE.json config 4's layer: one 3x3 convolution, pad 1, stride (stride, stride), c_in -> c_out
    (He-normal weights and small biases from `seed`; a ReLU when asked), on inputs [N, c_in, height, W]:
    (fp32 ONNX, int8 Q/DQ ONNX, (input scale, input zero point)).  The INT8 file quantizes the
    input ~N(0, 1) per tensor and the output by MinMax over a float run on a seeded sample."""
    rng = np.random.default_rng(seed)
    std = np.sqrt(2.0 / (c_in * 9))
    w = {"conv.w": rng.normal(0.0, std, (c_out, c_in, 3, 3)).astype(np.float32),
         "conv.b": rng.normal(0.0, 0.05, c_out).astype(np.float32)}

    def build(quant):
        b = _Builder(quant, w)
        x = b.qdq("x")
        y = b.conv("conv", x, 3, 3, stride, stride, (1, 1, 1, 1), relu)
        out = y
        if quant is not None:
            # quantized inside the graph, then an Identity and the output's Q/DQ (as rec-latin's head
            # ends: its codes leave the network, not a float)
            b.node("Identity", [b.qdq(y)], ["y"])
            out = b.qdq("y", params_of=y)
        b.g.inputs = [pb.ValueInfo("x", pb.FLOAT, ["N", c_in, height, "W"])]
        b.g.outputs = [pb.ValueInfo(out, pb.FLOAT, ["N", c_out, "H", "W"])]
        return pb.Model(b.g, 17, {})

    fp = build(None)
    sample = rng.normal(0.0, 1.0, (2, c_in, height, calib_width)).astype(np.float32)
    out = forward_float(netdef.compile_model(fp), sample)

    def params(lo, hi):
        lo, hi = min(lo, 0.0), max(hi, 0.0)
        s = np.float32((hi - lo) / 255.0)
        return float(s), int(np.clip(np.rint(-lo / float(s)), 0, 255))

    yname = "conv.relu" if relu else "conv.out"
    quant = {"x": params(float(sample.min()), float(sample.max())), yname: params(float(out.min()), float(out.max()))}
    return fp, build(quant), quant["x"]


def make_head(k: int, classes: int, w: np.ndarray, b: np.ndarray, sample: np.ndarray):
    """BASELINE.json config 4's head: one 1x1 convolution, k -> classes, with the given weights
    [classes, k] and biases [classes], on inputs [N, k, 1, W]: (fp32 ONNX, int8 Q/DQ ONNX, (input
    scale, input zero point)).  The INT8 file quantizes the input per tensor and the output by MinMax
    over a float run, both from `sample` [N, k, 1, W]; its output is the codes' Q/DQ, as rec-latin's
    head ends."""
    wt = {"head.w": np.asarray(w, np.float32).reshape(classes, k, 1, 1), "head.b": np.asarray(b, np.float32)}

    def build(quant):
        bl = _Builder(quant, wt)
        x = bl.qdq("x")
        y = bl.conv("head", x, 1, 1, 1, 1, (0, 0, 0, 0), False)
        out = y
        if quant is not None:
            bl.node("Identity", [bl.qdq(y)], ["y"])
            out = bl.qdq("y", params_of=y)
        bl.g.inputs = [pb.ValueInfo("x", pb.FLOAT, ["N", k, 1, "W"])]
        bl.g.outputs = [pb.ValueInfo(out, pb.FLOAT, ["N", classes, 1, "W"])]
        return pb.Model(bl.g, 17, {})

    fp = build(None)
    out = forward_float(netdef.compile_model(fp), np.asarray(sample, np.float32))

    def params(lo, hi):
        lo, hi = min(lo, 0.0), max(hi, 0.0)
        s = np.float32((hi - lo) / 255.0)
        return float(s), int(np.clip(np.rint(-lo / float(s)), 0, 255))

    quant = {"x": params(float(sample.min()), float(sample.max())), "head.out": params(float(out.min()), float(out.max()))}
    return fp, build(quant), quant["x"]
