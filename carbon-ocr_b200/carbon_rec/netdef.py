"""A recognizer file compiled into the layer list the GPU engine runs, and the
model blob ("CRECMDL1") that carries it across the C ABI.

The compile restates the reference executor's reading of a Fullerene ONNX file
(carbon/src/net/net.cpp) for the operators a recognizer holds:

* Q/DQ read away (net.cpp:330-388): a QuantizeLinear then DequantizeLinear on a
  tensor marks it as kept in uint8 with that scale and zero point; a
  DequantizeLinear of a constant gives its float values (int8 weights, axis 0,
  symmetric, also kept as int8 with their per-channel scales); a graph output's
  last Q/DQ is dropped (a zero point of 0 kept as a ReLU of its own).
* Fusion (net.cpp:548-576, 762-787): a Relu joins the Conv (or depthwise Conv)
  that makes its input when nothing else reads it; a residual Add joins the
  convolution that makes one of its inputs when nothing else reads that output
  and it has no ReLU yet, and the sum is quantized once, with the Add's
  parameters (the convolution's own Q/DQ is not used).
* Resize: nearest, asymmetric, floor, whole scales (net.cpp:790-810); a Resize
  whose output only a residual reads is read in place (net.cpp:500-525).
* Identity and Squeeze name their input.
* Each tensor's border (its zero point) is as wide as the widest padding of the
  convolutions that read it (net.cpp:488-493).

The blob layout is this package's own (little-endian):

    "CRECMDL1"  u32 version (1)  u32 kind (0: int8 Q/DQ, 1: float)  u32 values  u32 layers
    u32 input value  u32 output value  u32 crop height  u32 reserved
    per value : u32 channels  u32 u8  f32 scale  i32 zero  u32 pad_h  u32 pad_w
    per layer : u32 kind (0 conv, 1 depthwise, 2 resize)  u32 in  u32 out  i32 residual
                u32 kh kw sh sw pt pl pb pr  u32 cin cout relu  u32 fh fw res_fh res_shift
                u32 int8 (weights as int8 + per-channel scales)
                weights: int8  [cout][cin/groups][kh][kw] then f32 w_scale[cout]   (int8)
                         f32   [cout][cin/groups][kh][kw]                          (float)
                f32 bias[cout]
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

from . import onnx_pb as pb

MAGIC = b"CRECMDL1"
KIND_CONV, KIND_DW, KIND_RESIZE = 0, 1, 2


class RefuseError(ValueError):
    """A file the compile does not run (the reference refuses the same ones)."""


@dataclass
class Value:
    name: str
    c: int
    last: str = ""
    u8: bool = False
    scale: float = 1.0
    zero: int = 0
    ph: int = 0
    pw: int = 0


@dataclass
class Layer:
    kind: int
    node: str
    inp: int
    out: int = -1
    residual: int = -1
    kh: int = 1
    kw: int = 1
    sh: int = 1
    sw: int = 1
    pt: int = 0
    pl: int = 0
    pb: int = 0
    pr: int = 0
    cin: int = 0
    cout: int = 0
    relu: bool = False
    fh: int = 1
    fw: int = 1
    res_fh: int = 1
    res_shift: int = 0
    wf: np.ndarray | None = None  # float weights [cout][cin/g][kh][kw]
    w8: np.ndarray | None = None  # int8 weights, same shape
    w_scale: np.ndarray | None = None  # f32 [cout]
    bias: np.ndarray | None = None  # f32 [cout]
    int8: bool = False


@dataclass
class RecNet:
    values: list[Value]
    layers: list[Layer]
    inp: int
    out: int
    out_rank: int
    quantized: bool
    height: int = 32
    fp16_file: bool = False
    meta: dict = field(default_factory=dict)

    # ------------------------------------------------------------------ shape facts
    @property
    def classes(self) -> int:
        return self.values[self.out].c

    def frames_for(self, w: int) -> int:
        """Output frames for input width w (the recognizer's horizontal stride)."""
        h, x = self.height, w
        shapes = {self.inp: (h, x)}
        for l in self.layers:
            ih, iw = shapes[l.inp]
            if l.kind == KIND_RESIZE:
                shapes[l.out] = (ih * l.fh, iw * l.fw)
            else:
                shapes[l.out] = ((ih + l.pt + l.pb - l.kh) // l.sh + 1, (iw + l.pl + l.pr - l.kw) // l.sw + 1)
        return shapes[self.out][1]

    def shapes_for(self, w: int) -> dict[int, tuple[int, int]]:
        shapes = {self.inp: (self.height, w)}
        for l in self.layers:
            ih, iw = shapes[l.inp]
            if l.kind == KIND_RESIZE:
                shapes[l.out] = (ih * l.fh, iw * l.fw)
            else:
                shapes[l.out] = ((ih + l.pt + l.pb - l.kh) // l.sh + 1, (iw + l.pl + l.pr - l.kw) // l.sw + 1)
        return shapes

    def macs_per_width(self) -> dict[str, float]:
        """MACs per pixel of input width, by layer kind (the roofline's algorithmic work)."""
        w = 1024
        shapes = self.shapes_for(w)
        out = {"stem": 0.0, "conv": 0.0, "dw": 0.0, "head": 0.0}
        for i, l in enumerate(self.layers):
            if l.kind == KIND_RESIZE:
                continue
            oh, ow = shapes[l.out]
            taps = l.kh * l.kw
            if l.kind == KIND_DW:
                out["dw"] += oh * ow * taps * l.cout / w
            elif l.out == self.out:
                out["head"] += oh * ow * taps * l.cin * l.cout / w
            elif l.cin < 16:
                out["stem"] += oh * ow * taps * l.cin * l.cout / w
            else:
                out["conv"] += oh * ow * taps * l.cin * l.cout / w
        return out

    # ------------------------------------------------------------------ blob
    def to_blob(self) -> bytes:
        b = bytearray(MAGIC)
        b += struct.pack("<IIIIIIII", 1, 0 if self.quantized else 1, len(self.values), len(self.layers),
                         self.inp, self.out, self.height, 0)
        for v in self.values:
            b += struct.pack("<IIfiII", v.c, int(v.u8), float(v.scale), int(v.zero), v.ph, v.pw)
        for l in self.layers:
            b += struct.pack("<IIIi", l.kind, l.inp, l.out, l.residual)
            b += struct.pack("<8I", l.kh, l.kw, l.sh, l.sw, l.pt, l.pl, l.pb, l.pr)
            b += struct.pack("<3I", l.cin, l.cout, int(l.relu))
            b += struct.pack("<4I", l.fh, l.fw, l.res_fh, l.res_shift)
            b += struct.pack("<I", int(l.int8))
            if l.kind == KIND_RESIZE:
                continue
            if l.int8:
                w = np.ascontiguousarray(l.w8, np.int8).tobytes()
                b += w + b"\0" * ((-len(w)) % 4)
                b += np.ascontiguousarray(l.w_scale, np.float32).tobytes()
            else:
                b += np.ascontiguousarray(l.wf, np.float32).tobytes()
            b += np.ascontiguousarray(l.bias, np.float32).tobytes()
        return bytes(b)


# ----------------------------------------------------------------------------- compile

def _quantize_float(v: np.ndarray, scale: float, zero: int) -> np.ndarray:
    """net.cpp:84-90: round(v / scale) half to even by the 1.5 * 2^23 trick, + zero, clamped."""
    r = (np.asarray(v, np.float32) / np.float32(scale)).astype(np.float32)
    r = np.minimum(np.float32(4194304.0), np.maximum(np.float32(-4194304.0), r))
    r = (r + np.float32(12582912.0)) - np.float32(12582912.0)
    r = r + np.float32(zero)
    return np.minimum(np.float32(255.0), np.maximum(np.float32(0.0), r)).astype(np.uint8)


def compile_model(model: pb.Model) -> RecNet:
    g = model.graph
    if len(g.inputs) != 1:
        raise RefuseError("networks with one input only")
    x = g.inputs[0]
    if x.dtype not in (pb.FLOAT, pb.FLOAT16) or len(x.dims) != 4 or not isinstance(x.dims[1], int) or x.dims[1] <= 0:
        raise RefuseError("the input must be float or float16 [N, C, H, W] with C fixed")
    fp16 = x.dtype == pb.FLOAT16
    consts: dict[str, np.ndarray] = dict(g.initializers)
    qweights: dict[str, tuple[np.ndarray, np.ndarray]] = {}
    quant: dict[str, tuple[float, int]] = {}
    output_names: dict[str, str] = {}
    out_names = {o.name for o in g.outputs}

    # ---- read_qdq (net.cpp:330-388)
    rename: dict[str, str] = {}
    pending: dict[str, tuple[str, tuple[float, int]]] = {}
    nodes: list[pb.Node] = []
    for n0 in g.nodes:
        n = pb.Node(n0.op, [rename.get(i, i) for i in n0.inputs], list(n0.outputs), n0.name, dict(n0.attrs))
        if n.op == "Constant":
            consts[n.outputs[0]] = np.asarray(n.attrs["value"])
        elif n.op == "QuantizeLinear":
            if fp16:
                raise RefuseError("QuantizeLinear in a float16 network")
            s = np.asarray(consts[n.inputs[1]], np.float32).reshape(-1)
            if s.size != 1:
                raise RefuseError(f"'{n.inputs[1]}': a scale for the whole tensor, not per channel")
            z = 0
            if len(n.inputs) > 2 and n.inputs[2]:
                zt = consts[n.inputs[2]]
                if zt.dtype != np.uint8:
                    raise RefuseError("uint8 activations only")
                z = int(zt.reshape(-1)[0])
            pending[n.outputs[0]] = (n.inputs[0], (float(s[0]), z))
        elif n.op == "DequantizeLinear" and n.inputs[0] in pending:
            xname, q = pending[n.inputs[0]]
            rename[n.outputs[0]] = xname
            if n.outputs[0] in out_names:
                if q[1] == 0:
                    nodes.append(pb.Node("Relu", [xname], [xname + "/relu"], n.outputs[0] + "/relu"))
                    output_names[n.outputs[0]] = xname + "/relu"
                else:
                    output_names[n.outputs[0]] = xname
                continue
            if xname in quant and quant[xname] != q:
                raise RefuseError(f"'{xname}' is quantized twice, differently")
            quant[xname] = q
        elif n.op == "DequantizeLinear":
            t = consts[n.inputs[0]]
            s = np.asarray(consts[n.inputs[1]], np.float32).reshape(-1)
            z = np.zeros(s.size, np.int64)
            if len(n.inputs) > 2 and n.inputs[2]:
                z = np.asarray(consts[n.inputs[2]]).astype(np.int64).reshape(-1)
            axis = int(n.get("axis", 1))
            v = t.astype(np.int64).reshape(-1)
            if s.size > 1:
                inner = int(np.prod(t.shape[axis + 1:])) if t.ndim > axis + 1 else 1
                k = (np.arange(v.size) // inner) % s.size
            else:
                k = np.zeros(v.size, np.int64)
            f = ((v - z[k]).astype(np.float32) * s[k]).astype(np.float32).reshape(t.shape)
            consts[n.outputs[0]] = f
            if t.dtype == np.int8 and axis == 0:
                if np.any(z != 0):
                    raise RefuseError("int8 weights must be symmetric (zero point 0)")
                qweights[n.outputs[0]] = (t.astype(np.int8), s.astype(np.float32))
        else:
            nodes.append(n)
    for name in pending:
        if any(name in n.inputs for n in nodes):
            raise RefuseError(f"QuantizeLinear '{name}' is read without a DequantizeLinear")

    # ---- compile (net.cpp:461-500)
    values: list[Value] = []
    names: dict[str, int] = {}
    layers: list[Layer] = []

    def add_value(name: str, c: int) -> int:
        values.append(Value(name, c, name))
        names[name] = len(values) - 1
        return len(values) - 1

    def value(name: str) -> int:
        if name not in names:
            raise RefuseError(f"'{name}' is not a tensor the network computes")
        return names[name]

    def producer(v: int) -> int:
        for i, l in enumerate(layers):
            if l.out == v:
                return i
        return -1

    def join(name: str, v: int) -> None:
        names[name] = v
        values[v].last = name

    uses: dict[str, int] = {}
    for n in nodes:
        for i in n.inputs:
            uses[i] = uses.get(i, 0) + 1
    for o in g.outputs:
        uses[o.name] = uses.get(o.name, 0) + 1
    add_value(x.name, int(x.dims[1]))

    for n in nodes:
        op = n.op
        if op in ("Identity", "Squeeze"):
            if n.inputs[0] in consts:
                consts[n.outputs[0]] = consts[n.inputs[0]]
                if n.inputs[0] in qweights:
                    qweights[n.outputs[0]] = qweights[n.inputs[0]]
            else:
                names[n.outputs[0]] = value(n.inputs[0])
        elif op == "Conv":
            l = Layer(KIND_CONV, n.name, value(n.inputs[0]))
            w = np.asarray(consts[n.inputs[1]], np.float32)
            if w.ndim != 4:
                raise RefuseError(f"Conv '{n.name}': 2-d only")
            if n.get("auto_pad", "NOTSET") != "NOTSET":
                raise RefuseError("auto_pad")
            if list(n.get("dilations", [1, 1])) != [1, 1]:
                raise RefuseError("dilation")
            groups = int(n.get("group", 1))
            l.cout, l.cin = int(w.shape[0]), int(w.shape[1]) * groups
            l.kh, l.kw = int(w.shape[2]), int(w.shape[3])
            l.sh, l.sw = [int(s) for s in n.get("strides", [1, 1])]
            l.pt, l.pl, l.pb, l.pr = [int(p) for p in n.get("pads", [0, 0, 0, 0])]
            if l.cin != values[l.inp].c:
                raise RefuseError(f"'{n.name}' takes {l.cin} channels")
            l.wf = w
            if n.inputs[1] in qweights:
                l.w8, l.w_scale = qweights[n.inputs[1]]
            l.bias = np.zeros(l.cout, np.float32)
            if len(n.inputs) > 2 and n.inputs[2]:
                l.bias = np.asarray(consts[n.inputs[2]], np.float32).reshape(-1)
            if groups == 1:
                l.kind = KIND_CONV
            elif groups == l.cin and l.cout == l.cin:
                l.kind = KIND_DW
            else:
                raise RefuseError("groups other than 1 and depthwise")
            l.out = add_value(n.outputs[0], l.cout)
            layers.append(l)
        elif op == "Relu":
            v = value(n.inputs[0])
            p = producer(v)
            if p < 0 or layers[p].kind not in (KIND_CONV, KIND_DW) or layers[p].relu or uses.get(n.inputs[0], 0) != 1:
                raise RefuseError(f"Relu '{n.name}' does not follow a layer it can join")
            layers[p].relu = True
            join(n.outputs[0], v)
        elif op == "Add":
            a, b = value(n.inputs[0]), value(n.inputs[1])
            fused = False
            for mine, theirs in ((0, 1), (1, 0)):
                v = a if mine == 0 else b
                r = a if theirs == 0 else b
                p = producer(v)
                if p < 0 or uses.get(n.inputs[mine], 0) != 1 or v == r:
                    continue
                l = layers[p]
                if l.kind not in (KIND_CONV, KIND_DW) or l.relu or l.residual >= 0:
                    continue
                if values[r].c != l.cout:
                    raise RefuseError("Add: channels differ")
                del layers[p]
                l.residual = r
                join(n.outputs[0], l.out)
                layers.append(l)
                fused = True
                break
            if not fused:
                raise RefuseError(f"Add '{n.name}' that no convolution takes as its residual")
        elif op == "Resize":
            if (n.get("mode", "nearest") != "nearest" or n.get("coordinate_transformation_mode", "half_pixel") != "asymmetric"
                    or n.get("nearest_mode", "round_prefer_floor") != "floor"):
                raise RefuseError("Resize: nearest, asymmetric, floor")
            s = np.asarray(consts[n.inputs[2]], np.float32).reshape(-1)
            if s.size != 4 or s[0] != 1 or s[1] != 1 or s[2] < 1 or s[3] < 1 or s[2] != int(s[2]) or s[3] != int(s[3]):
                raise RefuseError("Resize: whole scales over H and W")
            l = Layer(KIND_RESIZE, n.name, value(n.inputs[0]))
            l.fh, l.fw = int(s[2]), int(s[3])
            l.cin = l.cout = values[l.inp].c
            l.out = add_value(n.outputs[0], l.cout)
            layers.append(l)
        else:
            raise RefuseError(f"op {op} ('{n.name}')")

    if len(g.outputs) != 1:
        raise RefuseError("a recognizer has one output")
    o = g.outputs[0]
    out_v = value(output_names.get(o.name, o.name))
    for v in values:
        if v.last in quant:
            v.u8 = True
            v.scale, v.zero = quant[v.last]
    values[out_v].u8 = values[out_v].u8  # the output keeps its storage: u8 logits are read through a table
    # upsampling read in place (net.cpp:500-525)
    p = 0
    while p < len(layers):
        up = layers[p]
        reads, reader = 0, -1
        for i, l in enumerate(layers):
            reads += (l.inp == up.out) + (l.residual == up.out)
            if l.residual == up.out:
                reader = i
        reads += int(out_v == up.out)
        a, b = values[up.inp], values[up.out]
        same = a.u8 == b.u8 and (not a.u8 or (a.scale == b.scale and a.zero == b.zero))
        pow2 = up.fw > 0 and (up.fw & (up.fw - 1)) == 0
        if up.kind != KIND_RESIZE or reads != 1 or reader < 0 or not pow2 or not same or layers[reader].res_fh != 1:
            p += 1
            continue
        rl = layers[reader]
        rl.residual, rl.res_fh = up.inp, up.fh
        f = up.fw
        while f > 1:
            rl.res_shift += 1
            f >>= 1
        del layers[p]
    for l in layers:
        if l.kind in (KIND_CONV, KIND_DW):
            v = values[l.inp]
            v.ph = max(v.ph, l.pt, l.pb)
            v.pw = max(v.pw, l.pl, l.pr)
    quantized = False
    for l in layers:
        if l.kind == KIND_RESIZE:
            continue
        xin = values[l.inp]
        if xin.u8 and l.w8 is None:
            raise RefuseError(f"'{l.node}': a uint8 input needs int8 weights")
        l.int8 = xin.u8
        quantized = quantized or l.int8
    h = x.dims[2] if isinstance(x.dims[2], int) and x.dims[2] > 0 else 32
    return RecNet(values, layers, 0, out_v, len(o.dims), quantized, int(h), fp16, dict(model.metadata))


def load(path) -> RecNet:
    return compile_model(pb.load(path))
