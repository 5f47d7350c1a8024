"""ONNX files read and written without the onnx package: protobuf's wire format for
the few messages a recognizer file uses.

Field numbers follow onnx.proto3 (the public schema): ModelProto (ir_version 1,
producer_name 2, graph 7, opset_import 8, metadata_props 14), GraphProto (node 1,
name 2, initializer 5, input 11, output 12), NodeProto (input 1, output 2, name 3,
op_type 4, attribute 5, domain 7), AttributeProto (name 1, f 2, i 3, s 4, t 5,
floats 7, ints 8, type 20), TensorProto (dims 1, data_type 2, float_data 4,
int32_data 5, int64_data 7, name 8, raw_data 9), ValueInfoProto (name 1, type 2),
TypeProto (tensor_type 1), TypeProto.Tensor (elem_type 1, shape 2),
TensorShapeProto (dim 1), Dimension (dim_value 1, dim_param 2).  These are the
fields the reference's own reader takes (carbon/src/net/onnx.cpp:130-300).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

FLOAT, UINT8, INT8, INT32, INT64, FLOAT16 = 1, 2, 3, 6, 7, 10
NP_OF = {FLOAT: np.float32, UINT8: np.uint8, INT8: np.int8, INT32: np.int32, INT64: np.int64, FLOAT16: np.float16}
CODE_OF = {np.dtype(v): k for k, v in NP_OF.items()}

# AttributeProto.AttributeType
A_FLOAT, A_INT, A_STRING, A_TENSOR, A_FLOATS, A_INTS = 1, 2, 3, 4, 6, 7


# ----------------------------------------------------------------------------- wire format

def _varint(v: int) -> bytes:
    if v < 0:
        v += 1 << 64
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(fieldno: int, wire: int) -> bytes:
    return _varint((fieldno << 3) | wire)


def _len(fieldno: int, payload: bytes) -> bytes:
    return _key(fieldno, 2) + _varint(len(payload)) + payload


def _int(fieldno: int, v: int) -> bytes:
    return _key(fieldno, 0) + _varint(v)


def _str(fieldno: int, s: str) -> bytes:
    return _len(fieldno, s.encode())


def _read_varint(b: bytes, i: int) -> tuple[int, int]:
    r = s = 0
    while True:
        c = b[i]
        i += 1
        r |= (c & 0x7F) << s
        s += 7
        if c < 0x80:
            return r, i


def _fields(b: bytes):
    i = 0
    while i < len(b):
        k, i = _read_varint(b, i)
        f, w = k >> 3, k & 7
        if w == 0:
            v, i = _read_varint(b, i)
        elif w == 1:
            v = b[i:i + 8]
            i += 8
        elif w == 2:
            n, i = _read_varint(b, i)
            v = b[i:i + n]
            i += n
        elif w == 5:
            v = b[i:i + 4]
            i += 4
        else:
            raise ValueError(f"protobuf wire type {w}")
        yield f, w, v


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


def _ints(w: int, v) -> list[int]:
    if w == 0:
        return [_signed(v)]
    out, j = [], 0
    while j < len(v):
        x, j = _read_varint(v, j)
        out.append(_signed(x))
    return out


# ----------------------------------------------------------------------------- messages

@dataclass
class Node:
    op: str
    inputs: list[str]
    outputs: list[str]
    name: str = ""
    attrs: dict = field(default_factory=dict)  # name -> int | float | str | list[int] | list[float] | np.ndarray

    def get(self, name, default=None):
        return self.attrs.get(name, default)


@dataclass
class ValueInfo:
    name: str
    dtype: int
    dims: list  # int or str (a free dimension)


@dataclass
class Graph:
    nodes: list[Node] = field(default_factory=list)
    initializers: dict = field(default_factory=dict)  # name -> np.ndarray
    inputs: list[ValueInfo] = field(default_factory=list)
    outputs: list[ValueInfo] = field(default_factory=list)
    name: str = "graph"


@dataclass
class Model:
    graph: Graph
    opset: int = 17
    metadata: dict = field(default_factory=dict)
    producer: str = "carbon-rec-b200"


def _tensor_bytes(name: str, a: np.ndarray) -> bytes:
    a = np.asarray(a)
    if not a.flags.c_contiguous:
        a = a.copy(order="C")  # (np.ascontiguousarray would make a 0-d scalar 1-d)
    out = b"".join(_int(1, int(d)) for d in a.shape)
    out += _int(2, CODE_OF[a.dtype])
    out += _str(8, name)
    out += _len(9, a.tobytes())
    return out


def _attr_bytes(name: str, v) -> bytes:
    out = _str(1, name)
    if isinstance(v, np.ndarray):
        return out + _len(5, _tensor_bytes(name, v)) + _int(20, A_TENSOR)
    if isinstance(v, bool) or isinstance(v, int):
        return out + _int(3, int(v)) + _int(20, A_INT)
    if isinstance(v, float):
        return out + _key(2, 5) + struct.pack("<f", v) + _int(20, A_FLOAT)
    if isinstance(v, str):
        return out + _str(4, v) + _int(20, A_STRING)
    if isinstance(v, (list, tuple)) and all(isinstance(x, int) for x in v):
        return out + b"".join(_int(8, x) for x in v) + _int(20, A_INTS)
    if isinstance(v, (list, tuple)):
        return out + _len(7, struct.pack(f"<{len(v)}f", *v)) + _int(20, A_FLOATS)
    raise TypeError(f"attribute {name}: {type(v)}")


def _value_info_bytes(v: ValueInfo) -> bytes:
    dims = b""
    for d in v.dims:
        dims += _len(1, _int(1, d) if isinstance(d, int) else _str(2, d))
    tensor_type = _int(1, v.dtype) + _len(2, dims)
    return _str(1, v.name) + _len(2, _len(1, tensor_type))


def encode(m: Model) -> bytes:
    g = m.graph
    gb = b""
    for n in g.nodes:
        nb = b"".join(_str(1, i) for i in n.inputs) + b"".join(_str(2, o) for o in n.outputs)
        nb += _str(3, n.name or n.outputs[0]) + _str(4, n.op)
        nb += b"".join(_len(5, _attr_bytes(k, v)) for k, v in n.attrs.items())
        gb += _len(1, nb)
    gb += _str(2, g.name)
    gb += b"".join(_len(5, _tensor_bytes(k, v)) for k, v in g.initializers.items())
    gb += b"".join(_len(11, _value_info_bytes(v)) for v in g.inputs)
    gb += b"".join(_len(12, _value_info_bytes(v)) for v in g.outputs)
    out = _int(1, 8) + _str(2, m.producer) + _len(7, gb) + _len(8, _str(1, "") + _int(2, m.opset))
    for k, v in m.metadata.items():
        out += _len(14, _str(1, k) + _str(2, v))
    return out


def _decode_tensor(b: bytes) -> tuple[str, np.ndarray]:
    dims, dtype, name, raw = [], 0, "", None
    fdata, idata = [], []
    for f, w, v in _fields(b):
        if f == 1:
            dims += _ints(w, v)
        elif f == 2:
            dtype = v
        elif f == 4:
            fdata += list(struct.unpack(f"<{len(v) // 4}f", v)) if w == 2 else [struct.unpack("<f", v)[0]]
        elif f in (5, 7):
            idata += _ints(w, v)
        elif f == 8:
            name = v.decode()
        elif f == 9:
            raw = v
    npt = NP_OF[dtype]
    if raw is not None:
        a = np.frombuffer(raw, npt).copy()
    elif fdata:
        a = np.array(fdata, np.float32).astype(npt)
    elif dtype == FLOAT16:
        a = np.array(idata, np.uint16).view(np.float16)
    else:
        a = np.array(idata, np.int64).astype(npt)
    return name, a.reshape(dims) if dims else a.reshape(())


def _decode_attr(b: bytes):
    name, val, kind = "", None, 0
    ints, floats = [], []
    for f, w, v in _fields(b):
        if f == 1:
            name = v.decode()
        elif f == 2:
            val = struct.unpack("<f", v)[0]
        elif f == 3:
            val = _signed(v)
        elif f == 4:
            val = v.decode()
        elif f == 5:
            val = _decode_tensor(v)[1]
        elif f == 7:
            floats += list(struct.unpack(f"<{len(v) // 4}f", v)) if w == 2 else [struct.unpack("<f", v)[0]]
        elif f == 8:
            ints += _ints(w, v)
        elif f == 20:
            kind = v
    if kind == A_INTS or (val is None and ints):
        val = ints
    elif kind == A_FLOATS or (val is None and floats):
        val = floats
    return name, val


def _decode_value_info(b: bytes) -> ValueInfo:
    name, dtype, dims = "", 0, []
    for f, _, v in _fields(b):
        if f == 1:
            name = v.decode()
        elif f == 2:
            for tf, _, tv in _fields(v):
                if tf != 1:
                    continue
                for ttf, _, ttv in _fields(tv):
                    if ttf == 1:
                        dtype = ttv
                    elif ttf == 2:
                        for sf, _, sv in _fields(ttv):
                            if sf != 1:
                                continue
                            d = -1
                            for df, _, dv in _fields(sv):
                                if df == 1:
                                    d = dv
                                elif df == 2:
                                    d = dv.decode()
                            dims.append(d)
    return ValueInfo(name, dtype, dims)


def decode(b: bytes) -> Model:
    g = Graph()
    opset, meta = 0, {}
    for f, _, v in _fields(b):
        if f == 7:
            for gf, _, gv in _fields(v):
                if gf == 1:
                    ins, outs, name, op, attrs = [], [], "", "", {}
                    for nf, _, nv in _fields(gv):
                        if nf == 1:
                            ins.append(nv.decode())
                        elif nf == 2:
                            outs.append(nv.decode())
                        elif nf == 3:
                            name = nv.decode()
                        elif nf == 4:
                            op = nv.decode()
                        elif nf == 5:
                            k, val = _decode_attr(nv)
                            attrs[k] = val
                    g.nodes.append(Node(op, ins, outs, name, attrs))
                elif gf == 5:
                    k, a = _decode_tensor(gv)
                    g.initializers[k] = a
                elif gf == 11:
                    g.inputs.append(_decode_value_info(gv))
                elif gf == 12:
                    g.outputs.append(_decode_value_info(gv))
        elif f == 8:
            dom, ver = "", 0
            for of, _, ov in _fields(v):
                if of == 1:
                    dom = ov.decode()
                elif of == 2:
                    ver = ov
            if dom in ("", "ai.onnx"):
                opset = ver
        elif f == 14:
            k = val = ""
            for mf, _, mv in _fields(v):
                if mf == 1:
                    k = mv.decode()
                elif mf == 2:
                    val = mv.decode()
            meta[k] = val
    g.inputs = [i for i in g.inputs if i.name not in g.initializers]
    return Model(g, opset, meta)


def load(path) -> Model:
    with open(path, "rb") as f:
        return decode(f.read())


def save(m: Model, path) -> None:
    with open(path, "wb") as f:
        f.write(encode(m))
