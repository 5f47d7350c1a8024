"""Host-side logic: the ONNX reader and writer, the compile to the model blob, the synthetic
inputs, and the C ABI library's symbols (no GPU call)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from carbon_rec import build, model, native, netdef, onnx_pb, synth

ROOT = Path(__file__).resolve().parents[1]


def test_onnx_round_trip(rec_latin):
    _, _, i8, fp = rec_latin
    for m in (i8, fp):
        back = onnx_pb.decode(onnx_pb.encode(m))
        assert [n.op for n in back.graph.nodes] == [n.op for n in m.graph.nodes]
        for k, v in m.graph.initializers.items():
            assert np.array_equal(back.graph.initializers[k], v)
        assert back.metadata == m.metadata


def test_rec_latin_compiles_to_the_model_card(rec_latin):
    n8, n32, _, _ = rec_latin
    # docs/MODELS.md:186-212 of the reference: 1.51 M parameters, 406,880 MAC per px of width
    params = sum(l.wf.size + l.bias.size for l in n32.layers if l.wf is not None)
    assert params == 1_512_000 or abs(params - 1.51e6) < 0.01e6
    macs = n32.macs_per_width()
    assert sum(macs.values()) == pytest.approx(406_880, rel=1e-9)
    # the split the roofline counts: stem and depthwise on CUDA cores, the dense convolutions
    # (3x3, 2x3 and the 1x1 mixing pair) and the head on the tensor cores
    assert macs == {"stem": 2_304.0, "conv": 352_512.0, "dw": 864.0, "head": 51_200.0}
    kinds = [l.kind for l in n8.layers]
    assert kinds.count(netdef.KIND_DW) == 2 and kinds.count(netdef.KIND_RESIZE) == 1
    assert all(l.int8 for l in n8.layers if l.kind != netdef.KIND_RESIZE)
    assert n8.values[n8.out].u8 and n8.classes == 800
    assert n8.frames_for(512) == 128
    # the residual Adds joined their convolutions; the Add's parameters are the sum's
    downs = [l for l in n8.layers if l.residual >= 0]
    assert len(downs) == 2 and all(not l.relu for l in downs)


def test_compile_refuses_what_it_does_not_run():
    g = onnx_pb.Graph()
    g.inputs = [onnx_pb.ValueInfo("x", onnx_pb.FLOAT, ["N", 1, 32, "W"])]
    g.nodes = [onnx_pb.Node("Sigmoid", ["x"], ["y"], "s")]
    g.outputs = [onnx_pb.ValueInfo("y", onnx_pb.FLOAT, ["N", 1, 32, "W"])]
    with pytest.raises(netdef.RefuseError):
        netdef.compile_model(onnx_pb.Model(g))


def test_blob_reads_back_in_the_oracle(orc, rec_latin, mini):
    for net in (rec_latin[0], rec_latin[1], mini[0], mini[1]):
        m = orc.model(net.to_blob())
        assert m.classes == net.classes
    with pytest.raises(ValueError):
        orc.model(b"CRECMDL1" + b"\0" * 40)


def test_input_table_is_the_reference_quantize(orc, rec_latin):
    n8 = rec_latin[0]
    t = orc.model(n8.to_blob()).input_table()
    x = n8.values[n8.inp]
    ink = np.float32(1.0) - np.arange(256, dtype=np.float32) / np.float32(255.0)
    from carbon_rec.netdef import _quantize_float
    assert np.array_equal(t, _quantize_float(ink, x.scale, x.zero))


def test_synth_finish_is_the_crop_rule(orc):
    rng = np.random.default_rng(0)
    for i in range(60):
        w = int(rng.integers(8, 120))
        raw = rng.integers(0, 256, (32, w)).astype(np.uint8)
        if i % 3 == 0:
            raw[:] = 30
            raw[10:20, ::7] = 230
        a = synth.finish(raw, w, w + 16)
        o = np.zeros((32, w + 16), np.uint8)
        o[:, :w] = raw
        orc.finish_crop(o, w)
        assert np.array_equal(a, o)


def test_synth_pages_are_seeded():
    p1, b1 = synth.pages(5, 1, 600, 400, 6)
    p2, b2 = synth.pages(5, 1, 600, 400, 6)
    assert np.array_equal(p1[0], p2[0]) and np.array_equal(b1[0], b2[0])
    assert b1[0].shape == (6, 4) and (b1[0][:, 2] > b1[0][:, 0]).all()


def header_functions():
    text = (ROOT / "include" / "carbon_rec.h").read_text()
    return sorted(set(re.findall(r"CREC_API\s+[\w\s\*]+?\b(crec_\w+)\s*\(", text)))


def test_library_builds_and_exports_the_header():
    lib = build.build()
    names = header_functions()
    assert len(names) >= 15
    assert sorted(native.EXPORTS) == names
    L = ctypes.CDLL(str(lib))
    for n in names:
        assert hasattr(L, n), n


def test_host_entry_points_without_a_gpu(orc):
    # the pure host functions of the C ABI: the width ladder and the crop rule, bit for bit
    for w in list(range(1, 2100, 7)) + [2049, 4000]:
        assert native.width_bucket(w) == orc.width_bucket(w)
    rng = np.random.default_rng(3)
    for _ in range(100):
        h = rng.uniform(4, 120)
        x0, y0 = rng.uniform(-100, 2000), rng.uniform(-50, 3000)
        box = [x0, y0, x0 + rng.uniform(1, 2400), y0 + h]
        a, wa = native.crop_region(box)
        b, wb = orc.crop_region(box)
        assert wa == wb and list(a) == list(b)


def test_open_fails_cleanly_without_a_gpu(rec_latin):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is here")
    with pytest.raises(native.CrecError):
        native.RecDevice(rec_latin[0].to_blob())


def test_no_alloc_decoder_refuses_missing_arrays_before_any_launch():
    """crec_ctc_greedy_noalloc checks its pointers before it touches the GPU: lines without
    their lengths or counts are refused whatever the frame count (with frames == 0 it would
    otherwise clear a null counts array), and with frames the logits and character arrays too."""
    for args in ((3, 0, 0, 0), (3, 0, 0, 8), (3, 0, 8, 0), (3, 5, 8, 8)):
        n, frames, lengths, counts = args
        with pytest.raises(native.CrecError) as e:
            native.ctc_greedy_noalloc(0, n, 800, frames, lengths, counts, 0, 0, 0)
        assert e.value.code == native.E_INVALID, args
    # nothing to do: no lines
    native.ctc_greedy_noalloc(0, 0, 800, 0, 0, 0, 0, 0, 0)
