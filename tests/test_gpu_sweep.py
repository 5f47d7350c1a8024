"""BASELINE.json config 4, the kernel sweep: 3x3 stride-1 convolutions C -> C for C in {32, 64,
128, 256}, H in {8, 16, 32}, W in {128, 512, 1024}, through the recognizer's own tcgen05
implicit-GEMM kernel (crec_conv_sweep sets the layer up exactly as a recognizer does), against
the reference's executor (oracle/_ref) on the same layer file:

* INT8: every output code bit for bit (inputs ~N(0, 1) quantized per tensor), at every shape
  with two lines, and at the configuration's N = 256 lines on one shape (three lines checked);
* FP16: every output within FP16_TOL of the reference's FP32 result on the same inputs (the
  float16 inputs widened), the layer's weights rounded to float16 as the FP16 engine keeps them."""
from __future__ import annotations

import tempfile
from pathlib import Path

import numpy as np
import pytest

from carbon_rec import model, native, netdef, onnx_pb
from oracle import oracle as O

pytestmark = pytest.mark.gpu

CHANNELS, HEIGHTS, WIDTHS = (32, 64, 128, 256), (8, 16, 32), (128, 512, 1024)
FP16_TOL = 2e-2  # max |y_fp16 - y_fp32|, outputs of magnitude up to ~8


@pytest.fixture(scope="module")
def ref():
    if not O.Reference.available():
        pytest.skip("the reference's compiled code (oracle/_ref) is not here")
    return O.Reference()


def reference_run(ref, onnx_model, x_nchw):
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "conv.onnx"
        onnx_pb.save(onnx_model, path)
        n, _, h, w = x_nchw.shape
        return ref.session(path).run(x_nchw, cap=n * 256 * h * w)


def int8_case(ref, c, h, w, n, check, seed):
    fp, i8, (xs, xz) = model.make_conv(c, c, h, seed=seed)
    net = netdef.compile_model(i8)
    yv = net.values[net.out]
    rng = np.random.default_rng(seed)
    q = np.clip(np.rint(rng.normal(0.0, 1.0, (n, h, w, c)) / xs) + xz, 0, 255).astype(np.uint8)
    y, ms = native.conv_sweep(net.to_blob(), native.INT8, q, c, repeat=1)
    xf = ((q[check].astype(np.float32) - xz) * np.float32(xs)).transpose(0, 3, 1, 2).copy()
    want = np.rint(reference_run(ref, i8, xf) / np.float32(yv.scale)).astype(np.int64) + yv.zero
    return y[check].transpose(0, 3, 1, 2), want, ms


@pytest.mark.parametrize("c", CHANNELS)
def test_sweep_int8_bit_exact(ref, c):
    for h in HEIGHTS:
        for w in WIDTHS:
            got, want, _ = int8_case(ref, c, h, w, 2, [0, 1], seed=c + h + w)
            assert np.array_equal(got.astype(np.int64), want), (c, h, w, int(np.count_nonzero(got != want)))


def test_sweep_int8_at_the_configured_batch(ref):
    got, want, ms = int8_case(ref, 64, 8, 128, 256, [0, 117, 255], seed=7)
    assert np.array_equal(got.astype(np.int64), want) and ms > 0


@pytest.mark.parametrize("c", CHANNELS)
def test_sweep_fp16_within_tolerance(ref, c):
    for h in HEIGHTS:
        for w in WIDTHS:
            fp, _, _ = model.make_conv(c, c, h, seed=c * h + w)
            rng = np.random.default_rng(c * h + w)
            x = rng.normal(0.0, 1.0, (2, h, w, c)).astype(np.float16)
            y, _ = native.conv_sweep(netdef.compile_model(fp).to_blob(), native.FP16, x, c, repeat=1)
            want = reference_run(ref, fp, x.astype(np.float32).transpose(0, 3, 1, 2).copy())
            worst = float(np.abs(y.astype(np.float32).transpose(0, 3, 1, 2) - want).max())
            assert worst <= FP16_TOL, (c, h, w, worst)
