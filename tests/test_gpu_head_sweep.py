"""BASELINE.json config 4's head GEMM, and the reference's own fused-head cases
(tests/cpp/cuda_ctc_head_test.cpp: (lines, K, classes, frames) = (5, 256, 800, 77), (3, 192, 1500,
40), (2, 128, 33, 200), (4, 320, 400, 9)), through this build's fused head (crec_head_sweep: the
tcgen05 GEMM with each frame's argmax and CTC probability in its epilogue).

* FP16, graded as the reference grades its GPU head: the logits W x F + b in float64 from the same
  float16 values; a frame's id is the first class of the highest logit, or a near tie (the
  chosen class's logit within FP32_ACC_TOL of the best; FP32 sums in another order may flip only
  such a tie), near ties at most 1% of the frames + 1; where the id is the best and not the blank
  (class 0), the probability within FP32_ACC_TOL / sum of 1 / sum_c exp(l_c - l_best).  This head
  writes no probability for a blank frame (CTC drops them): 0 there.
* INT8, bit for bit: the same shapes as a Q/DQ graph (per-tensor input, per-class int8 weights,
  quantized output), against the reference's executor (oracle/_ref): every dequantized logit,
  every id (the first class of the highest code), and every non-blank frame's probability against
  the oracle's ctc_greedy per-frame probabilities (class-order sums of exp_neg, as the reference's
  kernels.cpp sums them); plus config 4's [N T, 256] x [256, 800] at N = 256 lines of 256 frames.
  An INT8 head of more classes than its shared memory holds codes for (1500) is refused."""
from __future__ import annotations

import struct
import tempfile
from pathlib import Path

import numpy as np
import pytest

from carbon_rec import model, native, netdef, onnx_pb
from oracle import oracle as O

pytestmark = pytest.mark.gpu

CASES = [(5, 256, 800, 77), (3, 192, 1500, 40), (2, 128, 33, 200), (4, 320, 400, 9)]
FP32_ACC_TOL = 1e-3


def case_data(k, classes, frames, seed):
    """Features [frames, k] ~ N(0, 1), weights [classes, k] ~ N(0, 0.06) and biases ~ N(0, 0.5), the
    reference test's distributions; features and weights float16."""
    rng = np.random.default_rng(seed)
    f = rng.normal(0.0, 1.0, (frames, k)).astype(np.float16)
    w = rng.normal(0.0, 0.06, (classes, k)).astype(np.float16)
    b = rng.normal(0.0, 0.5, classes).astype(np.float32)
    return f, w, b


@pytest.mark.parametrize("n,k,classes,frames", CASES)
def test_head_fp16_matches_the_unfused_head(n, k, classes, frames):
    f, w, b = case_data(k, classes, n * frames, seed=k + classes)
    fp, _, _ = model.make_head(k, classes, w.astype(np.float32), b, f.astype(np.float32).T[None, :, None, :])
    ids, probs, _, ms = native.head_sweep(netdef.compile_model(fp).to_blob(), native.FP16, f, classes, repeat=2)
    grade_fp16(f, w, b, ids, probs, n * frames)
    assert ms > 0


def test_rec_cjk_head_from_its_head_file():
    """The factorized rec-cjk head's last layer (docs/MODELS.md:215-219 of the reference: a 1x1 from
    192 channels to 12,000 classes) given as the export writes it, a CTCHEAD1 file
    (crec_ctc_head_blob), through the fused FP16 head: 4 lines of 64 frames, graded as above."""
    f, w, b = case_data(192, 12000, 4 * 64, seed=12)
    head = b"CTCHEAD1" + struct.pack("<ii", 12000, 192) + w.tobytes() + b.tobytes()
    ids, probs, _, ms = native.head_sweep(native.ctc_head_blob(head), native.FP16, f, 12000, repeat=2)
    grade_fp16(f, w, b, ids, probs, 4 * 64)
    assert ms > 0


def grade_fp16(f, w, b, ids, probs, frames):
    classes = w.shape[0]
    logit = f.astype(np.float64) @ w.astype(np.float64).T + b.astype(np.float64)  # [frames, classes]
    best = logit.argmax(1)
    top = logit[np.arange(len(best)), best]
    assert ((ids >= 0) & (ids < classes)).all()
    tie = ids != best
    assert (top[tie] - logit[np.arange(len(best)), ids][tie] < FP32_ACC_TOL).all()
    assert tie.sum() <= frames // 100 + 1
    s = np.exp(logit - top[:, None]).sum(1)
    keep = ~tie & (best != 0)
    assert np.all(np.abs(probs[keep] - 1.0 / s[keep]) <= FP32_ACC_TOL / s[keep])
    assert (probs[~tie & (best == 0)] == 0).all()


@pytest.fixture(scope="module")
def ref():
    if not O.Reference.available():
        pytest.skip("the reference's compiled code (oracle/_ref) is not here")
    return O.Reference()


def int8_case(ref, orc, k, classes, frames, seed):
    f, w, b = case_data(k, classes, frames, seed)
    sample = f[:min(frames, 4096)].astype(np.float32).T[None, :, None, :]
    _, i8, (xs, xz) = model.make_head(k, classes, w.astype(np.float32), b, sample)
    q = np.clip(np.rint(f.astype(np.float32) / np.float32(xs)) + xz, 0, 255).astype(np.uint8)
    ids, probs, logits, _ = native.head_sweep(netdef.compile_model(i8).to_blob(), native.INT8, q, classes, repeat=1,
                                              logits=True)
    x = ((q.astype(np.float32) - xz) * np.float32(xs)).T[None, :, None, :].copy()
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "head.onnx"
        onnx_pb.save(i8, path)
        want = ref.session(path).run(x, cap=classes * frames)[0, :, 0, :]  # [classes, frames]
    assert np.array_equal(logits.T.view(np.int32), want.view(np.int32))
    assert np.array_equal(ids, want.argmax(0))
    _, fid, fpr = orc.ctc_greedy(want.T[:, :, None], np.ones(frames, np.int32))
    nb = ids != 0
    assert np.array_equal(fid[:, 0], ids)
    assert np.array_equal(probs[nb].view(np.int32), fpr[nb, 0].view(np.int32))
    assert (probs[~nb] == 0).all()
    return nb.mean()


@pytest.mark.parametrize("n,k,classes,frames", CASES)
def test_head_int8_bit_exact(ref, orc, n, k, classes, frames):
    if classes > 1024:
        # the INT8 head keeps its tile's 128 frames' class codes in shared memory for the CTC sums:
        # 1500 classes (194 KB of codes) do not fit, and the blob is refused as a model error
        f, w, b = case_data(k, classes, 64, 0)
        _, i8, _ = model.make_head(k, classes, w.astype(np.float32), b, f.astype(np.float32).T[None, :, None, :])
        with pytest.raises(native.CrecError) as e:
            native.head_sweep(netdef.compile_model(i8).to_blob(), native.INT8, np.zeros((64, k), np.uint8), classes)
        assert e.value.code == native.E_MODEL
        return
    int8_case(ref, orc, k, classes, n * frames, seed=3 * k + classes)


def test_head_int8_config4_batch(ref, orc):
    """[N T, 256] x [256, 800]: 256 lines of 256 frames (W = 1024)."""
    nonblank = int8_case(ref, orc, 256, 800, 256 * 256, seed=4)
    assert nonblank > 0.5  # random weights: most frames' best is not the blank
