"""BASELINE.json's page configurations as stated, on the GPU, against the reference's own CPU code.

* Config 5 (the bench's workload): 1024 page slots x 64 lines (65,536 lines), each slot a
  device buffer of its own, every line at its 32-px bucket, in runs of the bench's size.
  Every line's ids, frames and probability bits equal the reference's int8 path
  (oracle/_ref: crop_lines, the native executor on 1 - p / 255, ctc_greedy with
  lengths min(frames, width / 4); carbon/src/pipeline.cpp:138-162).
* Config 2: 16 pages x 64 lines through the FP16 engine: crops byte-equal to the reference's
  crop_lines, logits within FP16_LOGIT_TOL of the reference's FP32 executor on the same crops,
  at least FP16_ID_AGREEMENT of the frame ids agreeing.

The reference's results come from its compiled CPU code (it travels to a GPU box as built
files); each distinct (page, bucket) group of lines is cropped and run once, in threads with a
single-threaded session each."""
from __future__ import annotations

import queue
import tempfile
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import pytest

from carbon_rec import native, onnx_pb, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

FP16_LOGIT_TOL = 2e-2   # max |logit_fp16 - logit_fp32|
FP16_ID_AGREEMENT = 0.999
LINES = 64


def buckets(boxes):
    widths = np.array([native.crop_region(b)[1] for b in boxes])
    return ((widths + 31) // 32 * 32).astype(np.int32)


def reference_runs(ref, onnx_model, pages, boxes, bws, want_logits=False, threads=8):
    """The reference's path on every page's lines, grouped by bucket: per page a list of
    (ids, frames, probs) per line, its lengths, its crops at each line's bucket and (optionally)
    its logits [classes, bw / 4] per line."""
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "rec.onnx"
        onnx_pb.save(onnx_model, path)
        free = queue.Queue()
        for _ in range(threads):
            free.put(ref.session(path))  # a session is not thread-safe: one a worker at a time

        def one(p):
            s = free.get()
            try:
                return page(p, s)
            finally:
                free.put(s)

        def page(p, s):
            n = len(boxes[p])
            lines, lengths, crops, logits = [None] * n, np.zeros(n, np.int32), [None] * n, [None] * n
            for bw in np.unique(bws[p]):
                sel = np.nonzero(bws[p] == bw)[0]
                c, w = ref.crop_lines(pages[p], boxes[p][sel], int(bw))
                x = (np.float32(1.0) - c.astype(np.float32) / np.float32(255.0))[:, None]
                lg = s.run(x)
                ln = np.minimum(int(bw) // 4, w // 4).astype(np.int32)
                dec = ref.ctc_greedy(lg, ln)
                for j, i in enumerate(sel):
                    lines[i], lengths[i], crops[i] = dec[j], ln[j], c[j]
                    if want_logits:
                        logits[i] = lg[j]
            return lines, lengths, crops, logits

        with ThreadPoolExecutor(threads) as ex:
            return list(ex.map(one, range(len(pages))))


@pytest.fixture(scope="module")
def ref():
    if not O.Reference.available():
        pytest.skip("the reference's compiled code (oracle/_ref) is not here")
    return O.Reference()


def test_config5_every_line_int8_equals_the_reference(rec_latin, ref):
    import torch
    pages, boxes = synth.pages(5000, 32, 2480, 3508, LINES)  # bench.py's contents
    bws = [buckets(b) for b in boxes]
    want = reference_runs(ref, rec_latin[2], pages, boxes, bws)
    slots = 1024
    dev_pages = []
    for s in range(slots):
        t = torch.empty((3508, 2480), dtype=torch.uint8, device="cuda")
        t.copy_(torch.from_numpy(pages[s % 32]))
        dev_pages.append(t)
    page_of = np.repeat(np.arange(slots), LINES).astype(np.int32)
    allb = np.concatenate([boxes[s % 32] for s in range(slots)])
    bw_all = np.concatenate([bws[s % 32] for s in range(slots)])
    dev = native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=32768, max_width=1024,
                           max_columns=1 << 23, max_pages=slots)
    try:
        dev.set_pages_device([(t.data_ptr(), 2480, 3508, 2480) for t in dev_pages])
        got = dev.recognize_lines(page_of, allb, bw_all, flat=True)
        runs = dev.last_stats()["runs"]
    finally:
        dev.close()
    assert runs >= 2  # the bench's run size cuts the job into several runs
    chars = 0
    for s in range(slots):
        lines, lengths, _, _ = want[s % 32]
        for j in range(LINES):
            i = s * LINES + j
            o, k = int(got["offsets"][i]), int(got["counts"][i])
            ids, fr, pr = lines[j]
            assert got["lengths"][i] == lengths[j], (s, j)
            assert np.array_equal(got["ids"][o:o + k], ids) and np.array_equal(got["frames"][o:o + k], fr), (s, j)
            assert np.array_equal(got["probs"][o:o + k].view(np.int32), pr.view(np.int32)), (s, j)
            chars += k
    assert chars > 65536  # text-like pages: many characters, not mostly blank lines


def test_config2_fp16_as_stated(rec_latin, ref):
    """16 pages x 64 lines, FP16: crops byte-equal, logits within tolerance of FP32, ids agreeing."""
    pages, boxes = synth.pages(2000, 16, 2480, 3508, LINES)
    bws = [buckets(b) for b in boxes]
    want = reference_runs(ref, rec_latin[3], pages, boxes, bws, want_logits=True)
    page_of = np.repeat(np.arange(16), LINES).astype(np.int32)
    allb = np.concatenate(boxes)
    bw_all = np.concatenate(bws)
    dev = native.RecDevice(rec_latin[1].to_blob(), native.FP16, max_lines=1024, max_width=1024, max_pages=16,
                           max_page_bytes=16 * 2480 * 3508)
    try:
        dev.set_pages(pages)
        dev.arm_crops(1024)
        dev.arm_logits()
        got, lengths = dev.recognize_lines(page_of, allb, bw_all)
        crops = dev.crops(len(allb), 1024)
        logits = dev.logits(bw_all, 800)
    finally:
        dev.close()
    worst, agree, total = 0.0, 0, 0
    for p in range(16):
        _, ref_len, ref_crops, ref_logits = want[p]
        for j in range(LINES):
            i = p * LINES + j
            bw = int(bw_all[i])
            assert np.array_equal(crops[i][:, :bw], ref_crops[j]), (p, j)
            assert lengths[i] == ref_len[j]
            worst = max(worst, float(np.abs(logits[i] - ref_logits[j]).max()))
            n = int(lengths[i])
            agree += int((logits[i].argmax(0)[:n] == ref_logits[j].argmax(0)[:n]).sum())
            total += n
    assert worst <= FP16_LOGIT_TOL, worst
    assert agree / total >= FP16_ID_AGREEMENT, (agree, total)
    assert total > 30000
