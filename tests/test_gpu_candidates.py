"""The beam's candidates (crec_candidates; the reference's PipelineModels::candidates and
carbon::frame_candidates): for lines of the last recognize call, each frame's topk likeliest classes
but the blank with their log-probabilities, and the blank's.

* INT8: bit for bit the oracle's ctc_topk (pinned to the reference's cpu::ctc_topk in
  tests/test_oracle_reference.py) over the run's own logits (the device's logits hook), for topk
  0, 5 and 16 (a larger topk clamped to 16); lines of an earlier run of a call cut into several
  runs are refused, as are rows outside the call.
* FP16: the candidates' logits are made again in FP32 in channel order, so against the same
  ctc_topk over the fused head's logits the log-probabilities agree within FP16_LOGP_TOL and the
  ids but for near ties."""
from __future__ import annotations

import numpy as np
import pytest

from carbon_rec import native, synth

pytestmark = pytest.mark.gpu

FP16_LOGP_TOL = 5e-3


def run(blob, precision, pages, boxes, page_of, **kw):
    dev = native.RecDevice(blob, precision, max_pages=len(pages), max_page_bytes=sum(p.size for p in pages), **kw)
    dev.set_pages(pages)
    dev.arm_logits()
    got, lengths = dev.recognize(page_of, boxes, 1024)
    return dev, lengths, dev.logits([1024] * len(boxes), 800)


def test_candidates_int8_bit_exact(rec_latin, orc):
    pages, boxes = synth.pages(21, 2, 1600, 1200, 30)
    page_of = np.repeat(np.arange(2), 30).astype(np.int32)
    allb = np.concatenate(boxes)
    dev, lengths, logits = run(rec_latin[0].to_blob(), native.INT8, pages, allb, page_of, max_lines=64,
                               max_width=1024)
    try:
        rows = [0, 3, 17, 29, 30, 44, 59]
        for topk in (0, 5, 16):
            got = dev.candidates(rows, topk)
            for r, (ids, logp, blank) in zip(rows, got):
                want = orc.ctc_topk(logits[r], int(lengths[r]), topk)
                assert ids.shape == (lengths[r], topk)
                assert np.array_equal(ids, want[0]), (r, topk)
                assert np.array_equal(logp.view(np.int32), want[1].view(np.int32)), (r, topk)
                assert np.array_equal(blank.view(np.int32), want[2].view(np.int32)), (r, topk)
        for bad in (lambda: dev.candidates([60], 5), lambda: dev.candidates([-1], 5)):
            with pytest.raises(native.CrecError) as e:
                bad()
            assert e.value.code == native.E_RANGE
        # topk clamped to 16, as the reference's GPU device clamps it
        ids, logp, _ = dev.candidates([3], 40)[0]
        assert ids.shape[1] == 16 and np.array_equal(ids, orc.ctc_topk(logits[3], int(lengths[3]), 16)[0])
        # the same rows asked again give the same candidates (the head's input is still there)
        a, b = dev.candidates([17], 5)[0], dev.candidates([17], 5)[0]
        assert all(np.array_equal(x.view(np.int32), y.view(np.int32)) for x, y in zip(a, b))
    finally:
        dev.close()


def test_candidates_of_a_call_cut_into_runs(rec_latin, orc):
    """max_columns 19,456 (a multiple of the run granularity, 1024 columns): 60 lines of 1024
    columns (1056 with their gap) go in runs of 18, four runs; the last run's lines (54..59) have candidates equal to a one-run device's, the earlier ones
    are refused."""
    pages, boxes = synth.pages(22, 2, 1600, 1200, 30)
    page_of = np.repeat(np.arange(2), 30).astype(np.int32)
    allb = np.concatenate(boxes)
    one, _, logits = run(rec_latin[0].to_blob(), native.INT8, pages, allb, page_of, max_lines=64, max_width=1024)
    cut, lengths, _ = run(rec_latin[0].to_blob(), native.INT8, pages, allb, page_of, max_lines=64, max_width=1024,
                          max_columns=19456)
    try:
        assert cut.last_stats()["runs"] == 4
        rows = list(range(54, 60))
        for r, (x, y) in zip(rows, zip(cut.candidates(rows, 5), one.candidates(rows, 5))):
            want = orc.ctc_topk(logits[r], int(lengths[r]), 5)
            for a, b, c in zip(x, y, want):
                assert np.array_equal(a.view(np.int32), b.view(np.int32)) and np.array_equal(a.view(np.int32), c.view(np.int32))
        with pytest.raises(native.CrecError) as e:
            cut.candidates([53], 5)
        assert e.value.code == native.E_RANGE
    finally:
        one.close()
        cut.close()


def test_candidates_fp16_near_the_fused_heads(rec_latin, orc):
    pages, boxes = synth.pages(23, 1, 1600, 1200, 24)
    page_of = np.zeros(24, np.int32)
    dev, lengths, logits = run(rec_latin[1].to_blob(), native.FP16, pages, boxes[0], page_of, max_lines=64,
                               max_width=1024)
    try:
        rows = list(range(24))
        worst, flips, total = 0.0, 0, 0
        for r, (ids, logp, blank) in zip(rows, dev.candidates(rows, 5)):
            want = orc.ctc_topk(logits[r], int(lengths[r]), 5)
            worst = max(worst, float(np.abs(blank - want[2]).max()), float(np.abs(logp - want[1]).max()))
            flips += int((ids[:, 0] != want[0][:, 0]).sum())
            total += len(ids)
        assert worst <= FP16_LOGP_TOL, worst
        assert flips <= total // 100 + 1, (flips, total)
    finally:
        dev.close()
