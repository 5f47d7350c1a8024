"""The failure paths, in the forms that fault nothing: a bounded device wait made to run out
(a loader that never issues its copies, the wait limited to 1 ms), an injected sticky status
on the host, and a device allocation the GPU refuses.  Each checks the status the C ABI
returns and what the handle does after it."""
from __future__ import annotations

import time

import numpy as np
import pytest

from carbon_rec import native, synth

pytestmark = pytest.mark.gpu


def same(a, b):
    (la, na), (lb, nb) = a, b
    assert np.array_equal(na, nb)
    for x, y in zip(la, lb):
        assert np.array_equal(x.ids, y.ids) and np.array_equal(x.frames, y.frames)
        assert np.array_equal(x.probs.view(np.int32), y.probs.view(np.int32))


def test_a_wait_that_runs_out_ends_the_run_and_the_handle_goes_on(rec_latin):
    crops, widths, bws = synth.crops(7, 24, 96, 640)
    dev = native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=64, max_width=1024, max_pages=1)
    try:
        want = dev.recognize_crops(crops, widths, bws)
        dev.inject(native.INJECT_TIMEOUT)
        t0 = time.time()
        with pytest.raises(native.CrecError) as e:
            dev.recognize_crops(crops, widths, bws)
        assert e.value.code == native.E_TIMEOUT
        assert time.time() - t0 < 1.5  # 1 ms limits, not the default 2 s
        assert not dev.broken
        same(dev.recognize_crops(crops, widths, bws), want)  # the next run is whole again
    finally:
        dev.close()


def test_a_sticky_status_breaks_the_handle_for_good(rec_latin):
    pages, boxes = synth.pages(3, 1, 900, 700, 6)
    dev = native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=64, max_width=1024, max_pages=1)
    try:
        dev.set_pages(pages)
        dev.recognize([0] * 6, boxes[0], 1024)
        dev.inject(native.INJECT_STICKY)
        with pytest.raises(native.CrecError) as e:
            dev.recognize([0] * 6, boxes[0], 1024)
        assert e.value.code == native.E_STICKY
        assert dev.broken
        for call in (lambda: dev.recognize([0] * 6, boxes[0], 1024), lambda: dev.set_pages(pages),
                     lambda: dev.prefetch_pages(pages), lambda: dev.recognize_lines([0] * 6, boxes[0])):
            with pytest.raises(native.CrecError) as e:
                call()
            assert e.value.code == native.E_STICKY
    finally:
        dev.close()


def test_device_memory_refused_at_open(rec_latin):
    """More columns than any GPU holds: the first activation's cudaMalloc is refused, open returns
    CREC_E_NOMEM and frees what it had; a handle of ordinary size opens after it."""
    with pytest.raises(native.CrecError) as e:
        native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=64, max_width=1024, max_columns=1 << 40)
    assert e.value.code == native.E_NOMEM
    dev = native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=64, max_width=1024)
    dev.close()


def test_a_large_runs_first_bad_line_is_the_error(rec_latin):
    """A run of thousands of lines is laid out by the host pool in parts; the error reported is the
    first failing line's, as one pass in line order reports it, and the handle goes on."""
    pages, boxes = synth.pages(5, 1, 2480, 3508, 64)
    n = 6000
    bx = np.tile(np.asarray(boxes[0], np.float64), (n // 64 + 1, 1))[:n]
    bw = np.array([native.width_bucket(native.crop_region(b)[1]) for b in bx[:64]] * (n // 64 + 1), np.int32)[:n]
    dev = native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=8192, max_width=1024, max_pages=1,
                           max_page_bytes=pages[0].size, max_columns=1 << 22)
    try:
        dev.set_pages(pages)
        page_of = np.zeros(n, np.int32)
        want = dev.recognize_lines(page_of, bx, bw, flat=True)
        bad = page_of.copy()
        bad[[2500, 4100, 5999]] = 3  # no page 3
        with pytest.raises(native.CrecError) as e:
            dev.recognize_lines(bad, bx, bw, flat=True)
        assert e.value.code == native.E_INVALID and "line 2500:" in str(e.value)
        narrow = bw.copy()
        narrow[[4100, 4200]] = 32  # narrower than the line's crop
        with pytest.raises(native.CrecError) as e:
            dev.recognize_lines(page_of, bx, narrow, flat=True)
        assert e.value.code == native.E_RANGE and "line 4100 " in str(e.value)
        again = dev.recognize_lines(page_of, bx, bw, flat=True)
        for k in ("counts", "lengths", "offsets", "ids", "frames"):
            assert np.array_equal(again[k], want[k])
        assert np.array_equal(again["probs"].view(np.int32), want["probs"].view(np.int32))
    finally:
        dev.close()
