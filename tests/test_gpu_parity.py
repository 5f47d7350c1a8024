"""The CUDA path against the oracle, through the C ABI.

INT8: crops, every intermediate tensor, the logits' values, ids, frames and probabilities
bit for bit (the reference's int8 executor, restated in oracle/rec_oracle.c and pinned to
the reference's own code by tests/test_oracle_*.py).  FP16: logits within max-abs 2e-2 of
the FP32 recognizer and at least 99.9% of frame ids agreeing."""
from __future__ import annotations

import numpy as np
import pytest

from carbon_rec import native, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

FP16_LOGIT_TOL = 2e-2   # max |logit_fp16 - logit_fp32|
FP16_ID_AGREEMENT = 0.999


@pytest.fixture(scope="module")
def dev8(rec_latin):
    d = native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=512, max_width=2048, max_pages=8)
    yield d
    d.close()


@pytest.fixture(scope="module")
def dev16(rec_latin):
    d = native.RecDevice(rec_latin[1].to_blob(), native.FP16, max_lines=512, max_width=2048, max_pages=8)
    yield d
    d.close()


def oracle_lines(orc, m, crops, widths, bws):
    """Per line at its own bucket width: (logits, (ids, frames, probs), length)."""
    out = []
    for i in range(len(crops)):
        logits = m.run(crops[i:i + 1, :, :int(bws[i])])
        t = logits.shape[2]
        length = min(t, int(widths[i]) // 4)
        lines, _, _ = orc.ctc_greedy(logits, [length])
        out.append((logits[0], lines[0], length))
    return out


def assert_same_lines(got, lengths, want):
    for i, (g, (_, (ids, fr, pr), length)) in enumerate(zip(got, want)):
        assert lengths[i] == length, i
        assert np.array_equal(g.ids, ids), (i, g.ids[:12], ids[:12])
        assert np.array_equal(g.frames, fr), i
        assert np.array_equal(g.probs.view(np.int32), pr.view(np.int32)), i


def test_config1_int8_bit_exact(dev8, orc, rec_latin):
    crops, widths, bws = synth.crops(1, 64, 96, 640)
    dev8.arm_logits()
    got, lengths = dev8.recognize_crops(crops, widths, bws)
    want = oracle_lines(orc, orc.model(rec_latin[0].to_blob()), crops, widths, bws)
    assert_same_lines(got, lengths, want)
    logits = dev8.logits(bws, 800)
    for i, (l, _, _) in enumerate(want):
        assert np.array_equal(logits[i], l), i


def test_every_layer_int8_bit_exact(dev8, orc, rec_latin):
    net = rec_latin[0]
    crops, widths, bws = synth.crops(2, 5, 32, 700, bucket_step=8)
    dev8.recognize_crops(crops, widths, bws)
    m = orc.model(net.to_blob())
    for vi, v in enumerate(net.values):
        if vi in (net.inp, net.out):
            continue
        shapes = [net.shapes_for(int(b))[vi] for b in bws]
        sizes = [h * w * v.c for h, w in shapes]
        got = dev8.value(vi, sum(sizes))
        at = 0
        for i in range(len(bws)):
            _, keep = m.run(crops[i:i + 1, :, :int(bws[i])], keep_value=vi, keep_shape=(sizes[i],))
            assert np.array_equal(got[at:at + sizes[i]], keep), (vi, v.name, i)
            at += sizes[i]


def test_config1_fp16_within_tolerance(dev16, orc, rec_latin):
    crops, widths, bws = synth.crops(1, 64, 96, 640)
    dev16.arm_logits()
    got, lengths = dev16.recognize_crops(crops, widths, bws)
    logits = dev16.logits(bws, 800)
    m32 = orc.model(rec_latin[1].to_blob())
    agree = total = 0
    worst = 0.0
    for i in range(len(crops)):
        ref = m32.run(crops[i:i + 1, :, :int(bws[i])])[0]
        worst = max(worst, float(np.abs(logits[i] - ref).max()))
        agree += int((logits[i].argmax(0) == ref.argmax(0)).sum())
        total += ref.shape[1]
    assert worst <= FP16_LOGIT_TOL, worst
    assert agree / total >= FP16_ID_AGREEMENT, (agree, total)
    assert all(lengths[i] == min(int(bws[i]) // 4, int(widths[i]) // 4) for i in range(len(crops)))


def test_fp16_depthwise_is_its_operations(dev16, rec_latin):
    """The FP16 depthwise layers (1x9, one at an upsample read in place) against the same
    operations in numpy: per channel an FP32 fma chain over the taps in tap order from 0 (the
    product exact in float64), + bias, ReLU if the layer has it, rounded to FP16; a line's
    columns outside it read 0 (the FP16 zero point of the gap columns)."""
    net = rec_latin[1]
    crops, widths, bws = synth.crops(3, 6, 64, 900, bucket_step=32)
    dev16.recognize_crops(crops, widths, bws)
    checked = 0
    for layer in net.layers:
        if layer.kind != 1 or layer.kh != 1:
            continue
        vi, vo = layer.inp, layer.out
        w = layer.wf.reshape(layer.cout, layer.kw).astype(np.float16).astype(np.float32)  # [c][taps]
        b = layer.bias.astype(np.float32)
        shapes_i = [net.shapes_for(int(bw))[vi] for bw in bws]
        shapes_o = [net.shapes_for(int(bw))[vo] for bw in bws]
        ci, co = net.values[vi].c, net.values[vo].c
        xin = dev16.value(vi, sum(h * wd * ci for h, wd in shapes_i) * 2, np.float16)
        xout = dev16.value(vo, sum(h * wd * co for h, wd in shapes_o) * 2, np.float16)
        ai = ao = 0
        for (hi, wi), (ho, wo) in zip(shapes_i, shapes_o):
            assert hi == ho == 1 and wi == wo
            a = xin[ai:ai + wi * ci].reshape(wi, ci)[:, :layer.cout].astype(np.float64)
            got = xout[ao:ao + wo * co].reshape(wo, co)[:, :layer.cout]
            ai += wi * ci
            ao += wo * co
            pad = np.zeros((wi + layer.kw - 1, layer.cout))
            pad[layer.pl:layer.pl + wi] = a
            s = np.zeros((wo, layer.cout), np.float32)
            for t in range(layer.kw):
                s = (pad[t:t + wo] * w[:, t].astype(np.float64) + s.astype(np.float64)).astype(np.float32)
            v = (s + b).astype(np.float32)
            if layer.relu:
                v = np.maximum(v, np.float32(0))
            assert np.array_equal(got.view(np.uint16), v.astype(np.float16).view(np.uint16)), layer.node
            checked += 1
    assert checked >= 2 * len(bws)


def two_pages(seed=7):
    """tests/cpp/cuda_lines_test.cpp:47-109 of the reference: 1700 x 2200 and 900 x 640, one inverted."""
    rng = np.random.default_rng(seed)
    pages, boxes, page_of = [], [], []
    for p, (w, h, invert) in enumerate(((1700, 2200, False), (900, 640, True))):
        page = np.clip(rng.normal(235, 8, (h, w)), 0, 255).astype(np.uint8)
        for _ in range(400):
            x, y = int(rng.integers(0, w - 20)), int(rng.integers(0, h - 10))
            page[y:y + int(rng.integers(3, 20)), x:x + int(rng.integers(2, 8))] = int(rng.integers(0, 80))
        pages.append(255 - page if invert else page)
        k = 0
        while k < 150:
            bh = rng.uniform(8, 60)
            x0, y0 = rng.uniform(-30, w - 10), rng.uniform(-20, h - 5)
            bw = rng.uniform(5, 900)
            if (bw + 0.6 * bh) * 32 / (1.4 * bh) > 1000:
                continue
            boxes.append([x0, y0, x0 + bw, y0 + bh])
            page_of.append(p)
            k += 1
    return pages, np.asarray(boxes), np.asarray(page_of, np.int32)


def decodings_without_crop_copies(blob, pages, page_of, boxes, **kw):
    """The same run on a device that does not keep its finished crops (the crop kernel's final
    pass then works a word at a time): decodings, lengths and every line's logits."""
    dev = native.RecDevice(blob, native.INT8, max_lines=512, max_width=1024, max_pages=4, **kw)
    try:
        dev.set_pages(pages)
        dev.arm_logits()
        got, lengths = dev.recognize(page_of, boxes, 1024)
        return got, lengths, dev.logits([1024] * len(boxes), 800)
    finally:
        dev.close()


def assert_same_decodings(a, la, b, lb, logits_a, logits_b):
    for i in range(len(a)):
        assert np.array_equal(logits_a[i], logits_b[i]), i
        assert la[i] == lb[i], i
        assert np.array_equal(a[i].ids, b[i].ids) and np.array_equal(a[i].frames, b[i].frames), i
        assert np.array_equal(a[i].probs.view(np.int32), b[i].probs.view(np.int32)), i


@pytest.mark.parametrize("rule", [{}, {"flip_margin": 0}])
def test_pages_crops_and_ctc_bit_exact(rec_latin, orc, rule):
    pages, boxes, page_of = two_pages()
    crop_rule = native.CropRule.default(**rule)
    dev = native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=512, max_width=1024, max_pages=4,
                           crop=crop_rule)
    try:
        dev.set_pages(pages)
        dev.arm_crops(1024)
        dev.arm_logits()
        got, lengths = dev.recognize(page_of, boxes, 1024)
        crops = dev.crops(len(boxes), 1024)
        dev_logits = dev.logits([1024] * len(boxes), 800)
    finally:
        dev.close()
    ocr = O.CropRule.default(**rule)
    want_crops = np.zeros_like(crops)
    widths = np.zeros(len(boxes), np.int32)
    for p in range(2):
        sel = np.nonzero(page_of == p)[0]
        c, w = orc.crop_lines(pages[p], boxes[sel], 1024, ocr)
        want_crops[sel] = c
        widths[sel] = w
    assert np.array_equal(crops, want_crops)
    # the recognizer on a sample of the crops, at the run's bucket width
    m = orc.model(rec_latin[0].to_blob())
    sample = np.arange(0, len(boxes), 15)
    logits = m.run(want_crops[sample])
    lines, _, _ = orc.ctc_greedy(logits, np.minimum(256, widths[sample] // 4))
    for j, i in enumerate(sample):
        # every logit: with random weights these page crops decode mostly to blanks
        assert np.array_equal(dev_logits[i], logits[j]), int(i)
        assert lengths[i] == min(256, widths[i] // 4)
        ids, fr, pr = lines[j]
        assert np.array_equal(got[i].ids, ids) and np.array_equal(got[i].frames, fr)
        assert np.array_equal(got[i].probs.view(np.int32), pr.view(np.int32))
    got2, lengths2, logits2 = decodings_without_crop_copies(rec_latin[0].to_blob(), pages, page_of, boxes, crop=crop_rule)
    assert_same_decodings(got, lengths, got2, lengths2, dev_logits, logits2)


def tall_pages(seed=11):
    """Pages whose rows are not 4-byte aligned (odd widths) and lines up to 300 px tall: windows of
    3 to 19 taps each way (downscales to ~13x), boxes over every page edge."""
    rng = np.random.default_rng(seed)
    pages, boxes, page_of = [], [], []
    for p, (w, h) in enumerate(((2481, 1803), (1203, 2999))):
        page = np.clip(rng.normal(228, 12, (h, w)), 0, 255).astype(np.uint8)
        for _ in range(600):
            x, y = int(rng.integers(0, w - 40)), int(rng.integers(0, h - 40))
            page[y:y + int(rng.integers(4, 40)), x:x + int(rng.integers(2, 16))] = int(rng.integers(0, 90))
        pages.append(page)
        k = 0
        while k < 90:
            bh = rng.uniform(20, 300)
            x0, y0 = rng.uniform(-60, w - 30), rng.uniform(-80, h - 20)
            bw = rng.uniform(30, 2400)
            if (bw + 0.6 * bh) * 32 / (1.4 * bh) > 1000:
                continue
            boxes.append([x0, y0, x0 + bw, y0 + bh])
            page_of.append(p)
            k += 1
    return pages, np.asarray(boxes), np.asarray(page_of, np.int32)


def test_tall_lines_and_odd_strides_crop_bit_exact(rec_latin, orc):
    pages, boxes, page_of = tall_pages()
    dev = native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=256, max_width=1024, max_pages=4)
    try:
        dev.set_pages(pages)
        dev.arm_crops(1024)
        dev.arm_logits()
        got, lengths = dev.recognize(page_of, boxes, 1024)
        crops = dev.crops(len(boxes), 1024)
        dev_logits = dev.logits([1024] * len(boxes), 800)
    finally:
        dev.close()
    got2, lengths2, logits2 = decodings_without_crop_copies(rec_latin[0].to_blob(), pages, page_of, boxes)
    assert_same_decodings(got, lengths, got2, lengths2, dev_logits, logits2)
    ocr = O.CropRule.default()
    for p in range(2):
        sel = np.nonzero(page_of == p)[0]
        want, _ = orc.crop_lines(pages[p], boxes[sel], 1024, ocr)
        for j, i in enumerate(sel):
            assert np.array_equal(crops[i], want[j]), (p, int(i), boxes[i])


def wide_reach_pages(seed=13):
    """A page with lines 350 to 600 px tall (downscales ~15x to ~26x: 33 to 55 taps a sample, past
    the crop kernel's 31), 1000 to 1500 px tall (more than 1024 source rows), 250 to 340 px tall
    (~11x to ~15x, just inside), some over the page's edges, among ordinary 20 to 60 px lines, all
    in one run."""
    rng = np.random.default_rng(seed)
    w, h = 2481, 3508
    page = np.clip(rng.normal(226, 14, (h, w)), 0, 255).astype(np.uint8)
    for _ in range(3000):
        x, y = int(rng.integers(0, w - 60)), int(rng.integers(0, h - 60))
        page[y:y + int(rng.integers(4, 60)), x:x + int(rng.integers(2, 30))] = int(rng.integers(0, 90))
    boxes = []
    for lo, hi, count in ((350, 600, 40), (1000, 1500, 6), (250, 340, 12), (20, 60, 30)):
        k = 0
        while k < count:
            bh = rng.uniform(lo, hi)
            x0, y0 = rng.uniform(-100, w - 100), rng.uniform(-150, h - bh + 150)
            bw = rng.uniform(40, 2600)
            if (bw + 0.6 * bh) * 32 / (1.4 * bh) > 1000:
                continue
            boxes.append([x0, y0, x0 + bw, y0 + bh])
            k += 1
    boxes = np.asarray(boxes)[rng.permutation(len(boxes))]
    return page, boxes


def beyond_fast_reach(box) -> bool:
    """The host's rule: PIL's ksize 2 ceil(max(1, scale)) + 1 either way above 31 taps, or more than
    1024 source rows in the vertical windows' bound ceil(span + 2 support) + 4."""
    reg, width = native.crop_region(box)
    sx, sy = max(1.0, (reg[2] - reg[0]) / width), max(1.0, (reg[3] - reg[1]) / 32)
    taps = 2 * int(np.ceil(max(sx, sy))) + 1
    return taps > 32 or int(np.ceil((reg[3] - reg[1]) + 2 * sy)) + 4 > 1024


def test_wide_reach_lines_crop_bit_exact(rec_latin, orc):
    """Lines past the crop kernel's reach go through the scalar wide-reach kernel: their crops equal
    the oracle's (and the reference's compiled crop_lines where it is here) byte for byte, the
    others' too, and the decodings equal those of the run without crop copies."""
    page, boxes = wide_reach_pages()
    want_wide = sum(beyond_fast_reach(b) for b in boxes)
    assert 10 <= want_wide < len(boxes)
    page_of = np.zeros(len(boxes), np.int32)
    dev = native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=256, max_width=1024, max_pages=1,
                           max_page_bytes=page.size)
    try:
        dev.set_pages([page])
        dev.arm_crops(1024)
        dev.arm_logits()
        got, lengths = dev.recognize(page_of, boxes, 1024)
        assert dev.last_stats()["wide_lines"] == want_wide
        crops = dev.crops(len(boxes), 1024)
        dev_logits = dev.logits([1024] * len(boxes), 800)
    finally:
        dev.close()
    want, _ = orc.crop_lines(page, boxes, 1024, O.CropRule.default())
    for i in range(len(boxes)):
        assert np.array_equal(crops[i], want[i]), (i, boxes[i], beyond_fast_reach(boxes[i]))
    if O.Reference.available():
        ref_crops, _ = O.Reference().crop_lines(page, boxes, 1024)
        assert np.array_equal(np.asarray(crops)[:, :, :1024], ref_crops)
    got2, lengths2, logits2 = decodings_without_crop_copies(rec_latin[0].to_blob(), [page], page_of, boxes,
                                                            max_page_bytes=page.size)
    assert_same_decodings(got, lengths, got2, lengths2, dev_logits, logits2)


def test_scheduler_runs_are_independent_of_grouping(rec_latin):
    """Lines of several pages at their ladder buckets, cut into many runs (a small column budget) or
    one: the same decodings, each line's also the same as when it is read alone."""
    pages, boxes = synth.pages(11, 3, 1200, 900, 20)
    page_of = np.repeat(np.arange(3), 20).astype(np.int32)
    allb = np.concatenate(boxes)
    blob = rec_latin[0].to_blob()
    big = native.RecDevice(blob, native.INT8, max_lines=256, max_width=2048, max_pages=4)
    small = native.RecDevice(blob, native.INT8, max_lines=7, max_width=2048, max_columns=4096, max_pages=4)
    try:
        big.set_pages(pages)
        small.set_pages(pages)
        a, la = big.recognize_lines(page_of, allb)
        b, lb = small.recognize_lines(page_of, allb)
        assert np.array_equal(la, lb)
        for x, y in zip(a, b):
            assert np.array_equal(x.ids, y.ids) and np.array_equal(x.frames, y.frames)
            assert np.array_equal(x.probs.view(np.int32), y.probs.view(np.int32))
        bws = [native.width_bucket(native.crop_region(bx)[1]) for bx in allb]
        for i in (0, 17, 33, 59):
            one, l1 = big.recognize([page_of[i]], allb[i:i + 1], bws[i])
            assert l1[0] == la[i] and np.array_equal(one[0].ids, a[i].ids)
            assert np.array_equal(one[0].probs.view(np.int32), a[i].probs.view(np.int32))
        # permuted order: each line's result is its own
        perm = np.random.default_rng(0).permutation(len(allb))
        c, lc = big.recognize_lines(page_of[perm], allb[perm])
        for j, i in enumerate(perm):
            assert np.array_equal(c[j].ids, a[i].ids) and lc[j] == la[i]
    finally:
        big.close()
        small.close()


def test_prefetched_pages_give_the_same_decodings(rec_latin):
    """Two groups of pages alternating as the reference's pipeline gives them: the next group
    prefetched (uploaded into the other page buffer beside the current group's runs), then taken by
    set_pages; a prefetch that set_pages does not take (other pages) is uploaded again.  Every
    decoding equals the one of plain set_pages, bit for bit."""
    groups = [synth.pages(31 + g, 2, 1400, 1000, 12) for g in range(2)]
    blob = rec_latin[0].to_blob()
    plain = native.RecDevice(blob, native.INT8, max_lines=64, max_width=2048, max_pages=2)
    piped = native.RecDevice(blob, native.INT8, max_lines=64, max_width=2048, max_pages=2)
    try:
        want = []
        for pages, boxes in groups:
            plain.set_pages(pages)
            page_of = np.repeat(np.arange(2), 12).astype(np.int32)
            want.append(plain.recognize_lines(page_of, np.concatenate(boxes)))
        rows = [[native.rows_read(b, 1000) for b in boxes] for _, boxes in groups]
        order = [0, 1, 0, 1, 1]
        piped.set_pages(groups[0][0], rows[0])
        for k, g in enumerate(order):
            if k > 0:
                piped.set_pages(groups[g][0], rows[g])
            nxt = order[k + 1] if k + 1 < len(order) else None
            if nxt is not None and nxt != g:
                piped.prefetch_pages(groups[nxt][0], rows[nxt])
            elif nxt is not None:
                piped.prefetch_pages(groups[1 - g][0], rows[1 - g])  # not taken: the next set_pages uploads again
            page_of = np.repeat(np.arange(2), 12).astype(np.int32)
            got, lengths = piped.recognize_lines(page_of, np.concatenate(groups[g][1]))
            wl, wlen = want[g]
            assert np.array_equal(lengths, wlen)
            for x, y in zip(got, wl):
                assert np.array_equal(x.ids, y.ids) and np.array_equal(x.frames, y.frames)
                assert np.array_equal(x.probs.view(np.int32), y.probs.view(np.int32))
    finally:
        plain.close()
        piped.close()


def test_mini_model_odd_channels_bit_exact(mini, orc, golden):
    """A recognizer whose channel counts are not multiples of 16 (padded on the device)."""
    import hashlib
    n8 = mini[0]
    crops, widths, bws = synth.crops(21, 6, 40, 200, bucket_step=8)
    dev = native.RecDevice(n8.to_blob(), native.INT8, max_lines=16, max_width=256, max_pages=1)
    try:
        dev.arm_logits()
        got, lengths = dev.recognize_crops(crops, widths, bws)
        logits = dev.logits(bws, n8.classes)
    finally:
        dev.close()
    want = oracle_lines(orc, orc.model(n8.to_blob()), crops, widths, bws)
    assert_same_lines(got, lengths, want)
    for i, g in enumerate(golden["mini_int8"]["lines"]):
        assert hashlib.sha256(logits[i][None].tobytes()).hexdigest() == g["logits_sha256"], i


def test_config3_scale_int8(dev8, orc, rec_latin):
    """Config 3: 4096 crops, widths log-uniform in [64, 1024], 32-px buckets.  Properties at full
    size (a second run is identical; each line is its own), the oracle on a sample, and the
    reference's own executor on all of them where its build travelled here."""
    crops, widths, bws = synth.crops(3000, 4096, 64, 1024, log_uniform=True)
    got, lengths = dev8.recognize_crops(crops, widths, bws)
    again, lengths2 = dev8.recognize_crops(crops, widths, bws)
    assert np.array_equal(lengths, lengths2)
    for x, y in zip(got, again):
        assert np.array_equal(x.ids, y.ids) and np.array_equal(x.probs.view(np.int32), y.probs.view(np.int32))
    m = orc.model(rec_latin[0].to_blob())
    sample = np.random.default_rng(5).choice(4096, 24, replace=False)
    want = oracle_lines(orc, m, crops[sample], widths[sample], bws[sample])
    assert_same_lines([got[i] for i in sample], lengths[sample], want)
    if O.Reference.available():
        import tempfile
        from pathlib import Path
        from carbon_rec import onnx_pb
        ref = O.Reference()
        with tempfile.TemporaryDirectory() as d:
            path = Path(d) / "rec.int8.onnx"
            onnx_pb.save(rec_latin[2], path)
            s = ref.session(path)
            for bw in np.unique(bws):
                sel = np.nonzero(bws == bw)[0]
                x = (np.float32(1.0) - crops[sel, :, :bw].astype(np.float32) / np.float32(255.0))[:, None]
                logits = s.run(x)
                lines = ref.ctc_greedy(logits, np.minimum(bw // 4, widths[sel] // 4))
                for j, i in enumerate(sel):
                    assert np.array_equal(got[i].ids, lines[j][0]) and np.array_equal(got[i].frames, lines[j][1])
                    assert np.array_equal(got[i].probs.view(np.int32), lines[j][2].view(np.int32))


def test_fp16_pages_agree_with_fp32(orc, rec_latin):
    """Crops of text-like pages through the FP16 engine against the FP32 recognizer on the same
    crops: the logits within FP16_LOGIT_TOL and, over the frames the decoder reads (within each
    line's length), at least 99.9% of frame ids agreeing.  With random weights the ids that differ
    are near ties, so the share is measured over many frames: 256 lines, ~18,000 frames."""
    pages, boxes = synth.pages(2, 4, 2480, 3508, 64)
    page_of = np.repeat(np.arange(4), 64).astype(np.int32)
    allb = np.concatenate(boxes)
    dev = native.RecDevice(rec_latin[1].to_blob(), native.FP16, max_lines=512, max_width=2048, max_pages=8,
                           max_page_bytes=4 * 2480 * 3508)
    try:
        dev.set_pages(pages)
        dev.arm_logits()
        widths = np.array([native.crop_region(b)[1] for b in allb])
        bws = ((widths + 31) // 32 * 32).astype(np.int32)
        got, lengths = dev.recognize_lines(page_of, allb, bws)
        logits = dev.logits(bws, 800)
    finally:
        dev.close()
    m32 = orc.model(rec_latin[1].to_blob())
    agree = total = 0
    worst = 0.0
    for i in range(len(allb)):
        crop, _ = orc.crop_lines(pages[page_of[i]], allb[i:i + 1], int(bws[i]))
        ref = m32.run(crop)[0]
        worst = max(worst, float(np.abs(logits[i] - ref).max()))
        n = int(lengths[i])
        agree += int((logits[i].argmax(0)[:n] == ref.argmax(0)[:n]).sum())
        total += n
    assert worst <= FP16_LOGIT_TOL and agree / total >= FP16_ID_AGREEMENT, (worst, agree, total)


def test_errors_are_reported_and_the_device_goes_on(dev8, rec_latin):
    pages, boxes = synth.pages(3, 1, 800, 600, 4)
    dev8.set_pages(pages)
    wide = np.array([[10.0, 100.0, 790.0, 120.0]])
    with pytest.raises(native.CrecError) as e:
        dev8.recognize([0], wide, 64)  # crop_lines: wider than its batch
    assert e.value.code == native.E_RANGE and "px wide, the batch 64" in str(e.value)
    with pytest.raises(native.CrecError) as e:
        dev8.recognize([5], boxes[0][:1], 2048)  # a page not set
    assert e.value.code == native.E_INVALID
    with pytest.raises(native.CrecError) as e:
        dev8.recognize([0], boxes[0][:1], 100)  # not a multiple of the width step
    assert e.value.code == native.E_INVALID
    with pytest.raises(native.CrecError) as e:
        native.RecDevice(b"CRECMDL1" + b"\0" * 64, native.INT8)
    assert e.value.code == native.E_MODEL
    with pytest.raises(native.CrecError) as e:
        native.RecDevice(rec_latin[1].to_blob(), native.INT8)  # the float blob at INT8
    assert e.value.code == native.E_MODEL
    assert not dev8.broken
    got, lengths = dev8.recognize([0, 0], boxes[0][:2], 2048)
    assert len(got) == 2 and lengths.shape == (2,)
    empty, el = dev8.recognize([], np.zeros((0, 4)), 256)
    assert empty == [] and el.shape == (0,)


def test_pageable_pinned_and_strided_pages_upload_alike(rec_latin):
    """The same pages handed as pageable arrays (staged through the library's pinned chunks), as
    page-locked memory (copied from where they are) and as views into wider images (rows further
    apart than their width), with and without row runs, by set_pages and by prefetch_pages:
    the same decodings."""
    import torch
    pages, boxes = synth.pages(41, 2, 1500, 1100, 10)
    page_of = np.repeat(np.arange(2), 10).astype(np.int32)
    allb = np.concatenate(boxes)
    rows = [native.rows_read(b, 1100) for b in boxes]
    pinned = []
    for p in pages:
        t = torch.empty(p.shape, dtype=torch.uint8, pin_memory=True)
        t.numpy()[:] = p
        pinned.append(t)
    wide = []
    for p in pages:
        w = np.full((p.shape[0], p.shape[1] + 37), 255, np.uint8)
        w[:, :p.shape[1]] = p
        wide.append(w[:, :p.shape[1]])
    dev = native.RecDevice(rec_latin[0].to_blob(), native.INT8, max_lines=64, max_width=2048, max_pages=2)
    try:
        dev.set_pages(pages)
        want = dev.recognize_lines(page_of, allb)
        for variant in ([t.numpy() for t in pinned], wide, pages):
            for r in (None, rows):
                dev.set_pages(variant, r)
                got = dev.recognize_lines(page_of, allb)
                assert np.array_equal(got[1], want[1])
                for x, y in zip(got[0], want[0]):
                    assert np.array_equal(x.ids, y.ids) and np.array_equal(x.probs.view(np.int32), y.probs.view(np.int32))
                dev.prefetch_pages(variant, r)
                dev.set_pages(variant, r)  # takes the prefetch
                assert dev.last_stats()["h2d_bytes"] > 0
                got = dev.recognize_lines(page_of, allb)
                for x, y in zip(got[0], want[0]):
                    assert np.array_equal(x.ids, y.ids) and np.array_equal(x.probs.view(np.int32), y.probs.view(np.int32))
    finally:
        dev.close()
