"""The C restatement against the reference's own code compiled here (oracle/_ref), on fresh
seeded inputs: every comparison bit for bit.  Skipped where the reference's build is absent."""
from __future__ import annotations

import numpy as np
import pytest

from carbon_rec import model, onnx_pb, synth
from oracle import oracle as O


def test_resample_matches_reference(orc, ref):
    # the cases of tests/cpp/lines_test.cpp:89-152 of the reference: down, up, off the image
    rng = np.random.default_rng(23)
    for i in range(150):
        w, h = int(rng.integers(1, 120)), int(rng.integers(1, 120))
        img = rng.integers(0, 256, (h, w)).astype(np.uint8)
        if i % 3 == 0:
            x0, y0, x1, y1 = 0.0, 0.0, float(w), float(h)
        else:
            x0 = rng.uniform(-0.7 * w - 20, 1.2 * w)
            y0 = rng.uniform(-0.7 * h - 20, 1.2 * h)
            x1, y1 = x0 + rng.uniform(0.05, 1.6 * w + 10), y0 + rng.uniform(0.05, 1.6 * h + 10)
        ow, oh = int(rng.integers(1, 70)), int(rng.integers(1, 70))
        assert np.array_equal(orc.resample_gray(img, x0, y0, x1, y1, ow, oh),
                              ref.resample_gray(img, x0, y0, x1, y1, ow, oh, scalar=True))


@pytest.mark.parametrize("rule", [{}, {"flip_margin": 0}, {"flip_needs_dark": 0}])
def test_crop_lines_matches_reference(orc, ref, rule):
    # tests/cpp/cuda_lines_test.cpp:47-109 of the reference: 300 random boxes, two pages, one inverted
    rng = np.random.default_rng(7)
    for w, h, invert in ((1700, 2200, False), (900, 640, True)):
        page = np.clip(rng.normal(235, 8, (h, w)), 0, 255).astype(np.uint8)
        for _ in range(200):
            x, y = int(rng.integers(0, w - 20)), int(rng.integers(0, h - 10))
            page[y:y + int(rng.integers(3, 20)), x:x + int(rng.integers(2, 8))] = int(rng.integers(0, 80))
        if invert:
            page = 255 - page
        boxes = []
        while len(boxes) < 150:
            bh = rng.uniform(8, 60)
            x0, y0 = rng.uniform(-30, w - 10), rng.uniform(-20, h - 5)
            bw = rng.uniform(5, 900)
            if (bw + 0.6 * bh) * 32 / (1.4 * bh) > 2000:
                continue
            boxes.append([x0, y0, x0 + bw, y0 + bh])
        b = np.asarray(boxes)
        r = O.CropRule.default(**rule)
        a, wa = orc.crop_lines(page, b, 2048, r)
        c, wc = ref.crop_lines(page, b, 2048, r)
        assert np.array_equal(wa, wc)
        assert np.array_equal(a, c)


def test_ctc_greedy_matches_reference(orc, ref):
    # tests/cpp/cpu_test.cpp:1162-1210 of the reference: grids with ties, narrow and wide, blank-heavy
    rng = np.random.default_rng(17)
    for spread in (0.5, 3.0):
        for classes in (1, 7, 800):
            for frames in (1, 13, 131, 263):
                l = (rng.integers(-24, 25, (2, classes, frames)) * spread).astype(np.float32)
                l[:, 0, ::3] += 30.0
                lens = np.array([frames - frames // 5, frames], np.int32)
                got, _, _ = orc.ctc_greedy(l, lens)
                want = ref.ctc_greedy(l, lens)
                for (a, b, c), (x, y, z) in zip(got, want):
                    assert np.array_equal(a, x) and np.array_equal(b, y)
                    assert np.array_equal(c.view(np.int32), z.view(np.int32))


def test_ctc_topk_matches_reference(orc, ref):
    """The beam's candidates (cpu::ctc_topk, carbon::frame_candidates): tie-heavy integer grids and
    float logits, k from 0 to classes - 1, lines cut short of their frames."""
    rng = np.random.default_rng(29)
    for classes, frames in ((2, 5), (7, 40), (33, 17), (800, 72)):
        for grid in (True, False):
            l = (rng.integers(-12, 13, (classes, frames)) * 0.25 if grid else rng.normal(0, 3, (classes, frames)))
            l = l.astype(np.float32)
            for k in sorted({0, 1, min(5, classes - 1), min(16, classes - 1), classes - 1}):
                t_n = frames - frames // 4
                a = orc.ctc_topk(l, t_n, k)
                b = ref.ctc_topk(l, t_n, k)
                assert np.array_equal(a[0], b[0]), (classes, k)
                assert np.array_equal(a[1].view(np.int32), b[1].view(np.int32)), (classes, k)
                assert np.array_equal(a[2].view(np.int32), b[2].view(np.int32)), (classes, k)


@pytest.mark.parametrize("tag", ["int8", "fp32"])
def test_rec_latin_matches_reference(orc, ref, rec_latin, tmp_path, tag):
    n8, n32, i8, fp = rec_latin
    path = tmp_path / f"rec.{tag}.onnx"
    onnx_pb.save(i8 if tag == "int8" else fp, path)
    crops, widths, bws = synth.crops(31, 6, 32, 400, bucket_step=8)
    m = orc.model((n8 if tag == "int8" else n32).to_blob())
    s = ref.session(path)
    for i in range(len(crops)):
        c = crops[i:i + 1, :, :int(bws[i])]
        x = (np.float32(1.0) - c.astype(np.float32) / np.float32(255.0))[:, None]
        assert np.array_equal(m.run(c), s.run(x))


def test_reference_fixture_through_the_compile(orc, ref):
    # the reference's own miniature Q/DQ recognizer (z != 0 residuals, u8 logits) through this
    # package's ONNX compile and the restated executor
    from pathlib import Path
    from carbon_rec import netdef
    f = O.REFERENCE_ROOT / "tests" / "data" / "native-rec.int8.onnx"
    if not f.exists():
        pytest.skip("the reference's test data is not here")
    net = netdef.load(f)
    rng = np.random.default_rng(9)
    b = rng.integers(0, 256, (3, 32, 72)).astype(np.uint8)
    x = (np.float32(1.0) - b.astype(np.float32) / np.float32(255.0))[:, None]
    assert np.array_equal(orc.model(net.to_blob()).run(b), ref.session(f).run(x))
