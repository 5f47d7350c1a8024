"""The C restatement (oracle/rec_oracle.c) against the reference's own outputs stored in
tests/golden/golden.json (made by tests/golden/make_golden.py from the compiled reference)
and against the golden values of the reference's own tests."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from carbon_rec import model, netdef, synth
from oracle import oracle as O

import importlib.util
import sys
from pathlib import Path

_spec = importlib.util.spec_from_file_location("make_golden", Path(__file__).parent / "golden" / "make_golden.py")
make_golden = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(make_golden)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_crop_region_reference_test_numbers(orc):
    # tests/cpp/lines_test.cpp:37-49 of the reference: y0 44, y1 86, width 248, 62 frames
    reg, w = orc.crop_region([100, 50, 400, 80])
    assert reg[1] == 44.0 and reg[3] == 86.0 and w == 248 and w // 4 == 62
    assert reg[0] <= 100 - 0.3 * 30 and reg[2] >= 400 + 0.3 * 30
    assert abs((reg[2] - reg[0]) / (reg[3] - reg[1]) - w / 32.0) < 1e-9


def test_crop_region_sweep(orc, golden):
    for case in golden["crop_region_sweep"]:
        reg, w = orc.crop_region(case["box"])
        assert w == case["width"]
        assert list(reg) == case["region"]  # bit for bit


@pytest.mark.parametrize("name,rule", [("default", {}), ("no_flip", {"flip_margin": 0}),
                                       ("flip_any", {"flip_needs_dark": 0})])
def test_crop_lines_golden(orc, golden, name, rule):
    page, boxes = make_golden.crop_cases()
    crops, widths = orc.crop_lines(page, boxes, 1024, O.CropRule.default(**rule))
    g = golden[f"crop_lines_{name}"]
    assert widths.tolist() == g["widths"]
    assert [sha(c) for c in crops] == g["sha256"]


def test_identity_resample_keeps_every_byte(orc):
    # tests/cpp/lines_test.cpp:51-57 of the reference
    p = (np.arange(40 * 32) * 37 % 256).astype(np.uint8).reshape(32, 40)
    assert np.array_equal(orc.resample_gray(p, 0, 0, 40, 32, 40, 32), p)


def test_ground_is_the_median_of_the_border(orc):
    # tests/cpp/lines_test.cpp:182-192 of the reference
    c = np.array([10, 10, 10, 10, 0, 0, 0, 30, 20, 20, 20, 20], np.uint8)
    assert orc.crop_ground(c, 4, 3, 4) == 20
    assert orc.crop_ground(np.array([10, 30, 10, 30], np.uint8), 2, 2, 2) == 30
    assert orc.crop_ground(np.array([11, 11, 20, 20], np.uint8), 2, 2, 2) == 15


def test_light_on_dark_is_flipped_then_padded(orc):
    # tests/cpp/lines_test.cpp:194-215 of the reference
    c = np.full((32, 24), 7, np.uint8)
    for y in range(10, 22):
        for x in range(3, 13, 3):
            c[y, x] = 230
    orc.finish_crop(c, 16, O.CropRule.default())
    assert c[0, 0] == 248 and c[10, 3] == 25 and c[5, 20] == 248


def test_paper_outside_the_page(orc):
    # tests/cpp/lines_test.cpp:154-162 of the reference
    page = np.full((100, 200), 255, np.uint8)
    crops, w = orc.crop_lines(page, np.array([[-50, -20, 300, 140]], np.float64), 512)
    assert (crops == 255).all()


def test_width_ladder(orc):
    # tests/cpp/pipeline_test.cpp:20-33 of the reference
    ladder = [32, 48, 64, 88, 120, 160, 208, 272, 360, 472, 616, 808, 1056, 1376, 1792, 2048]
    prev = 0
    for b in ladder:
        assert orc.width_bucket(b) == b
        assert orc.width_bucket(prev + 1) == b
        prev = b
    assert orc.width_bucket(8) == 32 and orc.width_bucket(2049) == 2056


def test_ctc_collapse_and_ties(orc):
    # tests/cpp/lines_test.cpp:257-275 of the reference
    classes, frames = 4, 6
    best = [0, 2, 2, 0, 2, 3]
    logits = np.zeros((1, classes, frames), np.float32)
    for t, b in enumerate(best):
        logits[0, b, t] = 5.0
    lines, _, _ = orc.ctc_greedy(logits, [frames])
    assert lines[0][0].tolist() == [2, 2, 3] and lines[0][1].tolist() == [1, 4, 5]
    assert np.allclose(lines[0][2], np.exp(5.0) / (np.exp(5.0) + 3), atol=1e-6)
    assert orc.ctc_greedy(logits, [3])[0][0][0].tolist() == [2]
    assert len(orc.ctc_greedy(np.ones((1, classes, frames), np.float32), [frames])[0][0][0]) == 0


def test_exp_neg_skip_bound(orc):
    # tests/cpp/cpu_test.cpp:1141-1160 of the reference: exp_neg(0) = 1, terms past -17 under 2^-24
    assert orc.exp_neg(0.0) == 1.0
    xs = np.linspace(-87.0, -17.0, 20001, dtype=np.float32)
    assert max(orc.exp_neg(float(x)) for x in xs) < 2.0 ** -24


def test_ctc_greedy_golden(orc, golden):
    for (l, lengths), want in zip(make_golden.ctc_cases(), golden["ctc_greedy"]):
        lines, _, _ = orc.ctc_greedy(l, lengths)
        for (ids, fr, pr), w in zip(lines, want):
            assert ids.tolist() == w["ids"] and fr.tolist() == w["frames"]
            assert pr.tolist() == w["probs"]  # bit for bit


def test_rec_latin_blob_is_the_golden_model(rec_latin, golden):
    n8, n32, _, _ = rec_latin
    assert hashlib.sha256(n8.to_blob()).hexdigest() == golden["rec_latin_blob_sha256"]["int8"]
    assert hashlib.sha256(n32.to_blob()).hexdigest() == golden["rec_latin_blob_sha256"]["fp32"]


@pytest.mark.parametrize("tag", ["int8", "fp32"])
def test_rec_latin_logits_and_ctc_golden(orc, rec_latin, golden, tag):
    n8, n32, _, _ = rec_latin
    m = orc.model((n8 if tag == "int8" else n32).to_blob())
    crops, widths, bws = make_golden.rec_crops()
    for i, want in enumerate(golden["rec_latin_config1"]):
        bw = want["bw"]
        logits = m.run(crops[i:i + 1, :, :bw])
        assert sha(logits) == want[tag]["logits_sha256"]
        lines, _, _ = orc.ctc_greedy(logits, [min(logits.shape[2], want["width"] // 4)])
        ids, fr, pr = lines[0]
        assert ids.tolist() == want[tag]["ids"] and fr.tolist() == want[tag]["frames"]
        assert pr.tolist() == want[tag]["probs"]


def test_mini_int8_golden(orc, mini, golden):
    n8 = mini[0]
    assert hashlib.sha256(n8.to_blob()).hexdigest() == golden["mini_int8"]["blob_sha256"]
    m = orc.model(n8.to_blob())
    crops, widths, bws = synth.crops(21, 6, 40, 200, bucket_step=8)
    for i, want in enumerate(golden["mini_int8"]["lines"]):
        assert sha(m.run(crops[i:i + 1, :, :want["bw"]])) == want["logits_sha256"]


def test_synth_page_lines_read_as_text(orc, rec_latin):
    """The bench's synthetic pages draw glyphs dense enough that the random-weight recognizer
    reads a share of each line's frames as characters (21% on these 32 lines; 20% on config 1's
    crops): with near-blank lines the fused head's per-frame class-order sums would hardly run
    and the bench would not measure them."""
    pages, boxes = synth.pages(5000, 1, 2480, 3508, 32)
    m = orc.model(rec_latin[0].to_blob())
    crops, widths = orc.crop_lines(pages[0], boxes[0], 1024)
    chars = frames = 0
    for i in range(len(boxes[0])):
        bw = int((widths[i] + 31) // 32 * 32)
        logits = m.run(crops[i:i + 1, :, :bw])
        n = min(bw // 4, int(widths[i]) // 4)
        chars += int((logits[0].argmax(0)[:n] != 0).sum())
        frames += n
    assert 0.1 <= chars / frames <= 0.5, (chars, frames)
