"""Writes tests/golden/golden.json: outputs of the reference's own code on seeded inputs.

Run in a checkout where the reference's sources are present and oracle/_ref was built
from them (oracle/ref.mk; `python -c "import oracle.oracle as o; o.build()"`):

    python tests/golden/make_golden.py

Every value here comes from oracle/_ref/libcarbon_ref.so, i.e. the reference's own
crop_lines, crop_region, ctc_greedy and native executor compiled from its sources.
Large arrays are stored as SHA-256 digests; the tests recompute the same inputs from
the same seeds and compare digests.  The GPU box never runs this script.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "carbon-ocr_b200"))

from carbon_rec import model, netdef, onnx_pb, synth  # noqa: E402
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent / "golden.json"
MODELS = Path(__file__).resolve().parent / "_models"  # scratch, git-ignored


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def crop_cases():
    """Seed 7: a 700 x 300 page of random bytes with a dark band, and 60 boxes (inside, across the
    edges, off the page, light-on-dark), the crop rule's defaults."""
    rng = np.random.default_rng(7)
    page = rng.integers(0, 256, (300, 700)).astype(np.uint8)
    page[100:160, :] = (page[100:160, :] // 8).astype(np.uint8)  # a dark band (flip candidates)
    page[110:150, 40:660:9] = 235
    boxes = []
    while len(boxes) < 60:
        h = rng.uniform(6, 60)
        x0 = rng.uniform(-40, 680)
        y0 = rng.uniform(-20, 290)
        w = rng.uniform(4, 500)
        if (w + 0.6 * h) * 32 / (1.4 * h) > 1000:  # crops up to the batch width of 1024
            continue
        boxes.append([x0, y0, x0 + w, y0 + h])
    boxes[0] = [40.0, 112.0, 650.0, 148.0]  # the dark band: light text on dark
    boxes[1] = [-50.0, -20.0, 300.0, 140.0]  # mostly off the page
    return page, np.asarray(boxes, np.float64)


def ctc_cases():
    """Seed 17: logits on a coarse grid (ties), blank-heavy, [3, 7, 13] and [2, 800, 40]."""
    rng = np.random.default_rng(17)
    out = []
    for n, classes, frames, spread in ((3, 7, 13, 0.5), (2, 800, 40, 3.0)):
        l = (rng.integers(-24, 25, (n, classes, frames)) * spread).astype(np.float32)
        l[:, 0, ::3] += 30.0
        lengths = np.array([frames - frames // 5] + [frames] * (n - 1), np.int32)
        out.append((l, lengths))
    return out


def rec_crops():
    """Config 1's crops, seed 1: 8 lines, widths in [96, 640], 32-px buckets."""
    return synth.crops(1, 8, 96, 640)


def main() -> None:
    if not O.Reference.available():
        sys.exit("oracle/_ref/libcarbon_ref.so is not built (needs the reference's sources)")
    ref = O.Reference()
    g: dict = {}

    # crop_region: the reference test's numbers and a seeded sweep
    reg, w = ref.crop_region([100, 50, 400, 80])
    g["crop_region_100_50_400_80"] = {"region": list(reg), "width": w}
    rng = np.random.default_rng(3)
    sweep = []
    for _ in range(200):
        h = rng.uniform(4, 120)
        x0, y0 = rng.uniform(-100, 2000), rng.uniform(-50, 3000)
        box = [x0, y0, x0 + rng.uniform(1, 2400), y0 + h]
        r, ww = ref.crop_region(box)
        sweep.append({"box": box, "region": list(r), "width": ww})
    g["crop_region_sweep"] = sweep

    # crop_lines on the seeded page: widths and each crop's digest, out_width 1024, both flip rules
    page, boxes = crop_cases()
    for name, rule in (("default", O.CropRule.default()), ("no_flip", O.CropRule.default(flip_margin=0)),
                       ("flip_any", O.CropRule.default(flip_needs_dark=0))):
        crops, widths = ref.crop_lines(page, boxes, 1024, rule)
        g[f"crop_lines_{name}"] = {"widths": widths.tolist(), "sha256": [sha(c) for c in crops]}

    # ctc_greedy
    cases = []
    for l, lengths in ctc_cases():
        lines = ref.ctc_greedy(l, lengths)
        cases.append([{"ids": a.tolist(), "frames": b.tolist(), "probs": [float(x) for x in c]} for a, b, c in lines])
    g["ctc_greedy"] = cases

    # rec-latin (seed 0) INT8 and FP32 on the reference executor: logits digests and CTC results
    MODELS.mkdir(exist_ok=True)
    _, _, fp, i8 = model.make_rec_latin(0)
    onnx_pb.save(fp, MODELS / "rec-latin.onnx")
    onnx_pb.save(i8, MODELS / "rec-latin.int8.onnx")
    g["rec_latin_blob_sha256"] = {"int8": hashlib.sha256(netdef.compile_model(i8).to_blob()).hexdigest(),
                                  "fp32": hashlib.sha256(netdef.compile_model(fp).to_blob()).hexdigest()}
    crops, widths, bws = rec_crops()
    recs = []
    for i in range(len(crops)):
        bw = int(bws[i])
        c = crops[i:i + 1, :, :bw]
        x = (np.float32(1.0) - c.astype(np.float32) / np.float32(255.0))[:, None]
        entry = {"width": int(widths[i]), "bw": bw}
        for tag, f in (("int8", "rec-latin.int8.onnx"), ("fp32", "rec-latin.onnx")):
            logits = ref.session(MODELS / f).run(x)
            t = logits.shape[2]
            lens = np.array([min(t, int(widths[i]) // 4)], np.int32)
            (ids, fr, pr), = ref.ctc_greedy(logits, lens)
            entry[tag] = {"logits_sha256": sha(logits), "ids": ids.tolist(), "frames": fr.tolist(),
                          "probs": [float(v) for v in pr]}
        recs.append(entry)
    g["rec_latin_config1"] = recs

    # the reference's own miniature INT8 recognizer fixture, on inputs made of bytes
    fixture = O.REFERENCE_ROOT / "tests" / "data" / "native-rec.int8.onnx"
    if fixture.exists():
        rng = np.random.default_rng(9)
        b = rng.integers(0, 256, (3, 32, 72)).astype(np.uint8)
        b[:, 8:24, 10:60] //= 6
        x = (np.float32(1.0) - b.astype(np.float32) / np.float32(255.0))[:, None]
        logits = ref.session(fixture).run(x)
        g["native_rec_int8_fixture"] = {"blob_sha256": hashlib.sha256(netdef.load(fixture).to_blob()).hexdigest(),
                                        "logits_sha256": sha(logits), "shape": list(logits.shape)}
    # a miniature recognizer of this package's own (odd channel counts, 11 classes), INT8, seed 4
    _, _, mfp, m8 = model.make_mini(4)
    onnx_pb.save(m8, MODELS / "mini.int8.onnx")
    crops, widths, bws = synth.crops(21, 6, 40, 200, bucket_step=8)
    mini = []
    for i in range(len(crops)):
        bw = int(bws[i])
        x = (np.float32(1.0) - crops[i:i + 1, :, :bw].astype(np.float32) / np.float32(255.0))[:, None]
        logits = ref.session(MODELS / "mini.int8.onnx").run(x)
        mini.append({"bw": bw, "logits_sha256": sha(logits)})
    g["mini_int8"] = {"blob_sha256": hashlib.sha256(netdef.compile_model(m8).to_blob()).hexdigest(), "lines": mini}
    OUT.write_text(json.dumps(g, indent=1))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
