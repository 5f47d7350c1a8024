"""Seeded synthetic inputs of the benchmark configurations (no dataset is read).

* pages (configs 2 and 5): uint8 pages, background ~N(235, 8), `lines` text lines a page
  with heights uniform in [18, 60] px, aspect ratios in [4, 40] and rotation uniform in
  +-5 degrees; each line drawn as dark glyph strokes ~N(40, 15) along its rotated baseline,
  its box the rotated line's axis-aligned bounds (the reference's LineBox is axis-aligned,
  carbon/include/carbon/lines.h:40-42).
* crops (configs 1 and 3): 32-px line crops, background ~N(230, 10) with 3-6 px dark
  strokes ~N(40, 15), widths uniform (config 1) or log-uniform (config 3), each finished
  and padded to its bucket as the crop rule does (so they are what crop_lines gives).
"""
from __future__ import annotations

import math

import numpy as np


def page_lines(rng: np.random.Generator, width: int, height: int, n: int, hmin=18.0, hmax=60.0, amin=4.0,
               amax=40.0, max_angle=5.0):
    """(boxes [n, 4] float64, strokes [k, 5] int32: x0, y0, x1, y1, value) for one page."""
    boxes = np.zeros((n, 4), np.float64)
    strokes = []
    margin = 20
    for i in range(n):
        h = rng.uniform(hmin, hmax)
        w = min(rng.uniform(amin, amax) * h, width - 2 * margin - 2)
        ang = math.radians(rng.uniform(-max_angle, max_angle))
        rise = w * math.tan(ang)
        x0 = rng.uniform(margin, width - margin - w)
        span = h + abs(rise)
        y0 = rng.uniform(margin, max(margin + 1.0, height - margin - span))
        base = y0 + (abs(rise) if rise < 0 else 0.0)  # the line's top at its left end
        boxes[i] = (x0, y0, x0 + w, y0 + span)
        # glyph strokes along the line, 2-5 a glyph, as dense as config 1's crops: the random-weight
        # recognizer then reads about a quarter of a line's frames as characters (sparser strokes
        # decoded almost all blank, which would leave the fused head's per-frame sums idle)
        x = x0 + rng.uniform(0, 3)
        while x < x0 + w - 2:
            gw = rng.uniform(0.35, 0.6) * h  # a glyph
            k = int(rng.integers(2, 6))
            for _ in range(k):
                sx = x + rng.uniform(0, gw)
                sw = rng.uniform(0.08 * h, max(0.08 * h + 0.5, 0.16 * h))
                top = base + (sx - x0) * math.tan(ang) + rng.uniform(0.05, 0.3) * h
                sh = rng.uniform(0.45, 0.8) * h
                if rng.random() < 0.35:  # a horizontal bar instead
                    sw, sh = rng.uniform(0.3, 0.6) * h, rng.uniform(0.08 * h, max(0.08 * h + 0.5, 0.16 * h))
                v = int(np.clip(rng.normal(40, 15), 0, 255))
                strokes.append((int(sx), int(top), int(min(sx + sw, x0 + w)) + 1, int(top + sh) + 1, v))
            x += gw + rng.uniform(0.05, 0.25) * h * (3.0 if rng.random() < 0.15 else 1.0)
    return boxes, np.asarray(strokes, np.int32).reshape(-1, 5)


def draw_page(rng: np.random.Generator, width: int, height: int, strokes: np.ndarray, mean=235.0, std=8.0):
    page = np.clip(np.rint(rng.normal(mean, std, (height, width)).astype(np.float32)), 0, 255).astype(np.uint8)
    for x0, y0, x1, y1, v in strokes:
        x0, y0 = max(0, x0), max(0, y0)
        x1, y1 = min(width, x1), min(height, y1)
        if x1 > x0 and y1 > y0:
            page[y0:y1, x0:x1] = v
    return page


def pages(seed: int, count: int, width=2480, height=3508, lines=64, **kw):
    """`count` pages and their boxes: (list of [height, width] uint8, list of [lines, 4] boxes)."""
    rng = np.random.default_rng(seed)
    out_p, out_b = [], []
    for _ in range(count):
        b, s = page_lines(rng, width, height, lines, **kw)
        out_p.append(draw_page(rng, width, height, s))
        out_b.append(b)
    return out_p, out_b


def finish(crop: np.ndarray, width: int, out_width: int, flip_margin=48, flip_needs_dark=True) -> np.ndarray:
    """A crop's own width padded to out_width as carbon/src/lines.cpp:311-329 finishes it (numpy)."""
    c = np.zeros((crop.shape[0], out_width), np.uint8)
    c[:, :width] = crop[:, :width]
    h = crop.shape[0]
    border = np.concatenate([c[0, :width], c[h - 1, :width], c[:, width - 1]])
    srt = np.sort(border)
    cnt = len(srt)

    def ground(vals):
        return int(vals[cnt // 2]) if cnt % 2 else (int(vals[cnt // 2 - 1]) + int(vals[cnt // 2])) // 2

    g = ground(srt)
    body = c[:, :width].astype(np.int32)
    flip = False
    if flip_margin > 0:
        flip = int((body >= g + flip_margin).sum()) > int((body <= g - flip_margin).sum())
        if flip and flip_needs_dark:
            flip = 2 * int((body <= 127).sum()) > width * h
    if flip:
        c[:, :width] = 255 - c[:, :width]
    if width < out_width:
        gg = ground(np.sort(255 - border)) if flip else g
        c[:, width:] = gg
    return c


def crops(seed: int, n: int, wmin: int, wmax: int, log_uniform=False, bucket_step=32, height=32):
    """(crops [n, height, max bw] uint8, widths [n], bucket widths [n]) for configs 1 and 3."""
    rng = np.random.default_rng(seed)
    if log_uniform:
        ws = np.exp(rng.uniform(np.log(wmin), np.log(wmax), n))
    else:
        ws = rng.uniform(wmin, wmax, n)
    widths = np.clip((np.rint(ws / 8.0) * 8).astype(np.int32), 8, None)
    bws = ((widths + bucket_step - 1) // bucket_step * bucket_step).astype(np.int32)
    pitch = int(bws.max())
    out = np.zeros((n, height, pitch), np.uint8)
    for i in range(n):
        w = int(widths[i])
        c = rng.normal(230, 10, (height, w))
        x = 0
        while x < w:
            sw = int(rng.integers(3, 7))
            x += int(rng.integers(2, 10))
            if x >= w:
                break
            y0 = int(rng.integers(4, height // 2))
            y1 = int(rng.integers(height // 2 + 2, height - 3))
            if rng.random() < 0.7:
                c[y0:y1, x:min(w, x + sw)] = rng.normal(40, 15, (y1 - y0, min(w, x + sw) - x))
            else:
                yy = int(rng.integers(6, height - 8))
                x1 = min(w, x + int(rng.integers(5, 14)))
                c[yy:yy + sw // 2 + 1, x:x1] = rng.normal(40, 15, (sw // 2 + 1, x1 - x))
            x += sw
        c = np.clip(np.rint(c), 0, 255).astype(np.uint8)
        out[i, :, :bws[i]] = finish(c, w, int(bws[i]))
    return out, widths, bws
