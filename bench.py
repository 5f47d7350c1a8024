#!/usr/bin/env python
"""Throughput of rec-latin line recognition (crop + recognizer + fused greedy CTC) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the 1/2/4/8-GPU one; config 2 is its 16-page slice):
1024 synthetic 2480 x 3508 pages x 64 lines (65,536 lines), sharded by page over the N
ranks (strong scaling: the total is fixed).  Every page slot is a buffer of its own (1024
of them, 8.9 GB); their contents repeat 32 distinct seeded pages (seed 5000: background
~N(235, 8), lines 18-60 px high, aspect 4-40, +-5 degrees, glyph strokes dense enough that
about a quarter of the frames decode to characters), slot s holding page s % 32 and its 64
boxes; each line is read at its 32-px bucket (up to 1024).  A step is every line of the
rank's shard: cropped from its page, recognized, decoded; only ids, frames and
probabilities leave the GPU.

value: lines per second of the whole job (total lines / max over ranks of the device time,
CUDA events on the library's stream), INT8, the rank's pages resident in HBM (one device
buffer a slot).  The per-kernel profile behind `roofline` and `layers` comes from the same
steps run once more with the library's per-launch events on, outside the timed region.
e2e: the same through the public API with the host in the loop, as the reference's pipeline
drives its recognizer: the shard's pages in groups of --group pages, pageable host memory
(one buffer a slot); a group's step takes the pages prefetched beside the previous group
(set_pages), prefetches the next group's (their rows staged through pinned chunks and sent
while this group's runs go on), recognizes the group's lines and reads the decodings back.
The FP16 engine's numbers are reported beside the INT8 ones.

--impl reference: the reference's own CPU implementation of the path (oracle/_ref, the
int8 native executor with crop_lines and ctc_greedy, one pinned single-threaded session a
host core) on a bounded sample of the same workload, each step the 2,048 lines of the 32
distinct pages; rank 0 only.  It loads nothing of this repository's CUDA library (crop
widths come from the reference's own crop_region).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "carbon-ocr_b200"))

METRIC = "text lines/sec (rec-latin INT8 & FP16, crop+CTC fused) at 1/2/4/8 B200; % TC peak"
PAGES_TOTAL, LINES_PER_PAGE, DISTINCT, SEED = 1024, 64, 32, 5000
PAGE_W, PAGE_H = 2480, 3508
WORKLOAD = ("config5: 1024 synthetic 2480x3508 pages x 64 lines (65,536 lines), rec-latin crop+trunk+fused CTC, "
            "32-px buckets to 1024, sharded by page; one buffer a page slot (contents: 32 distinct seeded pages, "
            "seed 5000, text-like glyphs: ~25% of frames decode to characters)")


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--max-columns", type=int, default=1 << 23, help="input columns a device run at most (the scheduler's run size)")
    ap.add_argument("--max-lines", type=int, default=32768)
    ap.add_argument("--pages", type=int, default=PAGES_TOTAL, help="page slots of the whole job (1024: config 5)")
    ap.add_argument("--group", type=int, default=64, help="pages a set_pages group in the e2e leg")
    ap.add_argument("--no-fp16", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="config 4's kernel sweep instead (one GPU)")
    return ap.parse_args(argv)


def config_of(args, world: int) -> dict:
    """The workload both arms report (the reference arm's bounded sample is described in its
    cpu_baseline)."""
    return {"workload": WORKLOAD if args.pages == PAGES_TOTAL else
            f"{args.pages} of config 5's pages ({args.pages * LINES_PER_PAGE} lines)",
            "lines": args.pages * LINES_PER_PAGE, "parallelism": f"pages/{world}",
            "l2": "inputs larger than L2 (8.9 GB of pages, GB-scale activations)",
            "max_columns_per_run": args.max_columns, "e2e_group_pages": args.group}


def content(crop_width):
    """The 32 distinct pages, their boxes, the rows their crops read, and each box's bucket width
    (crop width rounded up to 32 px, the width from `crop_width(box)`)."""
    from carbon_rec import synth
    pages, boxes = synth.pages(SEED, DISTINCT, PAGE_W, PAGE_H, LINES_PER_PAGE)
    bws = [((np.array([crop_width(b) for b in bx]) + 31) // 32 * 32).astype(np.int32) for bx in boxes]
    return pages, boxes, bws


def shard(rank: int, world: int, pages_total: int):
    """The rank's page slots (slot s holds content page s % DISTINCT)."""
    return list(range(rank * pages_total // world, (rank + 1) * pages_total // world))


def lines_of(slots, boxes, bws, first: int = 0):
    """Every line of the given slots: page index (first + the slot's place among them), box, bucket."""
    page_of = np.concatenate([np.full(LINES_PER_PAGE, first + k, np.int32) for k in range(len(slots))])
    allb = np.concatenate([boxes[s % DISTINCT] for s in slots])
    bw = np.concatenate([bws[s % DISTINCT] for s in slots]).astype(np.int32)
    return page_of, allb, bw


def rows_read(boxes):
    from carbon_rec import native
    return [native.rows_read(b, PAGE_H) for b in boxes]


def reduce_max(v: float, world: int, device: str) -> float:
    """The job's time: the maximum of every rank's (a collective; every rank calls it)."""
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(v: float, world: int, device: str) -> float:
    """A count summed over the ranks (a collective; every rank calls it)."""
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# measured by ncu: dram__bytes_read.sum + dram__bytes_write.sum of the 11 conv_gemm launches of
# one 524,288-column run of 128 config-5 pages, 630.4 MB, / 11,
# x 4 (a 2,097,152-column run); scaled by columns to the bench's runs below (a lower bound: at the
# capture's size the outputs mostly stay in L2)
CONV_TRAFFIC_PER_LAUNCH = 630.4e6 / 11 * 4


class ClockSampler:
    """nvidia-smi samples of the SM clock and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.lines = gpu, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "of measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "of fallback"


def crop_source_bytes(boxes):
    """The page bytes a line's filter windows touch (rows x columns of its crop region widened by
    the resampler's support, clipped to the page): the crop's algorithmic read."""
    from carbon_rec import native
    total = 0
    for b in boxes:
        reg, w = native.crop_region(b)
        sx = max(1.0, (reg[2] - reg[0]) / w)
        sy = max(1.0, (reg[3] - reg[1]) / 32)
        x0, x1 = max(0, int(np.floor(reg[0] - sx))), min(PAGE_W, int(np.ceil(reg[2] + sx)))
        y0, y1 = max(0, int(np.floor(reg[1] - sy))), min(PAGE_H, int(np.ceil(reg[3] + sy)))
        total += max(0, x1 - x0) * max(0, y1 - y0)
    return total


def reference_sample(ref, model_path, pages, boxes, bws, cores: int, rounds: int):
    """One bounded sample of the workload on the reference's CPU path: the 2,048 lines of the 32
    distinct pages, `cores` pinned single-threaded workers, `rounds` passes: (seconds, lines)."""
    page_of = np.repeat(np.arange(DISTINCT), LINES_PER_PAGE).astype(np.int32)
    return ref.bench_pages(model_path, pages, page_of, np.concatenate(boxes), np.concatenate(bws), threads=cores,
                           rounds=rounds)


def cpu_baseline(pages, boxes, bws, target_s=12.0):
    """The reference's CPU path (oracle/_ref) on a bounded sample, all host cores."""
    from oracle import oracle as O
    from carbon_rec import model, onnx_pb
    if not O.Reference.available():
        return None, "oracle/_ref (the reference compiled from its sources) is not on this machine"
    import tempfile
    ref = O.Reference()
    cores = len(os.sched_getaffinity(0))
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "rec-latin.int8.onnx"
        onnx_pb.save(model.make_rec_latin(0)[3], path)
        t1, _ = reference_sample(ref, path, pages, boxes, bws, cores, 1)
        rounds = max(1, min(200, int(target_s / max(t1, 1e-3))))
        secs, done = reference_sample(ref, path, pages, boxes, bws, cores, rounds)
    return {"value": done / secs, "unit": "lines/s", "cores": cores, "kind": "reference",
            "sample": f"{DISTINCT * LINES_PER_PAGE} lines (the 32 distinct pages' 64 lines each, the same line "
                      f"distribution as config 5) x {rounds} passes, crop_lines + int8 native executor + ctc_greedy "
                      f"(oracle/_ref: the reference's CPU code compiled from its sources), {cores} pinned "
                      f"single-threaded workers, {secs:.1f} s; the box's host CPU, not the reference's published i7"}, None


def run_reference(args, rank: int, world: int):
    """The reference arm: rank 0 times the reference's CPU path; the other ranks do nothing."""
    if rank != 0:
        return 0
    base, why, secs = None, None, 0.0
    try:
        from oracle import oracle as O
        from carbon_rec import model, onnx_pb
        import tempfile
        if not O.Reference.available():
            why = "oracle/_ref (the reference compiled from its sources) is not on this machine"
        else:
            ref = O.Reference()
            pages, boxes, bws = content(lambda b: ref.crop_region(b)[1])
            cores = len(os.sched_getaffinity(0))
            times = []
            with tempfile.TemporaryDirectory() as d:
                path = Path(d) / "rec-latin.int8.onnx"
                onnx_pb.save(model.make_rec_latin(0)[3], path)
                for _ in range(args.warmup):
                    reference_sample(ref, path, pages, boxes, bws, cores, 1)
                for _ in range(args.steps):
                    times.append(reference_sample(ref, path, pages, boxes, bws, cores, 1))
            secs = sum(t for t, _ in times)
            lines = sum(d for _, d in times)
            base = {"value": lines / secs, "unit": "lines/s", "cores": cores, "kind": "reference",
                    "sample": f"each step: {DISTINCT * LINES_PER_PAGE} lines (the 32 distinct pages' 64 lines each, "
                              f"the same line distribution as config 5), crop_lines + int8 native executor + "
                              f"ctc_greedy (oracle/_ref), {cores} pinned single-threaded workers"}
    except Exception as e:  # noqa: BLE001
        why = f"{type(e).__name__}: {e}"
    if base is None:
        print(json.dumps({"impl": "reference", "unavailable": why}))
        return 0
    out = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "lines/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * secs / max(1, args.steps),
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8xs8->s32",
           "data": "synthetic (seeded pages, random-init rec-latin weights, seed 0)", "config": config_of(args, world),
           "cpu_baseline": base,
           "e2e": {"value": base["value"], "unit": "lines/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out))
    return 0


def run_sweep(args) -> int:
    """3x3 stride-1 convolutions C -> C for N = 256 lines of [H][W][C],
    C in {32, 64, 128, 256}, H in {8, 16, 32}, W in {128, 512, 1024}, INT8 and FP16, through the
    recognizer's implicit-GEMM kernel (crec_conv_sweep, inputs resident, the mean of `steps` launches
    after one warm-up, CUDA events): TOPS and the fraction of this GPU's measured tcgen05 rate."""
    import torch  # noqa: F401  (the CUDA context)
    from carbon_rec import model, native, netdef
    peaks = {native.INT8: native.mma_peak(0, native.INT8, 256), native.FP16: native.mma_peak(0, native.FP16, 256)}
    rng = np.random.default_rng(4)
    n = 256
    base8 = rng.integers(0, 256, n * 32 * 1024 * 256, dtype=np.uint8)
    base16 = (base8[: n * 32 * 1024 * 256].view(np.int8).astype(np.float16) / np.float16(40.0))
    rows = []
    for prec, name in ((native.INT8, "int8"), (native.FP16, "fp16")):
        for c in (32, 64, 128, 256):
            for h in (8, 16, 32):
                for w in (128, 512, 1024):
                    fp, i8, _ = model.make_conv(c, c, h, seed=c + h + w)
                    blob = netdef.compile_model(i8 if prec == native.INT8 else fp).to_blob()
                    size = n * h * w * c
                    x = (base8 if prec == native.INT8 else base16)[:size].reshape(n, h, w, c)
                    _, ms = native.conv_sweep(blob, prec, x, c, repeat=max(1, args.steps))
                    ops = 2.0 * n * h * w * c * c * 9
                    tops = ops / (ms * 1e-3) / 1e12
                    rows.append({"precision": name, "c": c, "h": h, "w": w, "ms": round(ms, 4), "tops": round(tops, 1),
                                 "frac": round(tops / peaks[prec], 4)})
    # the head GEMM [N T, K] x [K, classes] fused with the frames' argmax and CTC probabilities
    # (crec_head_sweep): config 4's [256 x 256, 256] x [256, 800] and the reference's GPU-head cases' K
    # and class counts at the same N T
    heads = []
    frames = n * 256
    for prec, name in ((native.INT8, "int8"), (native.FP16, "fp16")):
        for k, classes in ((256, 800), (128, 33), (192, 1500 if prec == native.FP16 else 1000), (320, 400)):
            hr = np.random.default_rng(k + classes)
            w = hr.normal(0.0, 0.06, (classes, k)).astype(np.float16).astype(np.float32)
            b = hr.normal(0.0, 0.5, classes).astype(np.float32)
            f = hr.normal(0.0, 1.0, (frames, k)).astype(np.float16)
            fp, i8, (xs, xz) = model.make_head(k, classes, w, b, f[:4096].astype(np.float32).T[None, :, None, :])
            if prec == native.INT8:
                x = np.clip(np.rint(f.astype(np.float32) / np.float32(xs)) + xz, 0, 255).astype(np.uint8)
            else:
                x = f
            blob = netdef.compile_model(i8 if prec == native.INT8 else fp).to_blob()
            _, _, _, ms = native.head_sweep(blob, prec, x, classes, repeat=max(1, args.steps))
            tops = 2.0 * frames * k * classes / (ms * 1e-3) / 1e12
            heads.append({"precision": name, "frames": frames, "k": k, "classes": classes, "ms": round(ms, 4),
                          "tops": round(tops, 1), "frac": round(tops / peaks[prec], 4)})
    out = {"metric": "config 4 kernel sweep: 3x3 s1 implicit-GEMM conv TOPS (N=256 lines)", "unit": "TOP/s",
           "peaks_measured": {"int8_n256_tops": peaks[native.INT8], "fp16_n256_tflops": peaks[native.FP16]},
           "timing": f"CUDA events, mean of {max(1, args.steps)} launches after a warm-up, inputs resident",
           "shapes": rows, "heads": heads}
    print(json.dumps(out))
    return 0


def main() -> int:
    args = parse()
    if args.sweep:
        return run_sweep(args)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world != args.gpus and "WORLD_SIZE" in os.environ:
        args.gpus = world
    import torch
    import torch.distributed as dist
    from carbon_rec import model, native, netdef

    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    pages, boxes, bws = content(lambda b: native.crop_region(b)[1])
    rows = rows_read(boxes)
    slots = shard(rank, world, args.pages)
    page_of, allb, bw_all = lines_of(slots, boxes, bws)
    _, _, fp, i8 = model.make_rec_latin(0)
    blobs = {"int8": netdef.compile_model(i8).to_blob(), "fp16": netdef.compile_model(fp).to_blob()}
    # the shard's pages in HBM, a buffer a slot (the device-time leg)
    dev_pages = []
    for s in slots:
        t = torch.empty((PAGE_H, PAGE_W), dtype=torch.uint8, device="cuda")
        t.copy_(torch.from_numpy(pages[s % DISTINCT]))
        dev_pages.append(t)
    # and in pageable host memory, a buffer a slot (the e2e leg), in groups of --group pages
    host_pages = [] if args.no_e2e else [pages[s % DISTINCT].copy() for s in slots]
    groups = [list(range(g, min(g + args.group, len(slots)))) for g in range(0, len(slots), args.group)]
    group_lines = [lines_of([slots[k] for k in g], boxes, bws) for g in groups]
    group_rows = [[rows[slots[k] % DISTINCT] for k in g] for g in groups]
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        return reduce_max(v, world, "cuda")

    def timed(dev, fn, steps):
        stream = torch.cuda.ExternalStream(dev.stream)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(steps):
            fn()
        end.record(stream)
        torch.cuda.synchronize()
        barrier()
        return start.elapsed_time(end) / 1000.0

    results = {}
    clocks = None
    for prec in (["int8"] if args.no_fp16 else ["int8", "fp16"]):
        dev = native.RecDevice(blobs[prec], native.INT8 if prec == "int8" else native.FP16, device=local,
                               max_lines=args.max_lines, max_width=1024, max_columns=args.max_columns,
                               max_pages=max(len(slots), args.group), max_page_bytes=args.group * PAGE_W * PAGE_H)
        dev.set_pages_device([(t.data_ptr(), PAGE_W, PAGE_H, PAGE_W) for t in dev_pages])
        step = lambda: dev.recognize_lines(page_of, allb, bw_all, flat=True)  # noqa: E731
        for _ in range(args.warmup):
            step()
        r = {}
        if prec == "int8":
            with ClockSampler(local) as cs:
                secs = timed(dev, step, args.steps)
            clocks = cs.summary()
        else:
            secs = timed(dev, step, args.steps)
        r["launches"] = int(dev.last_stats()["launches"])
        # the per-kernel CUDA-event profile (the roofline's launch durations, `layers`) from the
        # same steps run again: its event records stay out of the timed region above
        dev.profile(1)
        timed(dev, step, args.steps)
        r["layers"] = dev.profile_layers()
        r["prof"] = dev.profile(0)
        secs = max_over_ranks(secs)
        total_lines = args.pages * LINES_PER_PAGE
        r["value"] = total_lines * args.steps / secs
        r["ms_per_step"] = 1000 * secs / args.steps

        if not args.no_e2e:
            # a step: every group of the shard in turn, as the reference's pipeline feeds its
            # recognizer (carbon/src/pipeline.cpp:536-603): take the group prefetched beside the
            # previous group's runs, prefetch the next group (wrapping to the next step's first),
            # recognize this group's lines, read the decodings back
            def e2e_step():
                for k, g in enumerate(groups):
                    dev.set_pages([host_pages[j] for j in g], group_rows[k])
                    n = groups[(k + 1) % len(groups)]
                    dev.prefetch_pages([host_pages[j] for j in n], group_rows[(k + 1) % len(groups)])
                    po, bx, bwg = group_lines[k]
                    dev.recognize_lines(po, bx, bwg, flat=True)

            dev.prefetch_pages([host_pages[j] for j in groups[0]], group_rows[0])
            for _ in range(max(1, args.warmup // 2)):
                e2e_step()
            before = dev.last_stats()
            esecs = max_over_ranks(timed(dev, e2e_step, args.steps))
            after = dev.last_stats()
            h2d = (after["h2d_total"] - before["h2d_total"]) / args.steps
            d2h = (after["d2h_total"] - before["d2h_total"]) / args.steps
            r["e2e"] = {"value": total_lines * args.steps / esecs, "unit": "lines/s",
                        # the whole job's bytes a step: every rank's summed
                        "h2d_bytes_per_step": int(reduce_sum(h2d, world, "cuda")),
                        "d2h_bytes_per_step": int(reduce_sum(d2h, world, "cuda")),
                        "pages_uploaded_per_step": int(reduce_sum(len(slots), world, "cuda")),
                        "host_pages": "pageable, one buffer a slot (staged through pinned chunks by the library)"}
        results[prec] = r
        dev.close()

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            base, why = cpu_baseline(pages, boxes, bws)
            if base is None:
                base = {"unavailable": why}
        except Exception as e:  # noqa: BLE001
            base = {"unavailable": f"{type(e).__name__}: {e}"}

    if rank == 0:
        peaks, tag = measured_peaks()
        # the driver measures BF16 only: the INT8 and FP16 denominators are this GPU's own
        # tcgen05 rates (crec_mma_peak, back-to-back M = 128, N = 256, K = 32 bytes on every SM,
        # measured here); twice the measured BF16 rate is reported beside them as a cross-check
        tc = {"int8_n256_tops": native.mma_peak(local, native.INT8, 256),
              "int8_n64_tops": native.mma_peak(local, native.INT8, 64),
              "fp16_n256_tflops": native.mma_peak(local, native.FP16, 256),
              "two_x_bf16_tflops": 2.0 * peaks.get("bf16_tflops", 1590.0)}
        r8 = results["int8"]

        def kernel(r, name):
            return r["prof"].get(name, (0, 0.0, 0.0))

        def tensor_roof(r, peak, label):
            launches, ms, ops = kernel(r, "conv_gemm_tcgen05")
            achieved = (ops / (ms / 1000.0)) / 1e12 if ms > 0 else 0.0
            return {"bound": "tensor", "kernel": f"conv_gemm_tcgen05 ({label} implicit GEMM, all dense convs)",
                    "achieved": achieved, "peak": peak, "unit": "TOP/s", "frac": achieved / peak if peak else None,
                    "avg_launch_ms": ms / launches if launches else None,
                    "ops_per_launch": ops / launches if launches else None}

        roof = tensor_roof(r8, tc["int8_n256_tops"], "INT8")
        roof.update({"peak_source": "measured here: tcgen05 kind::i8 M=128 N=256 K=32 back to back (crec_mma_peak)",
                     "tensor_peaks_measured": tc,
                     # DRAM bytes a conv launch: the 11 launches of a 524,288-column run under ncu,
                     # scaled by columns to this run size; a lower bound (less stays in L2 at full size)
                     "traffic": CONV_TRAFFIC_PER_LAUNCH * args.max_columns / (1 << 21),
                     "traffic_unit": "bytes/launch"})
        # the other kernels' rooflines: the head on the tensor cores, crop+stem and decode on HBM
        n_lines = args.pages * LINES_PER_PAGE // world
        shard_bws = bw_all
        src = sum(crop_source_bytes(boxes[s % DISTINCT]) for s in slots[:DISTINCT])
        src_per_line = src / (min(len(slots), DISTINCT) * LINES_PER_PAGE)
        others = {}
        for prec, r in results.items():
            eb = 1 if prec == "int8" else 2
            cl, cms, _ = kernel(r, "crop_stem")
            # crop+stem: the windows' page bytes and the stem's output (16 rows x bw/2 x 32 channels)
            crop_bytes = (src_per_line * n_lines + 16 * 32 * eb * float((shard_bws // 2).sum())) * args.steps
            hl, hms, hops = kernel(r, "head_ctc_tcgen05")
            dl, dms, _ = kernel(r, "collapse")
            frames = float((shard_bws // 4).sum()) * args.steps
            decode_bytes = frames * 8 + n_lines * args.steps * 16  # each frame's id and probability, line records
            hpeak = tc["int8_n256_tops"] if prec == "int8" else tc["fp16_n256_tflops"]
            others[prec] = {
                "crop_stem": {"bound": "hbm", "achieved_gbs": crop_bytes / (cms / 1000) / 1e9 if cms else None,
                              "peak_gbs": peaks["hbm_gbs"], "frac": crop_bytes / (cms / 1000) / 1e9 / peaks["hbm_gbs"]
                              if cms else None, "note": tag},
                "head_ctc": {"bound": "tensor", "achieved": hops / (hms / 1000) / 1e12 if hms else None,
                             "peak": hpeak, "frac": hops / (hms / 1000) / 1e12 / hpeak if hms else None},
                "decode": {"bound": "hbm", "achieved_gbs": decode_bytes / (dms / 1000) / 1e9 if dms else None,
                           "peak_gbs": peaks["hbm_gbs"], "frac": decode_bytes / (dms / 1000) / 1e9 / peaks["hbm_gbs"]
                           if dms else None, "note": tag}}
        if "fp16" in results:
            others["fp16"]["conv"] = tensor_roof(results["fp16"], tc["fp16_n256_tflops"], "FP16")
        roof["others"] = others
        out = {
            "metric": METRIC, "value": r8["value"], "unit": "lines/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r8["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "u8xs8->s32 (INT8 engine)", "data": "synthetic (seeded pages, random-init "
            "rec-latin weights, seed 0)",
            "config": config_of(args, world),
            "e2e": r8.get("e2e"),
            "gpu_launches": r8["launches"] * args.steps,
            "roofline": roof,
            "kernels": {k: {"launches": v[0], "ms": v[1], "ops": v[2]} for k, v in r8["prof"].items()},
            "layers": [{"layer": i, "kernel": k, "launches": n, "ms": round(t, 3),
                        "tops": round(o / t / 1e9, 1) if t > 0 else None}
                       for i, (k, n, t, o) in enumerate(r8["layers"]) if n],
            "clocks": clocks,
            "cpu_baseline": base,
        }
        if "fp16" in results:
            f = results["fp16"]
            out["fp16"] = {"value": f["value"], "ms_per_step": f["ms_per_step"], "e2e": f.get("e2e"),
                           "layers": [{"layer": i, "kernel": k, "launches": n, "ms": round(t, 3),
                                       "tflops": round(o / t / 1e9, 1) if t > 0 else None}
                                      for i, (k, n, t, o) in enumerate(f["layers"]) if n]}
        print(json.dumps(out))
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
