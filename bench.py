#!/usr/bin/env python
"""Throughput of rec-latin line recognition (crop + recognizer + fused greedy CTC) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the 1/2/4/8-GPU one; config 2 is its 16-page slice):
1024 synthetic 2480 x 3508 pages x 64 lines (65,536 lines), sharded by page over the N
ranks (strong scaling: the total is fixed).  The pages are 32 distinct seeded pages
(seed 5000: background ~N(235, 8), lines 18-60 px high, aspect 4-40, +-5 degrees, glyph strokes
dense enough that about a quarter of the frames decode to characters), page slot s using page
s % 32 and its 64 boxes; each line is read at its 32-px bucket (up to
1024).  A step is every line of the rank's shard: cropped from its page, recognized,
decoded; only ids, frames and probabilities leave the GPU.

value: lines per second of the whole job (total lines / max over ranks of the device time,
CUDA events on the library's stream), INT8, pages already resident in HBM.  The per-kernel
profile behind `roofline` and `layers` comes from the same steps run once more with the
library's per-launch events on, outside the timed region.
e2e: the same through the public API with the host in the loop: each step uploads the
shard's pages (the rows the crops read, from pinned memory) and copies the decodings back.
The FP16 engine's numbers are reported beside the INT8 ones.

--impl reference: the reference's own CPU implementation of the path (oracle/_ref, the
int8 native executor with crop_lines and ctc_greedy, one pinned single-threaded session a
host core) on a bounded sample of the same workload; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "carbon-ocr_b200"))

METRIC = "text lines/sec (rec-latin INT8 & FP16, crop+CTC fused) at 1/2/4/8 B200; % TC peak"
PAGES_TOTAL, LINES_PER_PAGE, DISTINCT, SEED = 1024, 64, 32, 5000
PAGE_W, PAGE_H = 2480, 3508
WORKLOAD = ("config5: 1024 synthetic 2480x3508 pages x 64 lines (65,536 lines), rec-latin crop+trunk+fused CTC, "
            "32-px buckets to 1024, sharded by page; 32 distinct seeded pages (seed 5000, text-like glyphs: ~25% of "
            "frames decode to characters) resident before timing")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--max-columns", type=int, default=1 << 23, help="input columns a device run at most (the scheduler's run size)")
    ap.add_argument("--max-lines", type=int, default=32768)
    ap.add_argument("--pages", type=int, default=PAGES_TOTAL, help="page slots of the whole job (1024: config 5)")
    ap.add_argument("--no-fp16", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def workload(rank: int, world: int, pages_total: int = PAGES_TOTAL):
    """The rank's shard: distinct pages, and per line its page index (into the distinct pages),
    box and bucket width."""
    from carbon_rec import native, synth
    pages, boxes = synth.pages(SEED, DISTINCT, PAGE_W, PAGE_H, LINES_PER_PAGE)
    slots = range(rank * pages_total // world, (rank + 1) * pages_total // world)
    page_of = np.concatenate([np.full(LINES_PER_PAGE, s % DISTINCT, np.int32) for s in slots])
    allb = np.concatenate([boxes[s % DISTINCT] for s in slots])
    flat = np.concatenate(boxes)
    widths = np.array([native.crop_region(b)[1] for b in flat], np.int32)
    per_page = [widths[p * LINES_PER_PAGE:(p + 1) * LINES_PER_PAGE] for p in range(DISTINCT)]
    bws = np.concatenate([(per_page[s % DISTINCT] + 31) // 32 * 32 for s in slots]).astype(np.int32)
    return pages, boxes, page_of, allb, bws


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


# measured: dram__bytes_read.sum + dram__bytes_write.sum of all conv_gemm launches of one
# 524,288-column run / 11, x 4 (a 2,097,152-column run)
CONV_TRAFFIC_PER_LAUNCH = 646.2e6 / 11 * 4


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


def cpu_baseline(pages, page_of, boxes, bws, target_s=12.0):
    """The reference's CPU path (oracle/_ref) on a bounded sample, all host cores (one pinned
    single-threaded session each)."""
    from oracle import oracle as O
    from carbon_rec import model, onnx_pb
    if not O.Reference.available():
        return None, "oracle/_ref (the reference compiled from its sources) is not on this machine"
    import tempfile
    ref = O.Reference()
    cores = len(os.sched_getaffinity(0))
    n = min(len(page_of), 16 * LINES_PER_PAGE)  # config 2's 16 pages
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "rec-latin.int8.onnx"
        onnx_pb.save(model.make_rec_latin(0)[3], path)
        t1, done1 = ref.bench_pages(path, pages, page_of[:n], boxes[:n], bws[:n], threads=cores, rounds=1)
        rounds = max(1, min(200, int(target_s / max(t1, 1e-3))))
        secs, done = ref.bench_pages(path, pages, page_of[:n], boxes[:n], bws[:n], threads=cores, rounds=rounds)
    return {"value": done / secs, "unit": "lines/s", "cores": cores, "kind": "reference",
            "sample": f"{n} lines (config 2: 16 pages x 64) x {rounds} passes, crop_lines + int8 native executor "
                      f"+ ctc_greedy, {secs:.1f} s"}, None


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return 0
    from carbon_rec import synth
    pages, boxes, page_of, allb, bws = workload(0, 1)
    base, why = None, None
    times = []
    try:
        from oracle import oracle as O
        from carbon_rec import model, onnx_pb
        import tempfile
        if not O.Reference.available():
            why = "oracle/_ref (the reference compiled from its sources) is not on this machine"
        else:
            ref = O.Reference()
            cores = len(os.sched_getaffinity(0))
            n = 16 * LINES_PER_PAGE
            with tempfile.TemporaryDirectory() as d:
                path = Path(d) / "rec-latin.int8.onnx"
                onnx_pb.save(model.make_rec_latin(0)[3], path)
                for _ in range(args.warmup):
                    ref.bench_pages(path, pages, page_of[:n], allb[:n], bws[:n], threads=cores, rounds=1)
                for _ in range(args.steps):
                    t, done = ref.bench_pages(path, pages, page_of[:n], allb[:n], bws[:n], threads=cores, rounds=1)
                    times.append((t, done))
            secs = sum(t for t, _ in times)
            lines = sum(d for _, d in times)
            v = lines / secs
            base = {"value": v, "unit": "lines/s", "cores": cores, "kind": "reference",
                    "sample": f"each step: {n} lines (config 2: 16 pages x 64), crop_lines + int8 native executor + "
                              f"ctc_greedy, {cores} pinned workers"}
    except Exception as e:  # noqa: BLE001
        why = f"{type(e).__name__}: {e}"
    if base is None:
        print(json.dumps({"impl": "reference", "unavailable": why}))
        return 0
    out = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "lines/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * secs / max(1, args.steps),
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8xs8->s32",
           "data": "synthetic (seeded pages)", "config": {"workload": WORKLOAD + "; CPU sample: config 2's 16 pages"},
           "cpu_baseline": base,
           "e2e": {"value": base["value"], "unit": "lines/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out))
    return 0


def main() -> int:
    args = parse()
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
    pages, boxes, page_of, allb, bws = workload(rank, world, args.pages)
    _, _, fp, i8 = model.make_rec_latin(0)
    blobs = {"int8": netdef.compile_model(i8).to_blob(), "fp16": netdef.compile_model(fp).to_blob()}
    # pinned host pages (the e2e leg uploads from them) and their row runs
    pinned = []
    for p in pages:
        t = torch.empty(p.shape, dtype=torch.uint8, pin_memory=True)
        t.numpy()[:] = p
        pinned.append(t)
    host_pages = [t.numpy() for t in pinned]
    rows = [native.rows_read(boxes[i], PAGE_H) for i in range(DISTINCT)]

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
    prof = None
    layers = None
    stats = None
    for prec in (["int8"] if args.no_fp16 else ["int8", "fp16"]):
        dev = native.RecDevice(blobs[prec], native.INT8 if prec == "int8" else native.FP16, device=local,
                               max_lines=args.max_lines, max_width=1024, max_columns=args.max_columns,
                               max_pages=DISTINCT, max_page_bytes=DISTINCT * PAGE_W * PAGE_H)
        dev.set_pages(host_pages)  # resident for the device-time leg
        step = lambda: dev.recognize_lines(page_of, allb, bws, flat=True)  # noqa: E731
        for _ in range(args.warmup):
            step()
        if prec == "int8":
            with ClockSampler(local) as cs:
                secs = timed(dev, step, args.steps)
            clocks = cs.summary()
            stats = dev.last_stats()
            # the per-kernel CUDA-event profile (the roofline's launch durations, `layers`) from
            # the same steps run again: its event records stay out of the timed region above
            dev.profile(1)
            timed(dev, step, args.steps)
            layers = dev.profile_layers()
            prof = dev.profile(0)
        else:
            secs = timed(dev, step, args.steps)
        secs = max_over_ranks(secs)

        # a step: take the pages prefetched during the step before (their upload from pinned
        # memory ran beside that step's runs), give the next step's pages (uploaded beside this
        # step's runs, as the reference's pipeline does with prefetch_pages), recognize, read
        # the decodings back: one page upload and one result read-back a step
        def e2e_step():
            dev.set_pages(host_pages, rows)
            dev.prefetch_pages(host_pages, rows)
            dev.recognize_lines(page_of, allb, bws, flat=True)

        for _ in range(max(1, args.warmup // 2)):
            e2e_step()
        esecs = max_over_ranks(timed(dev, e2e_step, args.steps))
        # one step's bytes: the prefetch's page upload, then the recognize call's own copies
        dev.set_pages(host_pages, rows)
        dev.prefetch_pages(host_pages, rows)
        h2d_pages = dev.last_stats()["h2d_bytes"]
        dev.recognize_lines(page_of, allb, bws, flat=True)
        st = dev.last_stats()
        total_lines = args.pages * LINES_PER_PAGE
        results[prec] = {"value": total_lines * args.steps / secs, "ms_per_step": 1000 * secs / args.steps,
                         "e2e": {"value": total_lines * args.steps / esecs, "unit": "lines/s",
                                 # the whole job's bytes a step: every rank's summed
                                 "h2d_bytes_per_step": int(reduce_sum(h2d_pages + st["h2d_bytes"], world, "cuda")),
                                 "d2h_bytes_per_step": int(reduce_sum(st["d2h_bytes"], world, "cuda"))},
                         "launches_per_step": int(st["launches"])}
        dev.close()

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            base, why = cpu_baseline(pages, page_of, allb, bws)
            if base is None:
                base = {"unavailable": why}
        except Exception as e:  # noqa: BLE001
            base = {"unavailable": f"{type(e).__name__}: {e}"}

    if rank == 0:
        peaks, tag = measured_peaks()
        conv = prof.get("conv_gemm_tcgen05", (0, 0.0, 0.0)) if prof else (0, 0.0, 0.0)
        launches, ms, ops = conv
        # the driver measures BF16 only: the INT8 denominator is this GPU's own tcgen05 rate
        # (crec_mma_peak, back-to-back M = 128, N = 256, K = 32 MMAs on every SM, measured here);
        # twice the measured BF16 rate is reported beside it as a cross-check
        tc = {"int8_n256_tops": native.mma_peak(local, native.INT8, 256),
              "int8_n64_tops": native.mma_peak(local, native.INT8, 64),
              "fp16_n256_tflops": native.mma_peak(local, native.FP16, 256),
              "two_x_bf16_tflops": 2.0 * peaks.get("bf16_tflops", 1590.0)}
        peak_tops = tc["int8_n256_tops"]
        achieved = (ops / (ms / 1000.0)) / 1e12 if ms > 0 else 0.0
        r8 = results["int8"]
        out = {
            "metric": METRIC, "value": r8["value"], "unit": "lines/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r8["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "u8xs8->s32 (INT8 engine)", "data": "synthetic (seeded pages, random-init "
            "rec-latin weights, seed 0)",
            "config": {"workload": WORKLOAD if args.pages == PAGES_TOTAL else
                       f"{args.pages} of config 5's pages ({args.pages * LINES_PER_PAGE} lines)",
                       "lines": args.pages * LINES_PER_PAGE, "parallelism": f"pages/{world}",
                       "l2": "inputs larger than L2 (278 MB of pages; GB-scale activations)",
                       "max_columns_per_run": args.max_columns},
            "e2e": r8["e2e"],
            "gpu_launches": r8["launches_per_step"] * args.steps,
            "roofline": {"bound": "tensor", "kernel": "conv_gemm_tcgen05 (INT8 implicit GEMM, all dense convs)",
                         "achieved": achieved, "peak": peak_tops, "unit": "TOP/s",
                         "frac": achieved / peak_tops if peak_tops else None,
                         "peak_source": "measured here: tcgen05 kind::i8 M=128 N=256 K=32 back to back (crec_mma_peak)",
                         "tensor_peaks_measured": tc,
                         "avg_launch_ms": ms / launches if launches else None, "ops_per_launch": ops / launches if launches else None,
                         # DRAM bytes a conv launch: the 11 launches of a 524,288-column run under ncu
                         # (profiles/conv_gemm_tcgen05_int8_config5_128pages.md: 646 MB), scaled by
                         # columns to this run size; a lower bound (less stays in L2 at full size)
                         "traffic": CONV_TRAFFIC_PER_LAUNCH * args.max_columns / (1 << 21),
                         "traffic_unit": "bytes/launch"},
            "kernels": {k: {"launches": v[0], "ms": v[1], "ops": v[2]} for k, v in (prof or {}).items()},
            "layers": [{"layer": i, "kernel": k, "launches": n, "ms": round(t, 3),
                        "tops": round(o / t / 1e9, 1) if t > 0 else None}
                       for i, (k, n, t, o) in enumerate(layers or []) if n],
            "clocks": clocks,
            "cpu_baseline": base,
        }
        if "fp16" in results:
            out["fp16"] = {"value": results["fp16"]["value"], "ms_per_step": results["fp16"]["ms_per_step"],
                           "e2e": results["fp16"]["e2e"]}
        print(json.dumps(out))
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
