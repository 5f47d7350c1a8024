"""ctypes binding of the C ABI (include/carbon_rec.h), and a Python device object that
mirrors the reference's recognizer backend, carbon::PipelineModels
(carbon/include/carbon/pipeline.h:94-142): set_pages, prefetch_pages, recognize (the
lines of a group at one bucket width, their CTC decodings and the frames read),
broken.  Errors raise ``CrecError`` (the reference throws carbon::Error).

The library is built in-tree (carbon_rec/build.py) and loaded from there; there is no
fallback: without it, or without a B200, opening a device raises.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libcarbon_rec.so"

OK, E_INVALID, E_NOMEM, E_CUDA, E_STICKY, E_TIMEOUT, E_MODEL, E_RANGE = range(8)
INT8, FP16 = 0, 1
INJECT_TIMEOUT, INJECT_STICKY = 1, 2
_NAMES = {E_INVALID: "invalid argument", E_NOMEM: "out of memory", E_CUDA: "CUDA error", E_STICKY: "sticky CUDA error",
          E_TIMEOUT: "kernel wait timed out", E_MODEL: "model not supported", E_RANGE: "out of range"}

# every entry point include/carbon_rec.h declares
EXPORTS = ["crec_open", "crec_close", "crec_last_error", "crec_is_broken", "crec_set_pages", "crec_prefetch_pages",
           "crec_set_pages_device", "crec_recognize", "crec_recognize_lines", "crec_recognize_crops", "crec_ctc_greedy", "crec_ctc_greedy_noalloc", "crec_width_bucket", "crec_crop_region",
           "crec_stream", "crec_debug_crops", "crec_debug_value", "crec_debug_logits", "crec_last_stats", "crec_candidates",
           "crec_profile", "crec_profile_layers", "crec_mma_peak", "crec_debug_inject", "crec_conv_sweep",
           "crec_head_sweep", "crec_ctc_head_blob"]


class CrecError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{_NAMES.get(code, code)}: {message}")
        self.code = code


class CropRule(C.Structure):
    _fields_ = [("height", C.c_int), ("width_step", C.c_int), ("frame_px", C.c_int), ("pad_v", C.c_double),
                ("pad_h", C.c_double), ("flip_margin", C.c_int), ("flip_needs_dark", C.c_int)]

    @classmethod
    def default(cls, **kw) -> "CropRule":
        r = cls(32, 8, 4, 0.2, 0.3, 48, 1)
        for k, v in kw.items():
            setattr(r, k, v)
        return r


class Config(C.Structure):
    _fields_ = [("precision", C.c_int), ("device", C.c_int), ("max_lines", C.c_int), ("max_width", C.c_int),
                ("max_columns", C.c_int64), ("max_pages", C.c_int), ("max_page_bytes", C.c_int64),
                ("crop", CropRule), ("model", C.c_void_p), ("model_bytes", C.c_size_t)]


class Page(C.Structure):
    _fields_ = [("data", C.c_void_p), ("width", C.c_int), ("height", C.c_int), ("stride", C.c_int64)]


class RowRuns(C.Structure):
    _fields_ = [("runs", C.c_void_p), ("count", C.c_int)]


class Box(C.Structure):
    _fields_ = [("x0", C.c_double), ("y0", C.c_double), ("x1", C.c_double), ("y1", C.c_double)]


class Stats(C.Structure):
    _fields_ = [("runs", C.c_int64), ("launches", C.c_int64), ("h2d_bytes", C.c_int64), ("d2h_bytes", C.c_int64),
                ("h2d_total", C.c_int64), ("d2h_total", C.c_int64), ("wide_lines", C.c_int64)]


class ProfileEntry(C.Structure):
    _fields_ = [("kernel", C.c_char_p), ("launches", C.c_int64), ("ms", C.c_double), ("ops", C.c_double)]


class Lines(C.Structure):
    _fields_ = [("counts", C.c_void_p), ("lengths", C.c_void_p), ("offsets", C.c_void_p), ("ids", C.c_void_p),
                ("frames", C.c_void_p), ("probs", C.c_void_p), ("capacity", C.c_int64), ("total", C.c_int64)]


_lib = None


def lib() -> C.CDLL:
    """The CUDA library; raises if it was not built (there is no CPU fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with carbon_rec/build.py (nvcc, sm_100a)")
        L = C.CDLL(str(LIB_PATH))
        p, i, i64 = C.c_void_p, C.c_int, C.c_int64
        L.crec_open.argtypes = [C.POINTER(Config), C.POINTER(p)]
        L.crec_close.argtypes = [p]
        L.crec_last_error.argtypes = [p]
        L.crec_last_error.restype = C.c_char_p
        L.crec_is_broken.argtypes = [p]
        L.crec_set_pages.argtypes = [p, p, i, p]
        L.crec_prefetch_pages.argtypes = [p, p, i, p]
        L.crec_set_pages_device.argtypes = [p, p, i]
        L.crec_recognize.argtypes = [p, p, p, i, i, C.POINTER(Lines)]
        L.crec_recognize_lines.argtypes = [p, p, p, p, i, C.POINTER(Lines)]
        L.crec_recognize_crops.argtypes = [p, p, i, p, p, i, C.POINTER(Lines)]
        L.crec_ctc_greedy.argtypes = [p, i, i, i, p, C.POINTER(Lines), p, C.c_char_p, C.c_size_t]
        L.crec_ctc_greedy_noalloc.argtypes = [p, i, i, i, p, p, p, p, p, p, C.c_char_p, C.c_size_t]
        L.crec_width_bucket.argtypes = [i]
        L.crec_crop_region.argtypes = [C.POINTER(Box), C.POINTER(CropRule), p, C.POINTER(i)]
        L.crec_stream.argtypes = [p]
        L.crec_stream.restype = p
        L.crec_debug_crops.argtypes = [p, p, i]
        L.crec_debug_value.argtypes = [p, i, p, i64]
        L.crec_debug_logits.argtypes = [p, p, i64]
        L.crec_last_stats.argtypes = [p, C.POINTER(Stats)]
        L.crec_candidates.argtypes = [p, p, i, i, p, p, p, p, p, i64]
        L.crec_profile.argtypes = [p, i, C.POINTER(ProfileEntry), i]
        L.crec_profile_layers.argtypes = [p, C.POINTER(ProfileEntry), i]
        L.crec_mma_peak.argtypes = [i, i, i, i, C.POINTER(C.c_double)]
        L.crec_debug_inject.argtypes = [p, i]
        L.crec_conv_sweep.argtypes = [i, i, p, C.c_size_t, i, i, i, p, p, i, C.POINTER(C.c_double)]
        L.crec_head_sweep.argtypes = [i, i, p, C.c_size_t, i, p, p, p, p, i, C.POINTER(C.c_double)]
        L.crec_ctc_head_blob.argtypes = [p, C.c_size_t, p, C.c_size_t, C.POINTER(C.c_size_t), C.c_char_p, C.c_size_t]
        _lib = L
    return _lib


def mma_peak(device: int = 0, precision: int = 0, n: int = 256, iters: int = 4096) -> float:
    """The tensor cores' measured dense rate (TOP/s): back-to-back tcgen05.mma, M = 128, K = 32 bytes."""
    out = C.c_double(0.0)
    rc = lib().crec_mma_peak(device, precision, n, iters, C.byref(out))
    if rc != 0:
        raise CrecError(rc, "crec_mma_peak")
    return out.value


def ctc_greedy(logits_ptr: int, n: int, classes: int, frames: int, lengths, stream: int = 0):
    """carbon::cuda::ctc_greedy on device logits [n][classes][frames] at logits_ptr: (list of CtcLine, lengths)."""
    lens = np.ascontiguousarray(lengths, np.int32)
    cap = max(1, n * frames)
    bufs = dict(counts=np.zeros(n, np.int32), lengths=np.zeros(n, np.int32), offsets=np.zeros(n, np.int32),
                ids=np.zeros(cap, np.int32), frames=np.zeros(cap, np.int32), probs=np.zeros(cap, np.float32))
    s = Lines(*[bufs[k].ctypes.data for k in ("counts", "lengths", "offsets", "ids", "frames", "probs")], cap, 0)
    err = C.create_string_buffer(512)
    rc = lib().crec_ctc_greedy(int(logits_ptr), n, classes, frames, lens.ctypes.data, C.byref(s), stream or None,
                               err, 512)
    if rc != OK:
        raise CrecError(rc, err.value.decode())
    return RecDevice._unpack(bufs, n)


def ctc_greedy_noalloc(logits_ptr: int, n: int, classes: int, frames: int, lengths_ptr: int, counts_ptr: int,
                       ids_ptr: int, starts_ptr: int, probs_ptr: int, stream: int = 0) -> None:
    """crec_ctc_greedy_noalloc: every pointer a device address; queued on `stream`, not waited for."""
    err = C.create_string_buffer(256)
    rc = lib().crec_ctc_greedy_noalloc(int(logits_ptr), n, classes, frames, int(lengths_ptr), int(counts_ptr),
                                       int(ids_ptr), int(starts_ptr), int(probs_ptr), stream or None, err, 256)
    if rc != OK:
        raise CrecError(rc, err.value.decode())


def conv_sweep(blob: bytes, precision: int, x: np.ndarray, c_out: int, repeat: int = 3, device: int = 0,
               stride: int = 1):
    """crec_conv_sweep: x [n, h, w, c_in] (uint8 codes for INT8, float16 for FP16) through the blob's one
    convolution (3x3, pad 1, stride `stride`): (y [n, oh, w / stride, c_out], ms a launch)."""
    x = np.ascontiguousarray(x)
    n, h, w, _ = x.shape
    oh = (h + 2 - 3) // stride + 1
    y = np.zeros((n, oh, w // stride, c_out), x.dtype)
    ms = C.c_double(0.0)
    b = C.create_string_buffer(bytes(blob), len(blob))
    rc = lib().crec_conv_sweep(device, precision, C.cast(b, C.c_void_p), len(blob), n, h, w, x.ctypes.data, y.ctypes.data,
                               repeat, C.byref(ms))
    if rc != OK:
        raise CrecError(rc, "crec_conv_sweep")
    return y, ms.value


def head_sweep(blob: bytes, precision: int, x: np.ndarray, classes: int, repeat: int = 3, device: int = 0,
               logits: bool = False):
    """crec_head_sweep: x [frames, K] (uint8 codes for INT8, float16 for FP16) through the blob's one
    1x1 convolution as the fused head: (ids [frames], probs [frames], logits [frames, classes] or
    None, ms a launch)."""
    x = np.ascontiguousarray(x)
    frames = x.shape[0]
    ids = np.zeros(frames, np.int32)
    probs = np.zeros(frames, np.float32)
    lg = np.zeros((frames, classes), np.float32) if logits else None
    ms = C.c_double(0.0)
    b = C.create_string_buffer(bytes(blob), len(blob))
    rc = lib().crec_head_sweep(device, precision, C.cast(b, C.c_void_p), len(blob), frames, x.ctypes.data,
                               ids.ctypes.data, probs.ctypes.data, lg.ctypes.data if logits else None, repeat,
                               C.byref(ms))
    if rc != OK:
        raise CrecError(rc, "crec_head_sweep")
    return ids, probs, lg, ms.value


def ctc_head_blob(file_bytes: bytes) -> bytes:
    """crec_ctc_head_blob: a CTCHEAD1 file's bytes (<model>.head.bin) -> the FP16 blob of its head;
    raises CrecError(E_MODEL) with the reason for a file that is not a head."""
    f = C.create_string_buffer(bytes(file_bytes), len(file_bytes))
    n = C.c_size_t(0)
    err = C.create_string_buffer(256)
    rc = lib().crec_ctc_head_blob(C.cast(f, C.c_void_p), len(file_bytes), None, 0, C.byref(n), err, 256)
    if rc == E_RANGE:
        out = C.create_string_buffer(n.value)
        rc = lib().crec_ctc_head_blob(C.cast(f, C.c_void_p), len(file_bytes), C.cast(out, C.c_void_p), n.value,
                                      C.byref(n), err, 256)
        if rc == OK:
            return out.raw[:n.value]
    raise CrecError(rc, err.value.decode() or "crec_ctc_head_blob")


def width_bucket(crop_width: int) -> int:
    return lib().crec_width_bucket(int(crop_width))


def crop_region(box, rule: CropRule | None = None):
    rule = rule or CropRule.default()
    b = Box(*[float(v) for v in box])
    reg = np.zeros(4, np.float64)
    w = C.c_int()
    lib().crec_crop_region(C.byref(b), C.byref(rule), reg.ctypes.data, C.byref(w))
    return reg, w.value


def rows_read(boxes, height: int, rule: CropRule | None = None):
    """The rows a page's crops read, as [first, last) runs (carbon/src/pipeline.cpp:489-510): each
    line's crop region widened by twice the resampler's support and two rows, clipped to the
    page, sorted, runs closer than 16 rows joined."""
    import math
    rule = rule or CropRule.default()
    runs = []
    for b in np.asarray(boxes, np.float64).reshape(-1, 4):
        reg, _ = crop_region(b, rule)
        scale = max(1.0, (reg[3] - reg[1]) / rule.height)
        m = int(math.ceil(2 * scale)) + 2
        y0 = max(0, int(math.floor(reg[1])) - m)
        y1 = min(height, int(math.ceil(reg[3])) + m)
        if y1 > y0:
            runs.append((y0, y1))
    runs.sort()
    merged = []
    for r in runs:
        if merged and r[0] <= merged[-1][1] + 16:
            merged[-1] = (merged[-1][0], max(merged[-1][1], r[1]))
        else:
            merged.append(r)
    return merged


@dataclass
class CtcLine:
    """carbon::CtcLine: ids (blanks dropped, repeats collapsed), first frames, probabilities."""
    ids: np.ndarray
    frames: np.ndarray
    probs: np.ndarray


def _page_array(p) -> np.ndarray:
    """A page as the C ABI takes it: uint8 rows, each row's bytes contiguous (rows may be further
    apart, a view into a wider image); other arrays are copied."""
    a = np.asarray(p)
    if a.dtype == np.uint8 and a.ndim == 2 and a.strides[1] == 1 and a.strides[0] >= a.shape[1]:
        return a
    return np.ascontiguousarray(a, np.uint8)


def _boxes(boxes) -> np.ndarray:
    b = np.ascontiguousarray(np.asarray(boxes, np.float64).reshape(-1, 4))
    return b


class RecDevice:
    """One GPU's recognizer (the PipelineModels recognizer methods), over the C ABI."""

    def __init__(self, model_blob: bytes, precision: int = INT8, device: int = 0, max_lines: int = 256,
                 max_width: int = 2048, max_columns: int = 0, max_pages: int = 64, max_page_bytes: int = 0,
                 crop: CropRule | None = None):
        L = lib()
        self._blob = C.create_string_buffer(bytes(model_blob), len(model_blob))
        self.crop = crop or CropRule.default()
        cfg = Config(precision, device, max_lines, max_width, max_columns, max_pages, max_page_bytes, self.crop,
                     C.cast(self._blob, C.c_void_p), len(model_blob))
        h = C.c_void_p()
        rc = L.crec_open(C.byref(cfg), C.byref(h))
        self._h = h
        if rc != OK:
            msg = L.crec_last_error(h).decode() if h else ""
            L.crec_close(h)
            self._h = None
            raise CrecError(rc, msg)
        self.max_lines, self.max_width = max_lines, max_width
        self._keep: list = []

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().crec_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 (interpreter shutdown: the module may be gone)
            pass

    def _check(self, rc: int) -> None:
        if rc != OK:
            raise CrecError(rc, lib().crec_last_error(self._h).decode())

    @property
    def broken(self) -> bool:
        return bool(lib().crec_is_broken(self._h))

    @property
    def stream(self) -> int:
        return lib().crec_stream(self._h)

    def _runs(self, rows, keep):
        if rows is None:
            return None
        rr = []
        for r in rows:
            if r:
                a = np.ascontiguousarray(np.asarray(r, np.int32).reshape(-1))
                keep.append(a)
                rr.append(RowRuns(a.ctypes.data, len(a) // 2))
            else:
                rr.append(RowRuns(None, 0))
        return (RowRuns * len(rr))(*rr)

    def set_pages(self, pages, rows=None) -> None:
        """pages: list of 2-d uint8 arrays (paper 255); rows: per page a list of (first, last) row runs or None.
        The arrays are kept alive here until the next set_pages or prefetch_pages call returns."""
        arr = [_page_array(p) for p in pages]
        descs = (Page * max(1, len(arr)))(*[Page(a.ctypes.data, a.shape[1], a.shape[0], a.strides[0]) for a in arr])
        keep: list = []
        runs = self._runs(rows, keep)
        self._check(lib().crec_set_pages(self._h, descs, len(arr), runs))
        self._alive = arr

    def set_pages_device(self, pages) -> None:
        """pages: list of (device pointer, width, height, stride) already in this GPU's memory."""
        descs = (Page * max(1, len(pages)))(*[Page(int(d), int(w), int(hh), int(s)) for d, w, hh, s in pages])
        self._check(lib().crec_set_pages_device(self._h, descs, len(pages)))

    def prefetch_pages(self, pages, rows=None) -> None:
        """The next group's pages, uploaded beside the current group's work; a set_pages with the same
        arrays then takes them.  Kept alive here until the next set_pages or prefetch_pages call returns."""
        arr = [_page_array(p) for p in pages]
        descs = (Page * max(1, len(arr)))(*[Page(a.ctypes.data, a.shape[1], a.shape[0], a.strides[0]) for a in arr])
        keep: list = []
        runs = self._runs(rows, keep)
        self._check(lib().crec_prefetch_pages(self._h, descs, len(arr), runs))
        self._alive = arr

    def _lines(self, n: int, cap: int):
        bufs = dict(counts=np.empty(n, np.int32), lengths=np.empty(n, np.int32), offsets=np.empty(n, np.int32),
                    ids=np.empty(cap, np.int32), frames=np.empty(cap, np.int32), probs=np.empty(cap, np.float32))
        s = Lines(*[bufs[k].ctypes.data for k in ("counts", "lengths", "offsets", "ids", "frames", "probs")], cap, 0)
        return bufs, s

    @staticmethod
    def _flat(bufs, total: int) -> dict:
        """The decodings as flat arrays: counts, lengths, offsets per line; ids, frames, probs packed."""
        return {k: (v[:total] if k in ("ids", "frames", "probs") else v) for k, v in bufs.items()}

    @staticmethod
    def _unpack(bufs, n: int):
        out = []
        for i in range(n):
            o, k = int(bufs["offsets"][i]), int(bufs["counts"][i])
            out.append(CtcLine(bufs["ids"][o:o + k].copy(), bufs["frames"][o:o + k].copy(), bufs["probs"][o:o + k].copy()))
        return out, bufs["lengths"].copy()

    def recognize(self, page_of, boxes, bw: int):
        """PipelineModels::recognize: (list of CtcLine, lengths) for boxes of pages page_of at bucket width bw."""
        po = np.ascontiguousarray(page_of, np.int32)
        b = _boxes(boxes)
        n = len(po)
        bufs, s = self._lines(n, max(1, n * (bw // self.crop.frame_px)))
        self._check(lib().crec_recognize(self._h, po.ctypes.data, b.ctypes.data, n, int(bw), C.byref(s)))
        return self._unpack(bufs, n)

    def recognize_lines(self, page_of, boxes, bw=None, flat: bool = False):
        """Any number of lines, each at its own bucket width (bw[i], or the width ladder's bucket):
        (list of CtcLine, lengths), or with flat the arrays as the C ABI fills them."""
        po = np.ascontiguousarray(page_of, np.int32)
        b = _boxes(boxes)
        n = len(po)
        bwa = None if bw is None else np.ascontiguousarray(bw, np.int32)
        cap = max(1, (int(bwa.sum()) if bwa is not None else n * self.max_width) // self.crop.frame_px)
        bufs, s = self._lines(n, cap)
        self._check(lib().crec_recognize_lines(self._h, po.ctypes.data, b.ctypes.data,
                                               None if bwa is None else bwa.ctypes.data, n, C.byref(s)))
        return self._flat(bufs, s.total) if flat else self._unpack(bufs, n)

    def recognize_crops(self, crops, widths, bw):
        """Ready crops [n, height, pitch] uint8 (line i's first bw[i] columns finished and padded), their crop
        widths: (list of CtcLine, lengths)."""
        c = np.ascontiguousarray(crops, np.uint8)
        n, _, pitch = c.shape
        w = np.ascontiguousarray(widths, np.int32)
        b = np.ascontiguousarray(bw, np.int32)
        bufs, s = self._lines(n, max(1, int(b.sum()) // self.crop.frame_px))
        self._check(lib().crec_recognize_crops(self._h, c.ctypes.data, int(pitch), w.ctypes.data, b.ctypes.data, n,
                                               C.byref(s)))
        return self._unpack(bufs, n)

    def arm_crops(self, pitch: int) -> None:
        self._check(lib().crec_debug_crops(self._h, None, int(pitch)))

    def crops(self, n: int, pitch: int) -> np.ndarray:
        out = np.zeros((n, self.crop.height, pitch), np.uint8)
        self._check(lib().crec_debug_crops(self._h, out.ctypes.data, int(pitch)))
        return out

    def last_stats(self) -> dict:
        st = Stats()
        self._check(lib().crec_last_stats(self._h, C.byref(st)))
        return {"runs": st.runs, "launches": st.launches, "h2d_bytes": st.h2d_bytes, "d2h_bytes": st.d2h_bytes,
                "h2d_total": st.h2d_total, "d2h_total": st.d2h_total, "wide_lines": st.wide_lines}

    def profile(self, enable: int = -1) -> dict:
        """Per-kernel totals {name: (launches, ms, ops)} since profiling was (re)started; enable 1 (re)starts."""
        ent = (ProfileEntry * 8)()
        n = lib().crec_profile(self._h, int(enable), ent, 8)
        return {ent[i].kernel.decode(): (ent[i].launches, ent[i].ms, ent[i].ops) for i in range(max(n, 0))}

    def profile_layers(self) -> list:
        """Per layer (then the collapse): (kernel, launches, ms, ops) since profiling was (re)started."""
        ent = (ProfileEntry * 64)()
        n = lib().crec_profile_layers(self._h, ent, 64)
        if n < 0:
            self._check(-n)
        return [(ent[i].kernel.decode(), ent[i].launches, ent[i].ms, ent[i].ops) for i in range(n)]

    def inject(self, what: int) -> None:
        """Test hook: INJECT_TIMEOUT or INJECT_STICKY for the next device run (crec_debug_inject)."""
        self._check(lib().crec_debug_inject(self._h, int(what)))

    def arm_logits(self) -> None:
        self._check(lib().crec_debug_logits(self._h, None, 0))

    def logits(self, bws, classes: int) -> list:
        """The last run's logits, a [classes, bw / frame_px] array per line (bucket widths bws)."""
        t = [int(b) // self.crop.frame_px for b in bws]
        out = np.zeros(sum(t) * classes, np.float32)
        self._check(lib().crec_debug_logits(self._h, out.ctypes.data, out.size))
        res, at = [], 0
        for k in t:
            res.append(out[at:at + classes * k].reshape(classes, k))
            at += classes * k
        return res

    def candidates(self, rows, topk: int, capacity: int | None = None) -> list:
        """crec_candidates: the beam's candidates of lines `rows` of the last recognize call, a
        (ids [t, k], logp [t, k], blank [t]) per row (carbon::FrameCandidates; k = topk clamped to
        [0, min(16, classes - 1)])."""
        rows = np.ascontiguousarray(rows, np.int32)
        n = len(rows)
        cap = capacity if capacity is not None else 4096 * max(n, 1)
        frames = np.zeros(max(n, 1), np.int32)
        kk = C.c_int32(0)
        kmax = max(0, min(int(topk), 16))
        ids = np.zeros(max(cap * kmax, 1), np.int32)
        logp = np.zeros(max(cap * kmax, 1), np.float32)
        blank = np.zeros(max(cap, 1), np.float32)
        self._check(lib().crec_candidates(self._h, rows.ctypes.data, n, int(topk), C.byref(kk), frames.ctypes.data,
                                          ids.ctypes.data, logp.ctypes.data, blank.ctypes.data, cap))
        topk = kk.value
        out, at = [], 0
        for j in range(n):
            t = int(frames[j])
            out.append((ids[at * topk:(at + t) * topk].reshape(t, topk), logp[at * topk:(at + t) * topk].reshape(t, topk),
                        blank[at:at + t]))
            at += t
        return out

    def value(self, index: int, nbytes: int, dtype=np.uint8) -> np.ndarray:
        out = np.zeros(nbytes, np.uint8)
        self._check(lib().crec_debug_value(self._h, int(index), out.ctypes.data, nbytes))
        return out.view(dtype)
