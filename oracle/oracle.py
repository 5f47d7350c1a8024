"""ctypes bindings of the two CPU checkers.

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU
baseline import this module; the CUDA product path never does.

* ``Oracle``: the C restatement of the reference's path (oracle/rec_oracle.c),
  built into oracle/liborc.so by ``build()``.
* ``Reference``: the reference's own CPU code, compiled from its sources into
  oracle/_ref/libcarbon_ref.so (oracle/ref.mk) where the reference checkout is
  present; optional at run time (it travels to a GPU box only as a built file).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORC_SO = HERE / "liborc.so"
REF_SO = HERE / "_ref" / "libcarbon_ref.so"
REFERENCE_ROOT = Path(os.environ.get("CARBON_REFERENCE", "/root/reference"))

_p = C.c_void_p
_i = C.c_int
_i64 = C.c_int64
_d = C.c_double


def build(force: bool = False) -> None:
    """Compiles the C restatement, and the reference's own code where its checkout is here."""
    src = HERE / "rec_oracle.c"
    if force or not ORC_SO.exists() or ORC_SO.stat().st_mtime < src.stat().st_mtime:
        subprocess.check_call(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fPIC", "-shared",
                               "-fvisibility=hidden", str(src), "-o", str(ORC_SO), "-lm"])
    if (REFERENCE_ROOT / "carbon" / "src" / "lines.cpp").exists():
        subprocess.check_call(["make", "-s", "-f", "ref.mk", f"REF={REFERENCE_ROOT}", "-j8"], cwd=HERE)
        if (HERE.parent / "carbon-ocr_b200" / "carbon_rec" / "libcarbon_rec.so").exists():
            # INTEGRATION.md's adapter behind the reference's PipelineModels (tests/adapter_run.cpp)
            subprocess.check_call(["make", "-s", "-f", "ref.mk", f"REF={REFERENCE_ROOT}", "adapter"], cwd=HERE)


class CropRule(C.Structure):
    _fields_ = [("height", _i), ("width_step", _i), ("frame_px", _i), ("pad_v", _d), ("pad_h", _d),
                ("flip_margin", _i), ("flip_needs_dark", _i)]

    @classmethod
    def default(cls, **kw):
        r = cls(32, 8, 4, 0.2, 0.3, 48, 1)
        for k, v in kw.items():
            setattr(r, k, v)
        return r


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_p)


class _Common:
    lib: C.CDLL

    def ctc_topk(self, logits: np.ndarray, t_n: int, k: int):
        """One line's logits [classes, frames] -> the beam's candidates of its first t_n frames:
        (ids [t_n, k], logp [t_n, k], blank [t_n]) (carbon::frame_candidates)."""
        logits = np.ascontiguousarray(logits, np.float32)
        classes, frames = logits.shape
        ids = np.zeros((t_n, k), np.int32)
        logp = np.zeros((t_n, k), np.float32)
        blank = np.zeros(t_n, np.float32)
        r = self._ctc_topk(_ptr(logits), classes, frames, t_n, k, _ptr(ids), _ptr(logp), _ptr(blank))
        if r not in (None, 0):
            raise ValueError(f"ctc_topk failed ({r})")
        return ids, logp, blank

    def crop_lines(self, page: np.ndarray, boxes: np.ndarray, out_width: int, rule: CropRule | None = None):
        """boxes [n, 4] (x0, y0, x1, y1) on page [h, w] uint8 -> (crops [n, 32, out_width], widths [n])."""
        rule = rule or CropRule.default()
        page = np.ascontiguousarray(page, np.uint8)
        b = np.ascontiguousarray(boxes, np.float64).reshape(-1, 4)
        n = b.shape[0]
        out = np.zeros((n, rule.height, out_width), np.uint8)
        widths = np.zeros(n, np.int32)
        r = self._crop_lines(_ptr(page), page.shape[1], page.shape[0], page.strides[0], _ptr(b), n, out_width,
                             _ptr(out), _ptr(widths), C.byref(rule))
        if r != 0:
            raise ValueError(f"crop_lines failed ({r})")
        return out, widths


class Oracle(_Common):
    def __init__(self):
        if not ORC_SO.exists():
            build()
        L = self.lib = C.CDLL(str(ORC_SO))
        L.orc_crop_region.argtypes = [_p, _p, _p]
        L.orc_crop_region.restype = _i
        L.orc_width_bucket.argtypes = [_i]
        L.orc_width_bucket.restype = _i
        L.orc_resample_gray.argtypes = [_p, _i, _i, _i64, _d, _d, _d, _d, _i, _i, _p, _i64]
        L.orc_crop_ground.argtypes = [_p, _i, _i, _i64]
        L.orc_finish_crop.argtypes = [_p, _i, _i, _p]
        L.orc_finish_crop.restype = None
        L.orc_crop_lines.argtypes = [_p, _i, _i, _i64, _p, _i, _i, _p, _p, _p]
        L.orc_model_open.argtypes = [_p, C.c_size_t]
        L.orc_model_open.restype = _p
        L.orc_model_close.argtypes = [_p]
        L.orc_model_close.restype = None
        L.orc_model_classes.argtypes = [_p]
        L.orc_input_table.argtypes = [_p, _p]
        L.orc_input_table.restype = None
        L.orc_model_run.argtypes = [_p, _p, _i, _i, _p, _i, _p]
        L.orc_exp_neg.argtypes = [C.c_float]
        L.orc_exp_neg.restype = C.c_float
        L.orc_ctc_greedy.argtypes = [_p, _i, _i, _i, _p, _i, _p, _p, _p, _p, _p, _p]
        L.orc_ctc_greedy.restype = None
        L.orc_ctc_topk.argtypes = [_p, _i, _i, _i, _i, _p, _p, _p]
        L.orc_ctc_topk.restype = None
        L.orc_ctc_collapse.argtypes = [_p, _p, _i, _i, _p, _i, _p, _p, _p, _p]
        L.orc_ctc_collapse.restype = None
        self._crop_lines = L.orc_crop_lines
        self._ctc_topk = L.orc_ctc_topk

    def crop_region(self, box, rule: CropRule | None = None):
        rule = rule or CropRule.default()
        b = np.asarray(box, np.float64)
        reg = np.zeros(4, np.float64)
        w = self.lib.orc_crop_region(_ptr(b), C.byref(rule), _ptr(reg))
        return reg, w

    def width_bucket(self, w: int) -> int:
        return self.lib.orc_width_bucket(int(w))

    def resample_gray(self, img, x0, y0, x1, y1, ow, oh):
        img = np.ascontiguousarray(img, np.uint8)
        out = np.zeros((oh, ow), np.uint8)
        self.lib.orc_resample_gray(_ptr(img), img.shape[1], img.shape[0], img.strides[0], x0, y0, x1, y1, ow, oh,
                                   _ptr(out), ow)
        return out

    def crop_ground(self, crop, w, h, stride):
        return self.lib.orc_crop_ground(_ptr(crop), w, h, stride)

    def finish_crop(self, crop: np.ndarray, w: int, rule: CropRule | None = None):
        rule = rule or CropRule.default(height=crop.shape[0])
        self.lib.orc_finish_crop(_ptr(crop), w, crop.shape[1], C.byref(rule))

    def exp_neg(self, x: float) -> float:
        return self.lib.orc_exp_neg(x)

    def ctc_greedy(self, logits: np.ndarray, lengths, cap: int | None = None):
        """logits [n, classes, T] -> (list of (ids, frames, probs) per line, per-frame ids, per-frame probs)."""
        logits = np.ascontiguousarray(logits, np.float32)
        n, classes, frames = logits.shape
        cap = cap or frames
        lengths = np.ascontiguousarray(lengths, np.int32)
        counts = np.zeros(n, np.int32)
        ids = np.zeros((n, cap), np.int32)
        fr = np.zeros((n, cap), np.int32)
        pr = np.zeros((n, cap), np.float32)
        fid = np.zeros((n, frames), np.int32)
        fpr = np.zeros((n, frames), np.float32)
        self.lib.orc_ctc_greedy(_ptr(logits), n, classes, frames, _ptr(lengths), cap, _ptr(counts), _ptr(ids),
                                _ptr(fr), _ptr(pr), _ptr(fid), _ptr(fpr))
        lines = [(ids[i, :counts[i]].copy(), fr[i, :counts[i]].copy(), pr[i, :counts[i]].copy()) for i in range(n)]
        return lines, fid, fpr

    def ctc_collapse(self, frame_ids: np.ndarray, frame_probs: np.ndarray | None, lengths):
        frame_ids = np.ascontiguousarray(frame_ids, np.int32)
        n, frames = frame_ids.shape
        lengths = np.ascontiguousarray(lengths, np.int32)
        counts = np.zeros(n, np.int32)
        ids = np.zeros((n, frames), np.int32)
        fr = np.zeros((n, frames), np.int32)
        pr = np.zeros((n, frames), np.float32)
        fp = None if frame_probs is None else np.ascontiguousarray(frame_probs, np.float32)
        self.lib.orc_ctc_collapse(_ptr(frame_ids), None if fp is None else _ptr(fp), n, frames, _ptr(lengths),
                                  frames, _ptr(counts), _ptr(ids), _ptr(fr), _ptr(pr))
        return [(ids[i, :counts[i]].copy(), fr[i, :counts[i]].copy(), pr[i, :counts[i]].copy()) for i in range(n)]

    def model(self, blob: bytes) -> "OracleModel":
        return OracleModel(self, blob)


class OracleModel:
    """The restated executor on a model blob (carbon_rec.netdef.RecNet.to_blob)."""

    def __init__(self, orc: Oracle, blob: bytes):
        self.orc = orc
        self._blob = C.create_string_buffer(blob, len(blob))
        self.h = orc.lib.orc_model_open(self._blob, len(blob))
        if not self.h:
            raise ValueError("the oracle cannot read this model blob")
        self.classes = orc.lib.orc_model_classes(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            self.orc.lib.orc_model_close(self.h)
            self.h = None

    def input_table(self) -> np.ndarray:
        t = np.zeros(256, np.uint8)
        self.orc.lib.orc_input_table(self.h, _ptr(t))
        return t

    def run(self, crops: np.ndarray, keep_value: int = -1, keep_shape=None, keep_dtype=np.uint8):
        """crops [n, 32, bw] uint8 -> logits [n, classes, T] float32 (and a kept value's NHWC tensor)."""
        crops = np.ascontiguousarray(crops, np.uint8)
        n, _, bw = crops.shape
        frames = bw // 4
        logits = np.zeros((n, self.classes, frames), np.float32)
        keep = None
        if keep_value >= 0:
            keep = np.zeros(keep_shape, keep_dtype)
        t = self.orc.lib.orc_model_run(self.h, _ptr(crops), n, bw, _ptr(logits), keep_value,
                                       None if keep is None else _ptr(keep))
        if t != frames:
            logits = np.zeros((n, self.classes, t), np.float32)
            self.orc.lib.orc_model_run(self.h, _ptr(crops), n, bw, _ptr(logits), keep_value,
                                       None if keep is None else _ptr(keep))
        return (logits, keep) if keep_value >= 0 else logits


class Reference(_Common):
    """The reference's compiled CPU code (oracle/_ref), when it was built."""

    @staticmethod
    def available() -> bool:
        return REF_SO.exists()

    def __init__(self):
        L = self.lib = C.CDLL(str(REF_SO))
        L.ref_last_error.restype = C.c_char_p
        L.ref_crop_region.argtypes = [_p, _p, _p, _p]
        L.ref_crop_lines.argtypes = [_p, _i, _i, _i64, _p, _i, _i, _p, _p, _p]
        L.ref_resample_gray.argtypes = [_p, _i, _i, _i64, _d, _d, _d, _d, _i, _i, _p, _i64, _i]
        L.ref_finish_crop.argtypes = [_p, _i, _i, _p]
        L.ref_crop_ground.argtypes = [_p, _i, _i, _i64]
        L.ref_light_on_dark.argtypes = [_p, _i, _i, _i64, _i]
        L.ref_exp_neg.argtypes = [C.c_float]
        L.ref_exp_neg.restype = C.c_float
        L.ref_ctc_greedy.argtypes = [_p, _i, _i, _i, _p, _i, _p, _p, _p, _p]
        L.ref_ctc_collapse.argtypes = [_p, _p, _i, _i, _p, _i, _p, _p, _p, _p]
        L.ref_open.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, C.c_size_t]
        L.ref_open.restype = _p
        L.ref_close.argtypes = [_p]
        L.ref_close.restype = None
        L.ref_run.argtypes = [_p, _p, _i, _i, _i, _i, _p, _i64, _p, _p]
        L.ref_cut.argtypes = [C.c_char_p, C.c_char_p, _p, _i, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
        L.ref_free.argtypes = [_p]
        L.ref_free.restype = None
        L.ref_bench_batches.argtypes = [C.c_char_p, C.c_char_p, _i, _i, _i, _p, _p, _p, _p, _p, _i, _i]
        L.ref_bench_batches.restype = _d
        L.ref_bench_pages.argtypes = [C.c_char_p, C.c_char_p, _i, _i, _i, _p, _p, _p, _p, _i, _p, _p, _p, _p, _p, _i,
                                      C.POINTER(C.c_int64)]
        L.ref_bench_pages.restype = _d
        L.ref_ctc_topk.argtypes = [_p, _i, _i, _i, _i, _p, _p, _p]
        L.ref_ctc_topk.restype = _i
        L.ref_load_ctc_head.argtypes = [C.c_char_p, _p, _p, _p, _p, _i64]
        L.ref_load_ctc_head.restype = _i
        self._crop_lines = L.ref_crop_lines
        self._ctc_topk = L.ref_ctc_topk

    def error(self) -> str:
        return self.lib.ref_last_error().decode()

    def load_ctc_head(self, path, cap: int = 1 << 26):
        """carbon::load_ctc_head: (classes, k, weight float16 [classes, k], bias [classes]); raises
        ValueError with the reference's message for a file it refuses."""
        classes, k = C.c_int(), C.c_int()
        w = np.zeros(cap, np.uint16)
        b = np.zeros(cap, np.float32)
        if self.lib.ref_load_ctc_head(str(path).encode(), C.byref(classes), C.byref(k), _ptr(w), _ptr(b), cap) != 0:
            raise ValueError(self.error())
        n = classes.value * k.value
        return classes.value, k.value, w[:n].view(np.float16).reshape(classes.value, k.value), b[:classes.value]

    def crop_region(self, box, rule: CropRule | None = None):
        rule = rule or CropRule.default()
        b = np.asarray(box, np.float64)
        reg = np.zeros(4, np.float64)
        w = C.c_int()
        if self.lib.ref_crop_region(_ptr(b), C.byref(rule), _ptr(reg), C.byref(w)) != 0:
            raise ValueError(self.error())
        return reg, w.value

    def resample_gray(self, img, x0, y0, x1, y1, ow, oh, scalar=False):
        img = np.ascontiguousarray(img, np.uint8)
        out = np.zeros((oh, ow), np.uint8)
        if self.lib.ref_resample_gray(_ptr(img), img.shape[1], img.shape[0], img.strides[0], x0, y0, x1, y1, ow, oh,
                                      _ptr(out), ow, int(scalar)) != 0:
            raise ValueError(self.error())
        return out

    def crop_ground(self, crop, w, h, stride):
        return self.lib.ref_crop_ground(_ptr(crop), w, h, stride)

    def finish_crop(self, crop: np.ndarray, w: int, rule: CropRule | None = None):
        rule = rule or CropRule.default(height=crop.shape[0])
        if self.lib.ref_finish_crop(_ptr(crop), w, crop.shape[1], C.byref(rule)) != 0:
            raise ValueError(self.error())

    def exp_neg(self, x: float) -> float:
        return self.lib.ref_exp_neg(x)

    def ctc_greedy(self, logits: np.ndarray, lengths, cap: int | None = None):
        logits = np.ascontiguousarray(logits, np.float32)
        n, classes, frames = logits.shape
        cap = cap or frames
        lengths = np.ascontiguousarray(lengths, np.int32)
        counts = np.zeros(n, np.int32)
        ids = np.zeros((n, cap), np.int32)
        fr = np.zeros((n, cap), np.int32)
        pr = np.zeros((n, cap), np.float32)
        if self.lib.ref_ctc_greedy(_ptr(logits), n, classes, frames, _ptr(lengths), cap, _ptr(counts), _ptr(ids),
                                   _ptr(fr), _ptr(pr)) != 0:
            raise ValueError(self.error())
        return [(ids[i, :counts[i]].copy(), fr[i, :counts[i]].copy(), pr[i, :counts[i]].copy()) for i in range(n)]

    def bench_pages(self, model_path, pages, page_of, boxes, bws, threads: int, rounds: int = 1, first_cpu: int = 0,
                    isa: str = "", batch: int = 256):
        """The reference's CPU device on pages (crop_lines, ink, int8 session, ctc_greedy), `threads`
        pinned workers: (seconds of `rounds` timed passes, lines recognized in them)."""
        order = np.lexsort((np.arange(len(bws)), np.asarray(bws)))  # stable by bucket, as the pipeline sorts
        po = np.ascontiguousarray(np.asarray(page_of, np.int32)[order])
        bx = np.ascontiguousarray(np.asarray(boxes, np.float64).reshape(-1, 4)[order])
        bwo = np.asarray(bws, np.int32)[order]
        starts, counts, widths = [], [], []
        a = 0
        while a < len(bwo):
            b = a
            while b < len(bwo) and bwo[b] == bwo[a] and b - a < batch:
                b += 1
            starts.append(a)
            counts.append(b - a)
            widths.append(int(bwo[a]))
            a = b
        arr = [np.ascontiguousarray(p, np.uint8) for p in pages]
        data = (C.c_void_p * len(arr))(*[p.ctypes.data for p in arr])
        pw = np.array([p.shape[1] for p in arr], np.int32)
        ph = np.array([p.shape[0] for p in arr], np.int32)
        ps = np.array([p.strides[0] for p in arr], np.int64)
        st, ct, wd = (np.array(v, np.int32) for v in (starts, counts, widths))
        done = C.c_int64()
        secs = self.lib.ref_bench_pages(str(model_path).encode(), isa.encode(), threads, first_cpu, len(arr), data,
                                        _ptr(pw), _ptr(ph), _ptr(ps), len(st), _ptr(st), _ptr(ct), _ptr(wd), _ptr(po),
                                        _ptr(bx), rounds, C.byref(done))
        if secs < 0:
            raise ValueError(self.error())
        return secs, done.value

    def session(self, path, isa: str = "", model_bytes: bytes | None = None) -> "RefSession":
        return RefSession(self, path, isa, model_bytes)

    def cut(self, path, output: str, dims) -> bytes:
        d = np.asarray(dims, np.int64)
        out = C.c_void_p()
        n = C.c_size_t()
        if self.lib.ref_cut(str(path).encode(), output.encode(), _ptr(d), len(d), C.byref(out), C.byref(n)) != 0:
            raise ValueError(self.error())
        b = C.string_at(out, n.value)
        self.lib.ref_free(out)
        return b


class RefSession:
    def __init__(self, ref: Reference, path, isa: str, model_bytes: bytes | None):
        self.ref = ref
        self.h = ref.lib.ref_open(str(path).encode(), isa.encode(), model_bytes,
                                  len(model_bytes) if model_bytes else 0)
        if not self.h:
            raise ValueError(ref.error())

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.ref_close(self.h)
            self.h = None

    def run(self, x: np.ndarray, cap: int | None = None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        n, c, h, w = x.shape
        cap = cap or n * 1024 * max(w, 8)
        out = np.zeros(cap, np.float32)
        shape = np.zeros(8, np.int64)
        rank = C.c_int()
        if self.ref.lib.ref_run(self.h, _ptr(x), n, c, h, w, _ptr(out), cap, _ptr(shape), C.byref(rank)) != 0:
            raise ValueError(self.ref.error())
        s = tuple(int(v) for v in shape[:rank.value])
        return out[:int(np.prod(s))].reshape(s).copy()
