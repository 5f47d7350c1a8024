"""INTEGRATION.md's adapter (carbon::B200RecModels), linked and run behind the reference's
carbon::PipelineModels interface: tests/adapter_run.cpp drives it as carbon::Pipeline's recognize
stage does (set_pages with each page's RowRuns, prefetch_pages of the next group while the current
one is read, recognize a bucket width at a time, candidates, broken), and every line's CtcLine
and length equal the reference's CPU device's (carbon/src/pipeline.cpp:138-162: crop_lines, the
int8 executor on 1 - p / 255, ctc_greedy with lengths min(frames, width / 4), through the
reference's compiled code in oracle/_ref) bit for bit; the candidates of lines of the last run
equal the reference's cpu::ctc_topk over that run's logits; a recognize asking for another crop
rule than the one the adapter was opened with throws carbon::Error.

The driver is built where the reference's headers are (oracle/ref.mk, target `adapter`) and
travels as a built file; without it the test is skipped."""
from __future__ import annotations

import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest

from carbon_rec import native, synth
from oracle import oracle as O
from test_gpu_configs import buckets, reference_runs

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
ADAPTER = ROOT / "oracle" / "_ref" / "adapter_run"
TOPK = 5


@pytest.mark.skipif(not ADAPTER.exists() or not O.Reference.available(),
                    reason="the adapter driver or the reference's compiled code (oracle/_ref) is not here")
def test_adapter_behind_pipeline_models(rec_latin, tmp_path):
    ref = O.Reference()
    pages, boxes = synth.pages(31, 4, 2480, 3508, 40)
    bws = [buckets(b) for b in boxes]
    groups = [[0, 1], [2, 3]]
    inp = bytearray(struct.pack("<i", len(pages)))
    for p in pages:
        inp += struct.pack("<ii", p.shape[1], p.shape[0]) + p.tobytes()
    inp += struct.pack("<i", len(groups))
    for g in groups:
        inp += struct.pack("<i", len(g)) + struct.pack(f"<{len(g)}i", *g)
        for p in g:
            runs = native.rows_read(boxes[p], pages[p].shape[0])
            inp += struct.pack("<i", len(runs)) + b"".join(struct.pack("<ii", a, b) for a, b in runs)
    lines = [(gi, p, j) for gi, g in enumerate(groups) for p in g for j in range(len(boxes[p]))]
    inp += struct.pack("<i", len(lines))
    for gi, p, j in lines:
        inp += struct.pack("<iii", gi, p, int(bws[p][j])) + struct.pack("<4d", *boxes[p][j])
    # the last recognize call: the last group's widest bucket, its lines in input order
    last_bw = max(int(bws[p][j]) for p in groups[-1] for j in range(len(boxes[p])))
    last = [(p, j) for p in groups[-1] for j in range(len(boxes[p])) if int(bws[p][j]) == last_bw]
    rows = list(range(min(6, len(last))))
    inp += struct.pack("<ii", len(rows), TOPK) + struct.pack(f"<{len(rows)}i", *rows)
    (tmp_path / "in.bin").write_bytes(bytes(inp))
    (tmp_path / "rec.blob").write_bytes(rec_latin[0].to_blob())
    r = subprocess.run([str(ADAPTER), str(tmp_path / "rec.blob"), str(tmp_path / "in.bin"), str(tmp_path / "out.bin")],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    out, at = (tmp_path / "out.bin").read_bytes(), 0

    def take(fmt, n):
        nonlocal at
        v = np.frombuffer(out, fmt, n, at)
        at += v.nbytes
        return v

    want = reference_runs(ref, rec_latin[2], pages, boxes, bws, want_logits=True)
    chars = 0
    for gi, p, j in lines:
        length, count = take("<i4", 2)
        ids, frames, probs = take("<i4", count), take("<i4", count), take("<f4", count)
        w_ids, w_fr, w_pr = want[p][0][j]
        assert length == want[p][1][j], (p, j)
        assert np.array_equal(ids, w_ids) and np.array_equal(frames, w_fr), (p, j)
        assert np.array_equal(probs.view(np.int32), w_pr.view(np.int32)), (p, j)
        chars += int(count)
    assert chars > 500
    k = int(take("<i4", 1)[0])
    assert k == TOPK
    for r_ in rows:
        t = int(take("<i4", 1)[0])
        ids, logp, blank = take("<i4", t * k).reshape(t, k), take("<f4", t * k).reshape(t, k), take("<f4", t)
        p, j = last[r_]
        e_ids, e_logp, e_blank = ref.ctc_topk(want[p][3][j], int(want[p][1][j]), k)
        assert t == want[p][1][j]
        assert np.array_equal(ids, e_ids), (p, j)
        assert np.array_equal(logp.view(np.int32), e_logp.view(np.int32)), (p, j)
        assert np.array_equal(blank.view(np.int32), e_blank.view(np.int32)), (p, j)
    broken, refused = take("<i4", 2)
    assert broken == 0 and refused == 1
    assert at == len(out)
