"""The reference's CTC head file (<model>.head.bin, "CTCHEAD1": int32 classes, int32 k, the weight
[classes][k] in float16, the bias [classes] in float32; carbon/src/lines.cpp:372-398) through
crec_ctc_head_blob: it accepts and refuses the files the reference's own load_ctc_head accepts and
refuses (oracle/_ref), and a head it accepts becomes the same FP16 blob as the package's ONNX
compile of that layer (model.make_head with the file's weights), byte for byte.  The library is
only loaded here; nothing runs on a GPU."""
from __future__ import annotations

import struct

import numpy as np
import pytest

from carbon_rec import model, native, netdef
from oracle import oracle as O


def head_file(classes: int, k: int, seed: int) -> tuple[bytes, np.ndarray, np.ndarray]:
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.06, (classes, k)).astype(np.float16)
    b = rng.normal(0.0, 0.5, classes).astype(np.float32)
    return b"CTCHEAD1" + struct.pack("<ii", classes, k) + w.tobytes() + b.tobytes(), w, b


@pytest.mark.parametrize("classes,k", [(800, 256), (33, 128), (400, 320), (1500, 192)])
def test_head_file_is_the_compiled_layer(classes, k):
    f, w, b = head_file(classes, k, classes + k)
    blob = native.ctc_head_blob(f)
    sample = np.random.default_rng(0).normal(0.0, 1.0, (1, k, 1, 8)).astype(np.float32)  # calibrates the INT8 file only
    fp, _, _ = model.make_head(k, classes, w.astype(np.float32), b, sample)
    assert blob == netdef.compile_model(fp).to_blob()


def bad_files():
    good, _, _ = head_file(7, 16, 1)
    return {
        "magic": b"CTCHEAD2" + good[8:],
        "short header": good[:12],
        "truncated": good[:-1],
        "trailing byte": good + b"\0",
        "no classes": b"CTCHEAD1" + struct.pack("<ii", 0, 16),
        "negative k": b"CTCHEAD1" + struct.pack("<ii", 7, -16) + good[16:],
    }


@pytest.mark.parametrize("name", list(bad_files()))
def test_refused_as_the_reference_refuses(name, tmp_path):
    data = bad_files()[name]
    with pytest.raises(native.CrecError) as e:
        native.ctc_head_blob(data)
    assert e.value.code == native.E_MODEL
    if O.Reference.available():
        path = tmp_path / "rec.head.bin"
        path.write_bytes(data)
        with pytest.raises(ValueError):
            O.Reference().load_ctc_head(path)


@pytest.mark.skipif(not O.Reference.available(), reason="the reference's compiled code (oracle/_ref) is not here")
def test_accepted_as_the_reference_reads_it(tmp_path):
    f, w, b = head_file(120, 64, 9)
    path = tmp_path / "rec.head.bin"
    path.write_bytes(f)
    classes, k, rw, rb = O.Reference().load_ctc_head(path)
    assert (classes, k) == (120, 64)
    assert np.array_equal(rw.view(np.uint16), w.view(np.uint16)) and np.array_equal(rb.view(np.int32), b.view(np.int32))
    native.ctc_head_blob(f)  # and this library takes it
