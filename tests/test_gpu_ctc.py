"""crec_ctc_greedy (carbon::cuda::ctc_greedy) on device logits against the oracle's ctc_greedy,
bit for bit, on the reference test's cases: coarse grids with ties, blank-heavy frames, lengths
short of the frames, 1 to 800 classes."""
from __future__ import annotations

import numpy as np
import pytest

from carbon_rec import native

pytestmark = pytest.mark.gpu


def cases():
    rng = np.random.default_rng(17)
    for spread in (0.5, 3.0):
        for classes in (1, 7, 800):
            for frames in (1, 13, 131, 263):
                l = (rng.integers(-24, 25, (3, classes, frames)) * spread).astype(np.float32)
                l[:, 0, ::3] += 30.0
                yield l, np.array([frames - frames // 5, frames, 0], np.int32)


def test_ctc_greedy_on_device_logits_is_the_reference(orc):
    import torch
    for logits, lengths in cases():
        d = torch.from_numpy(logits).cuda()
        got, glen = native.ctc_greedy(d.data_ptr(), *logits.shape, lengths)
        torch.cuda.synchronize()
        want, _, _ = orc.ctc_greedy(logits, lengths)
        assert np.array_equal(glen, np.minimum(lengths, logits.shape[2]))
        for g, (ids, fr, pr) in zip(got, want):
            assert np.array_equal(g.ids, ids) and np.array_equal(g.frames, fr)
            assert np.array_equal(g.probs.view(np.int32), pr.view(np.int32))


def test_ctc_greedy_reports_errors():
    with pytest.raises(native.CrecError) as e:
        native.ctc_greedy(0, 2, 0, 5, [1, 1])
    assert e.value.code == native.E_INVALID
