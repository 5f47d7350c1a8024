"""crec_ctc_greedy_noalloc: greedy CTC decoding for callers that cannot let a library allocate
device memory (their memory belongs to their own allocator, or was fixed at start-up).  Its
scratch lives in a device array inside the library; this checks it gives crec_ctc_greedy's
results (bit for bit, as every CTC comparison here) on two calls in a row sharing that array,
and refuses sizes beyond it.  Collected last, so a run that stops at its first failure has
already run every other test; it also passes alone in a fresh process (its first call sets the
array up)."""
from __future__ import annotations

import numpy as np
import pytest

from carbon_rec import native

pytestmark = pytest.mark.gpu


def logits_case(seed: int, n: int, classes: int, frames: int):
    rng = np.random.default_rng(seed)
    l = (rng.integers(-24, 25, (n, classes, frames)) * 0.5).astype(np.float32)
    l[:, 0, ::3] += 30.0
    lengths = np.array([frames - (i % 7) * (frames // 9) for i in range(n)], np.int32)
    lengths[-1] = 0
    return l, lengths


def test_no_alloc_decoding_matches_ctc_greedy_twice():
    import torch
    for call, (n, classes, frames) in enumerate(((5, 800, 131), (9, 37, 263))):
        logits, lengths = logits_case(100 + call, n, classes, frames)
        d_logits = torch.from_numpy(logits).cuda()
        d_len = torch.from_numpy(lengths).cuda()
        counts = torch.full((n,), -1, dtype=torch.int32, device="cuda")
        ids = torch.full((n, frames), -1, dtype=torch.int32, device="cuda")
        starts = torch.full((n, frames), -1, dtype=torch.int32, device="cuda")
        probs = torch.full((n, frames), -1.0, dtype=torch.float32, device="cuda")
        native.ctc_greedy_noalloc(d_logits.data_ptr(), n, classes, frames, d_len.data_ptr(), counts.data_ptr(),
                                  ids.data_ptr(), starts.data_ptr(), probs.data_ptr())
        torch.cuda.synchronize()
        want, _ = native.ctc_greedy(d_logits.data_ptr(), n, classes, frames, lengths)
        c, i, s, p = (t.cpu().numpy() for t in (counts, ids, starts, probs))
        for k, line in enumerate(want):
            m = int(c[k])
            assert m == len(line.ids), (call, k)
            assert np.array_equal(i[k, :m], line.ids) and np.array_equal(s[k, :m], line.frames)
            assert np.array_equal(p[k, :m].view(np.int32), line.probs.view(np.int32))


def test_no_alloc_refuses_sizes_beyond_its_scratch():
    with pytest.raises(native.CrecError) as e:
        native.ctc_greedy_noalloc(1, 4096, 800, 256, 1, 1, 1, 1, 1)
    assert e.value.code == native.E_RANGE and "524288" in str(e.value)


def test_no_alloc_without_frames_clears_the_counts():
    """frames == 0: every line's count is 0 (a memset on the caller's array; no kernel)."""
    import torch
    n = 6
    d_len = torch.zeros(n, dtype=torch.int32, device="cuda")
    counts = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    native.ctc_greedy_noalloc(0, n, 800, 0, d_len.data_ptr(), counts.data_ptr(), 0, 0, 0)
    torch.cuda.synchronize()
    assert counts.cpu().numpy().tolist() == [0] * n
