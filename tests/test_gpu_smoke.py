"""The driver's smoke step, `__graft_entry__.smoke()`: three lines of a small page through the
library on cuda:0, the crops, every logit and the decodings bit-exact against the oracle."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def test_smoke():
    import __graft_entry__

    __graft_entry__.smoke()
