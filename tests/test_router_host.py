"""The layer router's host logic on CPU (host/fpga_layers.py:125-134, 258-284):
counting calls, flags and agreement, and the summary's wording."""

from __future__ import annotations

import numpy as np


def test_counters_and_summary():
    from insitu_b200.router import RouteCounters
    c = RouteCounters(n_layers=2, verified=True)
    assert "NEVER ASKED" in c.summary()
    st = np.zeros((1, 2, 6), np.int64)
    st[0, 1, 1] = 3                            # rescales
    c.add_call(1, 0.5, st, clips=0)
    assert (c.steps, c.tokens, c.rescales, c.flagged) == (1, 1, 3, 0)
    st2 = np.zeros((2, 2, 6), np.int64)
    st2[1, 0, 3] = 1                           # an accumulator overflow
    c.add_call(2, 0.25, st2, clips=0)
    c.add_call(1, 0.25, np.zeros((1, 2, 6)), clips=4)
    assert (c.steps, c.tokens, c.overflows, c.clips, c.flagged) == (3, 4, 1, 4, 2)
    assert abs(c.dev_ms - 1.0) < 1e-12

    got = np.arange(2 * 4 * 64).reshape(2, 4, 64)
    assert c.compare(got, got.reshape(2, 256).copy()) is None
    bad = got.copy()
    bad[1, 2, 7] += 1
    assert c.compare(got, bad) == "1 of 512 channels"
    assert "shape" in c.compare(got, got[:1])
    assert (c.agree, c.disagree) == (1, 2)
    s = c.summary()
    assert "3 (2 layers x 1 calls, 4 tokens)" in s
    assert "1 exact, 2 different" in s
    assert "overflows 1, seam clips 4, steps with a range/saturation flag 2" in s


def test_unverified_summary_has_no_agreement_line():
    from insitu_b200.router import RouteCounters
    c = RouteCounters(n_layers=1, verified=False)
    c.add_call(1, 1.0, np.zeros((1, 1, 6)), 0)
    assert "agreement" not in c.summary()
