"""The idle-gap analysis of ``benchmarks/step_profile.py`` on synthetic
timelines (the profiler itself needs a GPU)."""

import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                "benchmarks"))
import step_profile as sp  # noqa: E402


def test_gaps_between_serial_kernels():
    ev = [(0, 10, "a"), (12, 20, "b"), (20, 30, "c"), (130, 140, "d")]
    assert sp.idle_gaps(ev) == [(2, "a", "b"), (100, "c", "d")]


def test_overlapping_streams_leave_no_false_gap():
    # "long" on one stream covers "x" and "y" on another
    ev = [(0, 100, "long"), (10, 20, "x"), (30, 40, "y"), (105, 110, "z")]
    assert sp.idle_gaps(ev) == [(5, "long", "z")]


def test_report_bins():
    text = sp.gap_report([(1.0, "a", "b"), (5.0, "b", "c"), (50.0, "c", "d"), (500.0, "d", "e")])
    assert text.startswith("idle 0.556 ms in 4 gaps")
    assert "< 2 us 1" in text and "2-10 us 1" in text and ">= 100 us 1" in text
    assert text.splitlines()[1].strip().startswith("500.0 us  after d  before e")
