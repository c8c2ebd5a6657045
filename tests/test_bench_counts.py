"""bench.py's executed-work count (the denominator of roofline.executed) on a
hand-built one-tile layout."""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _layout():
    h = w = 16
    bins = np.array([[0, 2]], np.int32)                  # one tile, intersects 0 and 1
    istrips = np.zeros((2, 4, 2), np.int32)
    istrips[0, :, 1] = [2, 0, 0, 1]                      # records per strip
    istrips[1, :, 1] = [0, 3, 0, 0]
    fidx = np.ones((h, w), np.int32)
    fts = np.full((h, w), 0.5, np.float32)
    fidx[4:8] = 0                                        # strip 1: saturated after intersect 0
    fts[4:8] = 0.0
    return h, w, bins, istrips, fidx, fts


def test_executed_work_counts_walked_records_and_active_visits():
    h, w, bins, istrips, fidx, fts = _layout()
    pe_f, vis_f, pe_b, vis_b = bench.executed_work(bins, istrips, None, None, fidx, fts, h, w,
                                                   1, 2)
    # forward: strips 0, 2, 3 walk both intersects, strip 1 stops after
    # intersect 0; records 2 + 0 + 0 + 1, active (intersect, strip) pairs 2
    assert (pe_f, vis_f) == (64 * 3, 64 * 2)
    # backward: each strip from its largest final_idx down: the same here
    assert (pe_b, vis_b) == (64 * 3, 64 * 2)


def test_executed_work_with_visit_lists():
    h, w, bins, istrips, fidx, fts = _layout()
    # strip s's list at 3 s: count, then ids
    visits = np.array([1, 0, 0,   1, 1, 0,   0, 0, 0,   2, 0, 1], np.int32)
    _, _, pe_b, vis_b = bench.executed_work(bins, istrips, None, None, fidx, fts, h, w, 1, 2,
                                            visits=visits)
    assert pe_b == 64 * (2 + 3 + 0 + 1) and vis_b == 64 * (1 + 1 + 0 + 2)
