"""bench.py's executed-work count (the denominator of roofline.executed) on a
hand-built one-tile layout."""
import os
import sys

import numpy as np
import pytest

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


def test_reference_work_count_follows_the_per_pixel_stop():
    """raster_work: every pixel visits its tile's intersects up to its stop
    and every edge of each (forward: final_idx where T fell below 1e-4, else
    the tile's end; backward: final_idx)."""
    import torch

    class Trainer:
        h = w = 16
        tbx = 1
        counters = torch.tensor([2, 0, 0, 0], dtype=torch.int32)
        tile_bins = torch.tensor([[0, 2]], dtype=torch.int32)
        prim_sorted = torch.tensor([0, 1], dtype=torch.int32)
        edge_offs = torch.tensor([0, 60, 90], dtype=torch.int32)    # 60 and 30 edges
        fidx = torch.zeros(16, 16, dtype=torch.int32)
        fts = torch.zeros(16, 16)

    tr = Trainer()
    tr.fidx[8:] = 1
    tr.fts[8:] = 0.5          # rows 8-15 never saturate: the forward walks to the end
    pe_f, vis_f, pe_b, vis_b, n = bench.raster_work(tr)
    assert n == 2
    assert (pe_f, vis_f) == (128 * 60 + 128 * 90, 128 * 1 + 128 * 2)
    assert (pe_b, vis_b) == (128 * 60 + 128 * 90, 128 * 1 + 128 * 2)
    tr.fts[8:] = 0.0          # now saturated at final_idx 1: the same stops
    assert bench.raster_work(tr)[:2] == (pe_f, vis_f)
    tr.fidx[8:] = 0           # saturated after intersect 0 everywhere
    assert bench.raster_work(tr)[:4] == (256 * 60, 256, 256 * 60, 256)


def test_profile_summaries_hold_the_traffic_bench_reports():
    """roofline.traffic comes from the committed ncu summaries: each kernel the
    bench reports has its per-launch DRAM bytes there."""
    for kernel, summary in (("raster_backward_kernel", "raster_fill_config2.md"),
                            ("raster_forward_kernel", "raster_fill_config2.md"),
                            ("raster_backward_kernel", "raster_stroke_config4.md")):
        t = bench.ncu_traffic(kernel, summary)
        assert isinstance(t, int) and t > 0, (kernel, summary)
    assert bench.ncu_traffic("raster_backward_kernel", "no_such_summary.md") is None


def test_band_option_parses_and_rejects_bad_specs():
    assert bench.parse_band("3/8") == (3, 8)
    assert bench.parse_band("0/1") == (0, 1)
    for bad in ("8/8", "-1/4", "3", "a/b", "1/0"):
        with pytest.raises(ValueError):
            bench.parse_band(bad)
    args = bench.parse_args(["--workload", "config3", "--band", "2/4", "--host-profile"])
    assert args.band == "2/4" and args.host_profile


def test_reference_arm_line_keeps_the_contract():
    """The reference arm (the C oracle on the host) prints the repo arm's
    metric, unit and workload with impl, cpu_baseline and a copy-free e2e."""
    args = bench.parse_args(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    res = bench.run_reference(args, 0, 1)
    assert res["impl"] == "reference" and res["metric"] == bench.METRIC
    assert res["unit"] == bench.UNIT and res["higher_is_better"] is True
    assert res["config"]["workload"] == bench.WORKLOAD_CONFIG2
    assert res["value"] > 0 and res["steps"] == 1
    assert res["cpu_baseline"]["value"] == res["value"] and res["cpu_baseline"]["cores"] >= 1
    assert res["e2e"] == {"value": res["value"], "unit": bench.UNIT,
                          "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert bench.run_reference(args, 1, 2) is None  # other ranks exit without work
