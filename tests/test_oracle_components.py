"""The component-labelling oracle (oracle/components.py) against the
reference's own relaxation (restated for small masks) and closed-form stats."""
import numpy as np
import pytest

from oracle import components as cc


@pytest.mark.parametrize("seed,density", [(0, 0.3), (1, 0.55), (2, 0.7), (3, 0.0), (4, 1.0)])
def test_raw_labels_match_the_reference_relaxation(seed, density):
    rng = np.random.default_rng(seed)
    mask = rng.random((13, 19)) < density
    np.testing.assert_array_equal(cc.labels_4(mask), cc.relax_labels_4(mask))


def test_stats_layout_and_order():
    mask = np.zeros((6, 8), bool)
    mask[0, 5:8] = True            # component A: first pixel (0, 5)
    mask[2:5, 1] = True            # component B: first pixel (2, 1)
    mask[4, 1:4] = True            # joins B
    mask[5, 7] = True              # component C: first pixel (5, 7)
    n, lab, stats, centres = cc.with_stats_4(mask)
    assert n == 4
    assert lab[0, 6] == 1 and lab[3, 1] == 2 and lab[4, 3] == 2 and lab[5, 7] == 3
    np.testing.assert_array_equal(stats[0], [5, 0, 3, 1, 3])
    np.testing.assert_array_equal(stats[1], [1, 2, 3, 3, 5])
    np.testing.assert_array_equal(stats[2], [7, 5, 1, 1, 1])
    np.testing.assert_allclose(centres[1], [(1 + 1 + 1 + 2 + 3) / 5, (2 + 3 + 4 + 4 + 4) / 5],
                               rtol=1e-7)
    raw = cc.labels_4(mask)
    assert raw[0, 7] == 0 * 8 + 5 + 1 and raw[4, 3] == 2 * 8 + 1 + 1


def test_empty_mask():
    n, lab, stats, centres = cc.with_stats_4(np.zeros((4, 5), bool))
    assert n == 1 and not lab.any() and stats.shape == (0, 5) and centres.shape == (0, 2)


def test_host_wrapper_checks_and_largest_component_centre():
    import torch

    from repo_b200 import components as comp
    with pytest.raises(ValueError, match="mask must be"):
        comp.connected_components_labels_4(torch.zeros(2, 3, 4))
    with pytest.raises(ValueError, match="max_iters"):
        comp.connected_components_labels_4(torch.zeros(2, 3), max_iters=0)
    with pytest.raises(ValueError, match="CUDA"):
        comp.connected_components_with_stats_4(torch.zeros(2, 3))
    # the centre pick is host glue over the stats: check it on the oracle's
    mask = np.zeros((7, 9), bool)
    mask[1:6, 2:7] = True          # 5x5 square: centre (4, 3) in (x, y)
    mask[0, 8] = True
    n, lab, stats, centres = cc.with_stats_4(mask)
    row, col, label, area, m = comp.select_largest_component_center(
        torch.from_numpy(lab), torch.from_numpy(stats), torch.from_numpy(centres))
    # the lone pixel (0, 8) comes first in raster order: the square is label 2
    assert (row, col, label, area) == (3, 4, 2, 25) and int(m.sum()) == 25
    with pytest.raises(ValueError, match="at least one foreground"):
        comp.select_largest_component_center(torch.from_numpy(lab), torch.zeros(0, 5),
                                             torch.zeros(0, 2))


@pytest.mark.parametrize("i", [0, 1, 2])
def test_oracle_matches_reference_golden(i):
    """Raw labels, count, compact labels and stats bit for bit, centres to
    float32 rounding, against the reference's own outputs
    (tests/golden/components.npz, from manbo/ops/connected_components.py run
    by tests/golden/make_golden.py on a GPU)."""
    from conftest import load_golden
    g = load_golden("components")
    mask = g[f"m{i}_mask"].astype(bool)
    np.testing.assert_array_equal(cc.labels_4(mask), g[f"m{i}_raw"])
    n, lab, stats, centres = cc.with_stats_4(mask)
    assert n == int(g[f"m{i}_n"][0])
    np.testing.assert_array_equal(lab, g[f"m{i}_labels"])
    np.testing.assert_array_equal(stats, g[f"m{i}_stats"])
    np.testing.assert_allclose(centres, g[f"m{i}_centers"], rtol=1e-6, atol=0)
