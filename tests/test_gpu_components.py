"""4-connected component labelling kernels (cs_ccl_labels_4 / _compact_4 /
_stats_4) against the CPU oracle (oracle/components.py) and the reference's
own labels and stats (tests/golden/components.npz, made by
tests/golden/make_golden.py from manbo/ops/connected_components.py on a GPU)."""
import numpy as np
import pytest
import torch

from conftest import load_golden as golden
from oracle import components as cc

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _spiral(n):
    m = np.zeros((n, n), bool)
    top, left, bottom, right = 0, 0, n - 1, n - 1
    while top <= bottom and left <= right:
        m[top, left:right + 1] = True
        m[top:bottom + 1, right] = True
        if top + 2 <= bottom:
            m[bottom, left:right + 1] = True
        if left + 2 <= right and top + 2 <= bottom:
            m[top + 2:bottom + 1, left] = True
        top, left, bottom, right = top + 2, left + 2, bottom - 2, right - 2
        if top <= bottom:
            m[top - 1, left - 2 + 1 if left - 1 >= 0 else 0] = True
    return m


def _masks():
    rng = np.random.default_rng(11)
    out = {}
    for (h, w), d in (((13, 19), 0.3), ((64, 97), 0.55), ((257, 131), 0.6), ((40, 40), 0.8)):
        out[f"random_{h}x{w}_{d}"] = rng.random((h, w)) < d
    out["spiral"] = _spiral(63)
    comb = np.zeros((48, 61), bool)
    comb[0, :] = True
    comb[:, ::2] = True                      # one-pixel-wide teeth joined at the top
    out["comb"] = comb
    snake = np.zeros((41, 53), bool)
    snake[::2, :] = True                     # rows joined alternately at the ends
    snake[1::4, -1] = True
    snake[3::4, 0] = True
    out["snake"] = snake
    out["all"] = np.ones((37, 45), bool)
    out["empty"] = np.zeros((20, 30), bool)
    iso = np.zeros((90, 90), bool)
    iso[::2, ::2] = True                     # 2025 components: more than one scan block
    out["isolated"] = iso
    out["one_pixel"] = np.zeros((1, 1), bool) | True
    out["row"] = np.ones((1, 77), bool)
    return out


MASKS = _masks()


@pytest.mark.parametrize("name", sorted(MASKS))
def test_labels_and_stats_match_oracle(name):
    from repo_b200 import components as comp
    mask = MASKS[name]
    t = torch.from_numpy(mask.astype(np.uint8)).to(DEV)
    raw = comp.connected_components_labels_4(t).cpu().numpy()
    np.testing.assert_array_equal(raw, cc.labels_4(mask))
    n, lab, stats, centres = comp.connected_components_with_stats_4(t)
    wn, wlab, wstats, wcent = cc.with_stats_4(mask)
    assert n == wn
    np.testing.assert_array_equal(lab.cpu().numpy(), wlab)
    np.testing.assert_array_equal(stats.cpu().numpy(), wstats)
    np.testing.assert_allclose(centres.cpu().numpy(), wcent, rtol=1e-6, atol=0)


@pytest.mark.parametrize("i", [0, 1, 2])
def test_labels_and_stats_match_reference_golden(i):
    from repo_b200 import components as comp
    g = golden("components")
    t = torch.from_numpy(g[f"m{i}_mask"]).to(DEV)
    np.testing.assert_array_equal(comp.connected_components_labels_4(t).cpu().numpy(),
                                  g[f"m{i}_raw"])
    n, lab, stats, centres = comp.connected_components_with_stats_4(t)
    assert n == int(g[f"m{i}_n"][0])
    np.testing.assert_array_equal(lab.cpu().numpy(), g[f"m{i}_labels"])
    np.testing.assert_array_equal(stats.cpu().numpy(), g[f"m{i}_stats"])
    # the reference sums coordinates with float32 atomics in any order
    np.testing.assert_allclose(centres.cpu().numpy(), g[f"m{i}_centers"], rtol=1e-6, atol=0)


def test_largest_component_centre_on_the_gpu_labels():
    from repo_b200 import components as comp
    mask = np.zeros((7, 9), bool)
    mask[1:6, 2:7] = True
    mask[0, 8] = True
    n, lab, stats, centres = comp.connected_components_with_stats_4(
        torch.from_numpy(mask).to(DEV))
    row, col, label, area, m = comp.select_largest_component_center(lab, stats, centres)
    assert (row, col, label, area) == (3, 4, 2, 25) and int(m.sum()) == 25


def test_manbo_names_run_the_kernels():
    import manbo
    mask = MASKS["random_64x97_0.55"]
    t = torch.from_numpy(mask).to(DEV)
    raw = manbo.ops.connected_components_labels_4_tilelang(t, max_iters=4096, threads=256)
    np.testing.assert_array_equal(raw.cpu().numpy(), cc.labels_4(mask))
    n, lab, stats, centres = manbo.ops.connected_components_with_stats_4_tilelang(t)
    assert n == cc.with_stats_4(mask)[0]
