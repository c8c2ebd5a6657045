"""Parity at the benchmark configurations' full sizes, against the CPU oracle.

* Config 3 (2040x1356, 4096 closed paths x 6 segments, S=16): the whole image
  on one GPU, and the same image rendered as 8 tile-row bands (the multi-GPU
  partition, here one band after the other on one GPU) whose rows stitch to
  the oracle's image and whose gradients sum to the oracle's.
* Config 4 (1024x1024, 2048 open strokes): forward and backward of all
  strokes through the drop-in API.

Tolerances as in test_gpu_parity: integer outputs bit for bit, images within
1e-6 of the oracle (identical arithmetic), gradients within 1e-3 relative L2
and 1e-5 absolute (or 1e-3 of the largest magnitude).
"""
import numpy as np
import pytest
import torch

import oracle
from repo_b200 import bands, render, scenes

from test_gpu_parity import (_np, _t, assert_grad_close, check_binning, fill_inputs,
                             gpu_fill, gpu_fill_backward)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def config3():
    sc = scenes.config3()
    args = fill_inputs(sc)
    cn, offs, col, op, dep, h, w, bg, rules, aa, s = args
    st = oracle.render_fill(cn, offs, col, op, dep, h, w, bg, fill_rules=rules, aa_widths=aa,
                            samples=s)
    v_out = scenes.seeded_grad(31, h, w).numpy()
    want = oracle.fill_backward(st, v_out, True, False)
    return sc, args, st, v_out, want


def test_config3_full_image_matches_oracle(config3):
    sc, args, st, v_out, want = config3
    cn, offs, col, op, dep, h, w, bg, rules, aa, s = args
    b, inv, out, fts, fidx = gpu_fill(*args)
    check_binning(b, st)
    np.testing.assert_array_equal(_np(fidx), st["final_idx"])
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6
    assert np.abs(_np(fts) - st["final_Ts"]).max() <= 1e-6
    got = gpu_fill_backward(b, col, op, inv, rules, bg, fts, fidx, v_out, h, w)
    for k in ["v_colors", "v_opacities", "v_inv_sigma2s", "v_cubics_px", "curve_contrib_rgb"]:
        assert_grad_close(got[k], want[k], k)


def test_config3_eight_bands_stitch_to_the_oracle(config3):
    sc, args, st, v_out, want = config3
    cn, offs, col, op, dep, h, w, bg, rules, aa, s = args
    split = bands.balanced_bands(bands.tile_row_work(sc, torch.device("cuda")), 8)
    assert split[0][0] == 0 and split[-1][1] == (h + 15) // 16
    image = np.full_like(st["image"], np.nan)
    # final_idx indexes the band's own intersect list: compare the primitive
    # it names (pixels where something was composited)
    final_prim = np.full_like(st["final_idx"], -7)
    sums = {}
    for band in split:
        b, inv, out, fts, fidx = gpu_fill(*args, tile_rows=band)
        y0, y1 = band[0] * 16, min(band[1] * 16, h)
        image[y0:y1] = _np(out)[y0:y1]
        final_prim[y0:y1] = _np(b.prim_ids_sorted)[_np(fidx)[y0:y1]]
        # the band's gradients: only its rows carry an image gradient
        vb = np.zeros_like(v_out)
        vb[y0:y1] = v_out[y0:y1]
        got = gpu_fill_backward(b, col, op, inv, rules, bg, fts, fidx, vb, h, w)
        for k in ["v_colors", "v_opacities", "v_inv_sigma2s", "v_cubics_px"]:
            sums[k] = got[k] + sums.get(k, 0.0)
    hit = st["final_Ts"] < 1.0
    np.testing.assert_array_equal(final_prim[hit], st["prim_ids_sorted"][st["final_idx"]][hit])
    assert np.abs(image - st["image"]).max() <= 1e-6
    for k in ["v_colors", "v_opacities", "v_inv_sigma2s", "v_cubics_px"]:
        assert_grad_close(sums[k], want[k], k)


def test_config4_all_strokes_forward_and_backward_match_oracle():
    import manbo
    sc = scenes.config4()
    h, w, s = sc.height, sc.width, sc.samples
    p = int(sc.cubics_norm().shape[0])
    offs = np.arange(p + 1, dtype=np.int32)
    st = oracle.render_stroke(sc.cubics_norm().numpy(), offs, sc.colors.numpy(),
                              sc.opacities.numpy(), sc.stroke_widths.numpy(), sc.depths.numpy(),
                              h, w, sc.background.numpy(), aa_widths=sc.aa_widths.numpy(),
                              samples=s)
    v_out = scenes.seeded_grad(41, h, w).numpy()
    want = oracle.stroke_backward(st, v_out)
    cn = _t(sc.cubics_norm()).requires_grad_(True)
    col = _t(sc.colors).requires_grad_(True)
    op = _t(sc.opacities).requires_grad_(True)
    sw = _t(sc.stroke_widths).requires_grad_(True)
    aw = _t(sc.aa_widths).requires_grad_(True)
    out = manbo.ops.render_cubic_polyline_splat_tilelang(
        cn, _t(offs), col, op, sw, _t(sc.depths), h, w, 16, 16, _t(sc.background),
        aa_widths=aw, distance_samples=s)
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6
    (out * _t(v_out)).sum().backward()
    assert_grad_close(_np(cn.grad), want["v_cubics_norm"], "v_cubics_norm")
    assert_grad_close(_np(col.grad), want["v_colors"], "v_colors")
    assert_grad_close(_np(op.grad), want["v_opacities"], "v_opacities")
    assert_grad_close(_np(sw.grad), want["v_stroke_widths"], "v_stroke_widths")
    assert_grad_close(_np(aw.grad), want["v_aa_widths"], "v_aa_widths")
