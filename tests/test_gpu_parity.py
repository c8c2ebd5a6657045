"""GPU parity of the sm_100a kernels against the CPU oracle and the reference's
golden vectors.

Tolerances (north star): tile lists, sort order and every integer output bit
for bit; images within 1e-4 abs; gradients within 1e-3 relative L2 and 1e-5
abs.  Against the oracle the per-pixel arithmetic is identical by
construction, so the forward image is expected to match exactly and only the
order of gradient accumulation differs.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden, rel_l2
from repo_b200 import render, scenes

pytestmark = pytest.mark.gpu

DEV = "cuda"
IMG_ATOL = 1e-4
GRAD_REL = 1e-3
GRAD_ABS = 1e-5


def _t(a, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV)


def _np(t):
    return t.detach().cpu().numpy()


def assert_grad_close(got, want, name):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    r = rel_l2(got, want)
    a = float(np.abs(got - want).max()) if got.size else 0.0
    scale = float(np.abs(want).max()) if want.size else 0.0
    assert r <= GRAD_REL, f"{name}: rel L2 {r:.3e}"
    assert a <= max(GRAD_ABS, GRAD_REL * scale), f"{name}: max abs {a:.3e} (scale {scale:.3e})"


def gpu_fill(cubics_norm, offs, colors, opac, depths, h, w, bg, rules, aa, s, tile_rows=None):
    widths = torch.clamp(_t(aa, torch.float32), min=1e-4)
    inv = render._inv_sigma2(widths)
    col, op, rl = _t(colors, torch.float32), _t(opac, torch.float32), _t(rules, torch.int32)
    b = render.bin_primitives(_t(cubics_norm, torch.float32), _t(offs, torch.int32),
                              _t(depths, torch.float32), widths, h, w, s, colors=col,
                              opacities=op, inv_sigma2s=inv, fill_rules=rl, tile_rows=tile_rows)
    out, fts, fidx = render.forward_raster(b, _t(bg, torch.float32), h, w)
    return b, inv, out, fts, fidx


def gpu_fill_backward(b, colors, opac, inv, rules, bg, fts, fidx, v_out, h, w):
    v_edges, v_colors, v_opac, v_inv, _, contrib, icontrib = render.raster_backward(
        b, int(np.asarray(colors).shape[0]), _t(bg, torch.float32), fts, fidx,
        _t(v_out, torch.float32), h, w, collect_contrib=True, collect_isect_contrib=True)
    v_cpx = render.edge_grads_to_cubics(v_edges, int(b.cubics_px.shape[0]), b.samples)
    return {"v_edges": _np(v_edges), "v_colors": _np(v_colors), "v_opacities": _np(v_opac),
            "v_inv_sigma2s": _np(v_inv), "v_cubics_px": _np(v_cpx),
            "curve_contrib_rgb": _np(contrib), "curve_isect_contrib": _np(icontrib)}


def fill_inputs(sc):
    return (sc.cubics_norm().numpy(), sc.seg_offsets().numpy(), sc.colors.numpy(),
            sc.opacities.numpy(), sc.depths.numpy(), sc.height, sc.width,
            sc.background.numpy(), sc.fill_rules.numpy(), sc.aa_widths.numpy(), sc.samples)


def check_binning(b, st):
    np.testing.assert_array_equal(_np(b.cubics_px), st["cubics_px"])
    np.testing.assert_array_equal(_np(b.edges_px), st["edges_px"])
    np.testing.assert_array_equal(_np(b.prim_tile_ranges), st["prim_tile_ranges"])
    np.testing.assert_array_equal(_np(b.num_tiles_hit), st["num_tiles_hit"])
    np.testing.assert_array_equal(_np(b.tile_bins), st["tile_bins"])
    np.testing.assert_array_equal(_np(b.prim_ids_sorted), st["prim_ids_sorted"])
    np.testing.assert_array_equal(_np(b.isect_ids_sorted), st["isect_ids_sorted"])


FILL_SCENES = {
    "small_a": lambda: scenes.small_fill_scene(101),
    "small_b": lambda: scenes.small_fill_scene(102, h=37, w=53, paths=11, samples=5),
    "ties": lambda: _with_ties(scenes.small_fill_scene(103, paths=9, mixed=False)),
    "config1": scenes.config1,
    "config2": scenes.config2,
}


def _with_ties(sc):
    sc.depths = torch.full_like(sc.depths, 0.25)
    return sc


@pytest.mark.parametrize("name", list(FILL_SCENES))
def test_fill_forward_matches_oracle(name):
    sc = FILL_SCENES[name]()
    args = fill_inputs(sc)
    cn, offs, col, op, dep, h, w, bg, rules, aa, s = args
    st = oracle.render_fill(cn, offs, col, op, dep, h, w, bg, fill_rules=rules, aa_widths=aa,
                            samples=s)
    b, inv, out, fts, fidx = gpu_fill(*args)
    check_binning(b, st)
    np.testing.assert_array_equal(_np(fidx), st["final_idx"])
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6
    assert np.abs(_np(fts) - st["final_Ts"]).max() <= 1e-6


@pytest.mark.parametrize("name", list(FILL_SCENES))
def test_fill_backward_matches_oracle(name):
    sc = FILL_SCENES[name]()
    args = fill_inputs(sc)
    cn, offs, col, op, dep, h, w, bg, rules, aa, s = args
    st = oracle.render_fill(cn, offs, col, op, dep, h, w, bg, fill_rules=rules, aa_widths=aa,
                            samples=s)
    v_out = scenes.seeded_grad(7, h, w).numpy()
    want = oracle.fill_backward(st, v_out, True, True)
    b, inv, out, fts, fidx = gpu_fill(*args)
    got = gpu_fill_backward(b, col, op, inv, rules, bg, fts, fidx, v_out, h, w)
    for k in ["v_colors", "v_opacities", "v_inv_sigma2s", "v_cubics_px", "curve_contrib_rgb",
              "curve_isect_contrib"]:
        assert_grad_close(got[k], want[k], k)


@pytest.mark.parametrize("case", ["fill_small_a", "fill_small_b", "fill_ties", "fill_config1"])
def test_fill_matches_reference_golden(case):
    g = load_golden(case)
    h, w, s = (int(v) for v in g["hw_s"])
    args = (g["cubics_norm"], g["offs"], g["colors"], g["opacities"], g["depths"], h, w,
            g["background"], g["fill_rules"], g["aa_widths"], s)
    b, inv, out, fts, fidx = gpu_fill(*args)
    for k in ["cubics_px", "edges_px", "prim_tile_ranges", "num_tiles_hit", "tile_bins",
              "prim_ids_sorted", "isect_ids_sorted"]:
        np.testing.assert_array_equal(_np(getattr(b, k)), g[k], err_msg=k)
    np.testing.assert_array_equal(_np(fidx), g["final_idx"])
    assert np.abs(_np(out) - g["image"]).max() <= IMG_ATOL
    assert np.abs(_np(fts) - g["final_Ts"]).max() <= IMG_ATOL
    got = gpu_fill_backward(b, g["colors"], g["opacities"], inv, g["fill_rules"],
                            g["background"], fts, fidx, g["v_output"], h, w)
    for k in ["v_colors", "v_opacities", "v_inv_sigma2s", "v_cubics_px", "curve_contrib_rgb",
              "curve_isect_contrib"]:
        assert_grad_close(got[k], g[k], k)


def test_fill_api_autograd_matches_reference_golden():
    import manbo
    g = load_golden("fill_config1")
    h, w, s = (int(v) for v in g["hw_s"])
    cn = _t(g["cubics_norm"]).requires_grad_(True)
    col = _t(g["colors"]).requires_grad_(True)
    op = _t(g["opacities"]).requires_grad_(True)
    aw = _t(g["aa_widths"]).requires_grad_(True)
    out = manbo.ops.render_cubic_fill_splat_tilelang(
        cn, _t(g["offs"]), col, op, _t(g["depths"]), h, w, 16, 16, _t(g["background"]),
        fill_rules=_t(g["fill_rules"]), aa_widths=aw, distance_samples=s)
    assert np.abs(_np(out) - g["api_image"]).max() <= IMG_ATOL
    (out * _t(g["v_output"])).sum().backward()
    assert_grad_close(_np(cn.grad), g["api_v_cubics_norm"], "v_cubics_norm")
    assert_grad_close(_np(col.grad), g["api_v_colors"], "v_colors")
    assert_grad_close(_np(op.grad), g["api_v_opacities"], "v_opacities")
    assert_grad_close(_np(aw.grad), g["api_v_aa_widths"], "v_aa_widths")


def test_stage_wrappers_match_reference_golden():
    from manbo.ops import cubic_splatting as cs
    from manbo.ops import tile_bins as tb
    g = load_golden("fill_config1")
    h, w, s = (int(v) for v in g["hw_s"])
    tbounds = ((w + 15) // 16, (h + 15) // 16, 1)
    cn = _t(g["cubics_norm"])
    offs = _t(g["offs"])
    widths = torch.clamp(_t(g["aa_widths"]), min=1e-4)
    support = torch.repeat_interleave(widths * 3.0, (offs[1:] - offs[:-1]).long())
    cpx, seg_rng, seg_hit = cs.project_cubics_2d_forward_tilelang(
        cn, torch.zeros(cn.shape[0], device=DEV), support, h, w, tbounds)
    np.testing.assert_array_equal(_np(cpx), g["cubics_px"])
    np.testing.assert_array_equal(_np(seg_rng), g["seg_tile_ranges"])
    np.testing.assert_array_equal(_np(seg_hit), g["seg_num_tiles"])
    edges, peo, _, _, _ = cs._flatten_cubics_to_edges(cpx, offs, distance_samples=s)
    np.testing.assert_array_equal(_np(edges), g["edges_px"])
    np.testing.assert_array_equal(_np(peo), g["prim_edge_offsets"])
    pr, hit = cs._primitive_tile_ranges_from_segment_tile_ranges(seg_rng, offs, tbounds)
    np.testing.assert_array_equal(_np(pr), g["prim_tile_ranges"])
    cum = torch.cumsum(hit, 0, dtype=torch.int32)
    ids, pids = cs.map_cubic_to_intersects_tilelang(pr, _t(g["depths"]), cum, tbounds)
    np.testing.assert_array_equal(_np(ids), g["isect_ids"])
    np.testing.assert_array_equal(_np(pids), g["prim_ids"])
    ids_s, order = torch.sort(ids, stable=True)
    pids_s = torch.gather(pids, 0, order)
    bins = tb.get_tile_bin_edges_tilelang(int(ids.numel()), ids_s, num_tiles=tbounds[0] * tbounds[1],
                                          compact=True)
    np.testing.assert_array_equal(_np(bins), g["tile_bins"])
    rng = cs._build_fill_isect_edge_ranges(pids_s, peo, num_edges=int(edges.shape[0]))
    np.testing.assert_array_equal(_np(rng), g["isect_edge_ranges"])
    out, fts, fidx = cs.rasterize_cubic_fill_forward_tilelang(
        tbounds, (16, 16, 1), (w, h, 1), pids_s, bins, cpx, offs, _t(g["colors"]),
        _t(g["opacities"]), _t(g["fill_rules"]), _t(g["background"]),
        aa_widths=_t(g["aa_widths"]), edges_px=edges, isect_edge_ranges=rng, distance_samples=s)
    assert np.abs(_np(out) - g["image"]).max() <= IMG_ATOL
    np.testing.assert_array_equal(_np(fidx), g["final_idx"])
    vc, vcol, vop, vinv = cs.rasterize_cubic_fill_backward_tilelang(
        tbounds, (16, 16, 1), (w, h, 1), pids_s, bins, cpx, offs, _t(g["colors"]),
        _t(g["opacities"]), _t(g["fill_rules"]), _t(g["background"]), fts, fidx,
        _t(g["v_output"]), aa_widths=_t(g["aa_widths"]), edges_px=edges, isect_edge_ranges=rng,
        distance_samples=s)
    assert_grad_close(_np(vc), g["v_cubics_px"], "v_cubics_px")
    assert_grad_close(_np(vcol), g["v_colors"], "v_colors")


def test_stroke_matches_oracle_and_reference_golden():
    import manbo
    g = load_golden("stroke_small")
    h, w, s = (int(v) for v in g["hw_s"])
    st = oracle.render_stroke(g["cubics_norm"], g["offs"], g["colors"], g["opacities"],
                              g["stroke_widths"], g["depths"], h, w, g["background"],
                              aa_widths=g["aa_widths"], samples=s)
    cn = _t(g["cubics_norm"]).requires_grad_(True)
    col = _t(g["colors"]).requires_grad_(True)
    op = _t(g["opacities"]).requires_grad_(True)
    sw = _t(g["stroke_widths"]).requires_grad_(True)
    aw = _t(g["aa_widths"]).requires_grad_(True)
    out = manbo.ops.render_cubic_polyline_splat_tilelang(
        cn, _t(g["offs"]), col, op, sw, _t(g["depths"]), h, w, 16, 16, _t(g["background"]),
        aa_widths=aw, distance_samples=s)
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6
    assert np.abs(_np(out) - g["image"]).max() <= IMG_ATOL
    (out * _t(g["v_output"])).sum().backward()
    want = oracle.stroke_backward(st, g["v_output"])
    assert_grad_close(_np(cn.grad), want["v_cubics_norm"], "oracle v_cubics_norm")
    assert_grad_close(_np(sw.grad), want["v_stroke_widths"], "oracle v_stroke_widths")
    assert_grad_close(_np(cn.grad), g["api_v_cubics_norm"], "v_cubics_norm")
    assert_grad_close(_np(col.grad), g["api_v_colors"], "v_colors")
    assert_grad_close(_np(op.grad), g["api_v_opacities"], "v_opacities")
    assert_grad_close(_np(sw.grad), g["api_v_stroke_widths"], "v_stroke_widths")
    assert_grad_close(_np(aw.grad), g["api_v_aa_widths"], "v_aa_widths")


def test_stroke_config4_subset_matches_oracle():
    sc = scenes.config4()
    keep = 300
    cn = sc.cubics_norm()[:keep]
    offs = np.arange(keep + 1, dtype=np.int32)
    h, w = 256, 256  # render the top-left corner only: strokes mostly off-image
    args = dict(samples=sc.samples)
    st = oracle.render_stroke(cn.numpy(), offs, sc.colors[:keep].numpy(),
                              sc.opacities[:keep].numpy(), sc.stroke_widths[:keep].numpy(),
                              sc.depths[:keep].numpy(), h, w, sc.background.numpy(),
                              aa_widths=sc.aa_widths[:keep].numpy(), **args)
    import manbo
    out = manbo.ops.render_cubic_polyline_splat_tilelang(
        _t(cn), _t(offs), _t(sc.colors[:keep]), _t(sc.opacities[:keep]),
        _t(sc.stroke_widths[:keep]), _t(sc.depths[:keep]), h, w, 16, 16, _t(sc.background),
        aa_widths=_t(sc.aa_widths[:keep]), distance_samples=sc.samples)
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6


def test_ring_segments_match_reference_golden():
    import manbo
    g = load_golden("ring_segments")
    cp = _t(g["control_points"]).requires_grad_(True)
    seg, offs = manbo.ops.closed_cubic_fill_segments_tilelang(cp, subdiv=4)
    np.testing.assert_array_equal(_np(offs), g["offsets"])
    assert np.abs(_np(seg) - g["segments"]).max() <= 1e-5
    (seg * _t(g["grad_segments"])).sum().backward()
    assert np.abs(_np(cp.grad) - g["grad_control_points"]).max() <= 1e-5


def test_metrics_match_reference_golden():
    import manbo
    g = load_golden("metrics")
    x = _t(g["x"]).requires_grad_(True)
    y = _t(g["y"])
    loss = manbo.mse_loss_tilelang(x, y)
    assert abs(float(loss) - float(g["mse"])) <= 1e-6 * float(g["mse"])
    loss.backward()
    np.testing.assert_allclose(_np(x.grad), g["mse_grad"], rtol=1e-6, atol=1e-10)
    assert abs(float(manbo.psnr(x.detach(), y)) - float(g["psnr"])) <= 1e-4
    assert abs(float(manbo.ssim(x.detach(), y)) - float(g["ssim"])) <= 1e-5
    np.testing.assert_allclose(_np(manbo.ssim(x.detach(), y, size_average=False)),
                               g["ssim_per_image"], atol=1e-5)


def test_metrics_full_size_match_oracle():
    import manbo
    sc = scenes.config2()
    gen = torch.Generator().manual_seed(5)
    x = torch.rand(sc.target.shape, generator=gen)
    xg, yg = _t(x), _t(sc.target)
    assert abs(float(manbo.ssim(xg, yg)) - oracle.ssim(x.numpy(), sc.target.numpy())) <= 1e-5
    m = oracle.mse(x.numpy(), sc.target.numpy())
    assert abs(float(manbo.mse_loss_tilelang(xg, yg)) - m) <= 1e-5 * m
    assert abs(float(manbo.psnr(xg, yg)) - oracle.psnr(x.numpy(), sc.target.numpy())) <= 1e-4


# --------------------------------------------------------------------------
# edge cases


def test_empty_scene_returns_background():
    import manbo
    bg = torch.tensor([0.2, 0.4, 0.6], device=DEV)
    out = manbo.ops.render_cubic_fill_splat_tilelang(
        torch.zeros((0, 4, 2), device=DEV), torch.zeros((1,), dtype=torch.int32, device=DEV),
        torch.zeros((0, 3), device=DEV), torch.zeros((0,), device=DEV),
        torch.zeros((0,), device=DEV), 20, 30, 16, 16, bg)
    assert out.shape == (20, 30, 3)
    assert torch.equal(out, bg.view(1, 1, 3).expand(20, 30, 3))


def test_offscreen_scene_returns_background_and_no_grad():
    import manbo
    sc = scenes.small_fill_scene(5)
    ring = sc.ring + 10000.0
    cn = scenes.px_to_norm(scenes.ring_to_cubics(ring), sc.width, sc.height).to(DEV)
    cn.requires_grad_(True)
    out = manbo.ops.render_cubic_fill_splat_tilelang(
        cn, _t(sc.seg_offsets()), _t(sc.colors), _t(sc.opacities), _t(sc.depths), sc.height,
        sc.width, 16, 16, _t(sc.background))
    assert torch.equal(out, _t(sc.background).view(1, 1, 3).expand_as(out))


def test_ragged_offsets_and_empty_primitive():
    sc = scenes.small_fill_scene(17, paths=5, segs=4)
    cn = sc.cubics_norm().numpy()
    # primitive sizes 4, 0, 8, 3, 5 segments: cut and re-group the 20 segments
    offs = np.array([0, 4, 4, 12, 15, 20], np.int32)
    p = 5
    args = (cn, offs, sc.colors.numpy(), sc.opacities.numpy(), sc.depths.numpy(), sc.height,
            sc.width, sc.background.numpy(), sc.fill_rules.numpy(), sc.aa_widths.numpy(),
            sc.samples)
    st = oracle.render_fill(*args[:8], fill_rules=args[8], aa_widths=args[9], samples=args[10])
    b, inv, out, fts, fidx = gpu_fill(*args)
    check_binning(b, st)
    np.testing.assert_array_equal(_np(fidx), st["final_idx"])
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6
    assert p == offs.shape[0] - 1


def test_bad_offsets_raise_value_error():
    import manbo
    sc = scenes.small_fill_scene(3)
    offs = sc.seg_offsets().clone()
    offs[-1] -= 1
    with pytest.raises(ValueError, match="primitive_seg_offsets"):
        manbo.ops.render_cubic_fill_splat_tilelang(
            _t(sc.cubics_norm()), _t(offs), _t(sc.colors), _t(sc.opacities), _t(sc.depths),
            sc.height, sc.width, 16, 16, _t(sc.background))


def test_primitive_larger_than_staging_capacity_is_split():
    # one path of 48 segments x 23 edges = 1104 edges: a strip sees more of its
    # records than one warp buffer holds (64), so intersects span buffer chunks
    gen = torch.Generator().manual_seed(9)
    g = 48
    centre = torch.tensor([[40.0, 30.0]])
    ring = scenes.circle_rings(centre, torch.tensor([25.0]), torch.tensor([0.3]), g)
    ring = ring + 3.0 * (torch.rand(ring.shape, generator=gen) - 0.5)
    ring2 = scenes.circle_rings(torch.tensor([[30.0, 20.0]]), torch.tensor([12.0]),
                                torch.tensor([0.0]), g)
    cn = torch.cat([scenes.px_to_norm(scenes.ring_to_cubics(ring), 80, 64),
                    scenes.px_to_norm(scenes.ring_to_cubics(ring2), 80, 64)]).numpy()
    offs = np.array([0, g, 2 * g], np.int32)
    args = (cn, offs, np.array([[0.9, 0.2, 0.1], [0.1, 0.3, 0.8]], np.float32),
            np.array([0.8, 0.6], np.float32), np.array([0.3, 0.7], np.float32), 64, 80,
            np.array([1.0, 1.0, 1.0], np.float32), np.array([1, 0], np.int32),
            np.array([1.3, 0.8], np.float32), 24)
    st = oracle.render_fill(*args[:8], fill_rules=args[8], aa_widths=args[9], samples=args[10])
    b, inv, out, fts, fidx = gpu_fill(*args)
    np.testing.assert_array_equal(_np(fidx), st["final_idx"])
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6
    v_out = scenes.seeded_grad(3, 64, 80).numpy()
    want = oracle.fill_backward(st, v_out, True, True)
    got = gpu_fill_backward(b, args[2], args[3], inv, args[8], args[7], fts, fidx, v_out, 64, 80)
    for k in ["v_colors", "v_opacities", "v_inv_sigma2s", "v_cubics_px"]:
        assert_grad_close(got[k], want[k], k)


@pytest.mark.parametrize("paths", [40, 300, 5000])
def test_many_primitives_in_one_tile_sort_paths(paths):
    # all primitives overlap the same few tiles: exercises the warp, shared-memory
    # and large-tile sort paths, including equal depths
    gen = torch.Generator().manual_seed(paths)
    centres = 16.0 + 4.0 * torch.rand(paths, 2, generator=gen)
    radii = 2.0 + 6.0 * torch.rand(paths, generator=gen)
    ring = scenes.circle_rings(centres, radii, torch.zeros(paths), 4)
    cn = scenes.px_to_norm(scenes.ring_to_cubics(ring), 40, 40).numpy()
    offs = np.arange(0, 4 * paths + 1, 4, dtype=np.int32)
    depths = torch.rand(paths, generator=gen).numpy()
    depths[::7] = 0.5
    col = torch.rand(paths, 3, generator=gen).numpy()
    op = (0.05 + 0.2 * torch.rand(paths, generator=gen)).numpy()
    args = (cn, offs, col, op, depths, 40, 40, np.ones(3, np.float32),
            np.ones(paths, np.int32), np.ones(paths, np.float32), 6)
    st = oracle.render_fill(*args[:8], fill_rules=args[8], aa_widths=args[9], samples=args[10])
    b, inv, out, fts, fidx = gpu_fill(*args)
    check_binning(b, st)
    np.testing.assert_array_equal(_np(fidx), st["final_idx"])
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6


def test_tile_row_bands_stitch_to_full_image():
    sc = scenes.config1()
    args = fill_inputs(sc)
    h, w = args[5], args[6]
    _, _, full, full_ts, full_idx = gpu_fill(*args)
    tby = (h + 15) // 16
    cuts = [0, 3, 9, 10, tby]
    stitched = torch.zeros_like(full)
    for r0, r1 in zip(cuts[:-1], cuts[1:]):
        _, _, out, _, _ = gpu_fill(*args, tile_rows=(r0, r1))
        stitched[r0 * 16:min(h, r1 * 16)] = out[r0 * 16:min(h, r1 * 16)]
    assert torch.equal(stitched, full)


@pytest.mark.parametrize("rows", [None, (2, 9)])
def test_unit_lists_bucket_every_strip_by_work_and_change_no_result(rows):
    """The staging pass files the band's strips (4 per tile) into 64 buckets of
    staged work, heaviest first; the lists only schedule the raster warps, so
    results match the launch without them."""
    sc = scenes.config1()
    args = fill_inputs(sc)
    h, w = args[5], args[6]
    b, inv, out, fts, fidx = gpu_fill(*args, tile_rows=rows)
    tbx = (w + 15) // 16
    r0, r1 = b.tile_rows
    nunits = 4 * (r1 - r0) * tbx
    lists = _np(b.unit_order)
    counts = lists[:64]
    assert counts.sum() == nunits
    # work estimate of every strip: 2 per staged record + 5 per intersect of its tile
    bins = _np(b.tile_bins)[r0 * tbx:r1 * tbx]
    strips = _np(b.isect_strips)
    est = np.zeros(nunits, np.int64)
    for t in range(len(bins)):
        rs, re = bins[t]
        if re > rs:
            for st in range(4):
                est[4 * t + st] = 2 * int(strips[re - 1, st].sum()) + 5 * (re - rs)

    def bucket(v):  # two buckets per octave, heaviest first, no work last
        if v <= 0:
            return 63
        msb = int(v).bit_length() - 1
        half = (v >> (msb - 1)) & 1 if msb >= 1 else 0
        return 62 - min(2 * msb + half, 62)
    seen = []
    for bk in range(64):
        members = lists[64 + bk * nunits: 64 + bk * nunits + counts[bk]]
        assert all(bucket(est[u]) == bk for u in members), bk
        seen.extend(members.tolist())
    assert sorted(seen) == list(range(nunits))
    # the forward files every strip once more, by its measured work, for the backward
    bl = _np(b.unit_order_bwd)
    assert bl[:64].sum() == nunits
    seen_b = np.concatenate([bl[64 + bk * nunits: 64 + bk * nunits + bl[bk]] for bk in range(64)])
    assert sorted(seen_b.tolist()) == list(range(nunits))
    plain = render.replace_binning(b, unit_order=None, unit_order_bwd=None)
    out2, fts2, fidx2 = render.forward_raster(plain, _t(args[7], torch.float32), h, w)
    band = slice(r0 * 16, min(h, r1 * 16))  # rows outside the band are not written
    assert torch.equal(out[band], out2[band]) and torch.equal(fts[band], fts2[band])
    assert torch.equal(fidx[band], fidx2[band])
    v_out = np.asarray(scenes.seeded_grad(5, h, w), np.float32)
    g1 = gpu_fill_backward(b, args[2], args[3], inv, args[8], args[7], fts, fidx, v_out, h, w)
    g2 = gpu_fill_backward(plain, args[2], args[3], inv, args[8], args[7], fts, fidx, v_out, h, w)
    for k in g1:
        assert_grad_close(g1[k], g2[k], k)


def _stroke_binning(keep=300, h=256, w=256):
    """Config-4 strokes over a 256x256 corner, binned and rendered forward."""
    sc = scenes.config4()
    cn = _t(sc.cubics_norm()[:keep])
    offs = _t(np.arange(keep + 1, dtype=np.int32))
    aa = torch.clamp(_t(sc.aa_widths[:keep]), min=1e-4)
    col, op = _t(sc.colors[:keep]), _t(sc.opacities[:keep])
    b = render.bin_primitives(cn, offs, _t(sc.depths[:keep]), aa, h, w, sc.samples, colors=col,
                              opacities=op, inv_sigma2s=render._inv_sigma2(aa),
                              stroke_widths=_t(sc.stroke_widths[:keep]))
    bg = _t(sc.background)
    out, fts, fidx = render.forward_raster(b, bg, h, w)
    return b, bg, keep, out, fts, fidx


def _check_visit_lists(b, fidx, h, w):
    """Each strip's list: ascending ids inside its tile's [rs, re), ending at
    the strip's largest final_idx (the last intersect any of its pixels
    composited)."""
    tbx = (w + 15) // 16
    r0, r1 = b.tile_rows
    bins = _np(b.tile_bins)
    vl = _np(b.visit_lists)
    fi = _np(fidx)
    listed = 0
    for ty in range(r0, r1):
        for tx in range(tbx):
            t = ty * tbx + tx
            rs, re = (int(v) for v in bins[t])
            if re <= rs:  # no intersects, no list
                continue
            for st in range(4):
                base = 4 * (rs + t) + st * (re - rs + 1)
                n = int(vl[base])
                assert 0 <= n <= re - rs
                ids = vl[base + 1: base + 1 + n]
                assert np.all(np.diff(ids) > 0) and np.all((ids >= rs) & (ids < re))
                rows = slice(ty * 16 + 4 * st, min(h, ty * 16 + 4 * st + 4))
                cols = slice(tx * 16, min(w, tx * 16 + 16))
                if n:
                    assert ids[-1] == fi[rows, cols].max()
                listed += n
    return listed


@pytest.mark.parametrize("stroke", [False, True])
def test_visit_lists_walk_only_composited_intersects(stroke):
    """The forward lists, per strip, the intersects that composited a pixel of
    it; the backward walks only those and its gradients match the walk over
    every intersect up to final_idx."""
    if stroke:
        b, bg, p, out, fts, fidx = _stroke_binning()
        h = w = 256
    else:
        args = fill_inputs(scenes.config1())
        h, w = args[5], args[6]
        b, inv, out, fts, fidx = gpu_fill(*args)
        bg, p = _t(args[7], torch.float32), int(np.asarray(args[2]).shape[0])
    assert _check_visit_lists(b, fidx, h, w) > 0
    v_out = _t(np.asarray(scenes.seeded_grad(9, h, w), np.float32))
    plain = render.replace_binning(b, visit_lists=None)
    g1 = render.raster_backward(b, p, bg, fts, fidx, v_out, h, w, collect_contrib=True,
                                collect_isect_contrib=True)
    g2 = render.raster_backward(plain, p, bg, fts, fidx, v_out, h, w, collect_contrib=True,
                                collect_isect_contrib=True)
    assert int(b.counters[1]) == 0
    for name, a, c in zip(["v_edges", "v_colors", "v_opac", "v_inv", "v_sw", "contrib",
                           "icontrib"], g1, g2):
        if a is not None:
            assert_grad_close(_np(a), _np(c), name)


def test_fill_winner_codes_fall_back_and_reject_bad_codes():
    """The forward's closest-record codes (fills): the backward that
    evaluates only each pixel's stored winner gives the gradients of the one
    that walks every record; a code past its intersect's records sets
    CS_ERR_ARG and is ignored (every read stays inside the strip's records)."""
    from repo_b200 import _native as nat
    args = fill_inputs(scenes.config1())
    h, w = args[5], args[6]
    b, inv, out, fts, fidx = gpu_fill(*args)
    assert b.visit_winners is not None
    bg, p = _t(args[7], torch.float32), int(np.asarray(args[2]).shape[0])
    v_out = _t(np.asarray(scenes.seeded_grad(11, h, w), np.float32))
    g1 = render.raster_backward(b, p, bg, fts, fidx, v_out, h, w)
    good = b.visit_winners.clone()
    g2 = render.raster_backward(render.replace_binning(b, visit_winners=None), p, bg, fts, fidx,
                                v_out, h, w)
    assert int(b.counters[1]) == 0
    for name, a, c in zip(["v_edges", "v_colors", "v_opac", "v_inv"], g1, g2):
        assert_grad_close(_np(a), _np(c), name)
    b.visit_winners.fill_(0x7E7E)  # record 126 of intersects with fewer records
    render.raster_backward(b, p, bg, fts, fidx, v_out, h, w)
    assert int(b.counters[1]) == nat.CS_ERR_ARG
    b.counters[1] = 0
    b.visit_winners.copy_(good)


def test_visit_lists_that_do_not_fit_the_bins_set_an_error():
    """A visit list not written by this frame's forward (counts past the
    tile's intersects, ids outside it) is rejected strip by strip with
    CS_ERR_ARG in the status word; every read stays inside the list buffer."""
    from repo_b200 import _native as nat
    b, bg, p, out, fts, fidx = _stroke_binning()
    v_out = _t(np.asarray(scenes.seeded_grad(9, 256, 256), np.float32))
    good = b.visit_lists.clone()
    for fill in (1 << 30, -7):
        b.visit_lists.fill_(fill)
        b.counters[1] = 0
        render.raster_backward(b, p, bg, fts, fidx, v_out, 256, 256)
        assert int(b.counters[1]) == nat.CS_ERR_ARG
    # counts that fit, ids that do not
    bins = _np(b.tile_bins)
    bases = [4 * (int(rs) + t) + st * (int(re) - int(rs) + 1)
             for t, (rs, re) in enumerate(bins) if re > rs for st in range(4)]
    host = _np(good).copy()
    keep = np.zeros(host.shape, bool)
    keep[bases] = True
    assert (host[bases] > 0).any()
    host[~keep] = -1
    b.visit_lists.copy_(torch.from_numpy(host))
    b.counters[1] = 0
    render.raster_backward(b, p, bg, fts, fidx, v_out, 256, 256)
    assert int(b.counters[1]) == nat.CS_ERR_ARG
    b.visit_lists.copy_(good)
    b.counters[1] = 0
    g = render.raster_backward(b, p, bg, fts, fidx, v_out, 256, 256)
    assert int(b.counters[1]) == 0 and torch.isfinite(g[0]).all()


def test_image_size_not_multiple_of_tile():
    sc = scenes.small_fill_scene(77, h=45, w=61, paths=7)
    args = fill_inputs(sc)
    st = oracle.render_fill(*args[:8], fill_rules=args[8], aa_widths=args[9], samples=args[10])
    b, inv, out, fts, fidx = gpu_fill(*args)
    np.testing.assert_array_equal(_np(fidx), st["final_idx"])
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6


def test_process_fn_hooks_are_called_and_honoured():
    import manbo
    sc = scenes.small_fill_scene(8)
    stages = []

    def hook(stage, payload):
        stages.append(stage)
        if stage == "pre_backward_rasterize":
            return {"collect_curve_contrib_rgb": True, "collect_curve_isect_contrib": True}
        if stage == "post_backward_rasterize":
            assert payload["curve_contrib_rgb"] is not None
            return {"v_colors": torch.zeros_like(payload["v_colors"])}
        return None

    col = _t(sc.colors).requires_grad_(True)
    out = manbo.ops.render_cubic_fill_splat_tilelang(
        _t(sc.cubics_norm()), _t(sc.seg_offsets()), col, _t(sc.opacities), _t(sc.depths),
        sc.height, sc.width, 16, 16, _t(sc.background), process_fn=hook)
    out.sum().backward()
    assert stages == ["pre_backward_rasterize", "post_backward_rasterize"]
    assert float(col.grad.abs().sum()) == 0.0
