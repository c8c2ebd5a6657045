"""Adaptive de Casteljau flattening on the GPU (flatten_method="de_casteljau"):
the flatten kernels against the reference's own flatten (golden vectors from
its host branch), and the whole fill / stroke renderer on that flattening
against the CPU oracle and the reference's GPU renderer.

Tolerances as in test_gpu_parity: flatten outputs bit for bit, images within
1e-6 of the oracle (1e-4 of the reference), gradients within 1e-3 relative L2.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN, load_golden, rel_l2
from repo_b200 import _native as nat
from repo_b200 import render, scenes

pytestmark = pytest.mark.gpu

DEV = "cuda"
GRAD_REL = 1e-3


def _t(a, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a))
    return (t.to(dtype) if dtype is not None else t).to(DEV)


def _np(t):
    return t.detach().cpu().numpy()


def _grad_close(got, want, name):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    r = rel_l2(got, want)
    assert r <= GRAD_REL, f"{name}: rel L2 {r:.3e}"


@pytest.mark.parametrize("samples", [5, 16, 24, 33])
def test_flatten_matches_reference_golden(samples):
    g = load_golden("dc_flatten")
    status = torch.zeros((1,), dtype=torch.int32, device=DEV)
    edges, peo, seg, t0, t1 = render.flatten_de_casteljau(_t(g["cubics_px"]), _t(g["offs"]),
                                                          samples, status)
    assert int(status.item()) == 0
    n = int(seg[-1].item())
    np.testing.assert_array_equal(_np(seg), g[f"s{samples}_segment_edge_offsets"])
    np.testing.assert_array_equal(_np(peo), g[f"s{samples}_prim_edge_offsets"])
    np.testing.assert_array_equal(_np(edges[:n]), g[f"s{samples}_edges_px"])
    np.testing.assert_array_equal(_np(t0[:n]), g[f"s{samples}_edge_t_starts"])
    np.testing.assert_array_equal(_np(t1[:n]), g[f"s{samples}_edge_t_ends"])
    assert n <= int(nat.call("cs_de_casteljau_edge_capacity", len(g["cubics_px"]), samples))


def test_flatness_flags_and_split_match_reference_golden():
    from manbo.ops import cubic_splatting as cs
    g = load_golden("dc_flatten")
    cub = _t(g["cubics_px"])
    np.testing.assert_array_equal(_np(cs.cubic_adaptive_flatness_flags_tilelang(cub, tol_px=0.5)),
                                  g["flat_tol0.5"])
    np.testing.assert_array_equal(_np(cs.cubic_adaptive_flatness_flags_tilelang(cub, tol_px=3.0)),
                                  g["flat_tol3"])
    assert _np(cs.cubic_adaptive_flatness_flags_tilelang(cub, tol_px=0.5, force_flat=True)).all()
    left, right = cs.cubic_split_half_tilelang(cub)
    np.testing.assert_array_equal(_np(left), g["split_left"])
    np.testing.assert_array_equal(_np(right), g["split_right"])


def test_stage_wrappers_flatten_and_csr_grads_match_oracle():
    from manbo.ops import cubic_splatting as cs
    g = load_golden("dc_flatten")
    edges, peo, seg, t0, t1 = cs._flatten_cubics_to_edges(
        _t(g["cubics_px"]), _t(g["offs"]), distance_samples=16, flatten_method="de_casteljau")
    np.testing.assert_array_equal(_np(edges), g["s16_edges_px"])
    np.testing.assert_array_equal(_np(peo), g["s16_prim_edge_offsets"])
    rng = np.random.default_rng(5)
    v = rng.standard_normal((int(edges.shape[0]), 2, 2)).astype(np.float32)
    got = cs._accumulate_edge_grads_to_cubics(
        _t(v), len(g["cubics_px"]), distance_samples=16, flatten_method="de_casteljau",
        segment_edge_offsets=seg, edge_t_starts=t0, edge_t_ends=t1)
    want = oracle.edge_grads_csr(v, g["s16_segment_edge_offsets"], g["s16_edge_t_starts"],
                                 g["s16_edge_t_ends"])
    np.testing.assert_array_equal(_np(got), want)
    with pytest.raises(ValueError):
        cs._accumulate_edge_grads_to_cubics(_t(v), len(g["cubics_px"]), distance_samples=16,
                                            flatten_method="de_casteljau")


def _fill_api(sc, v_out):
    import manbo
    cn = _t(sc.cubics_norm()).requires_grad_(True)
    col = _t(sc.colors).requires_grad_(True)
    op = _t(sc.opacities).requires_grad_(True)
    aw = _t(sc.aa_widths).requires_grad_(True)
    out = manbo.ops.render_cubic_fill_splat_tilelang(
        cn, _t(sc.seg_offsets()), col, op, _t(sc.depths), sc.height, sc.width, 16, 16,
        _t(sc.background), fill_rules=_t(sc.fill_rules), aa_widths=aw,
        distance_samples=sc.samples, flatten_method="de_casteljau")
    (out * _t(v_out)).sum().backward()
    return out, cn.grad, col.grad, op.grad, aw.grad


@pytest.mark.parametrize("seed", [111, 112])
def test_fill_de_casteljau_matches_oracle(seed):
    sc = scenes.small_fill_scene(seed, paths=9)
    h, w = sc.height, sc.width
    st = oracle.render_fill(sc.cubics_norm().numpy(), sc.seg_offsets().numpy(), sc.colors.numpy(),
                            sc.opacities.numpy(), sc.depths.numpy(), h, w,
                            sc.background.numpy(), fill_rules=sc.fill_rules.numpy(),
                            aa_widths=sc.aa_widths.numpy(), samples=sc.samples,
                            flatten_method="de_casteljau")
    v_out = scenes.seeded_grad(seed, h, w).numpy()
    want = oracle.fill_backward(st, v_out)
    out, v_cn, v_col, v_op, v_aw = _fill_api(sc, v_out)
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6
    _grad_close(_np(v_cn), want["v_cubics_norm"], "v_cubics_norm")
    _grad_close(_np(v_col), want["v_colors"], "v_colors")
    _grad_close(_np(v_op), want["v_opacities"], "v_opacities")
    _grad_close(_np(v_aw), want["v_aa_widths"], "v_aa_widths")
    # the adaptive flatten really differs from the uniform one here
    ref_b = oracle.render_fill(sc.cubics_norm().numpy(), sc.seg_offsets().numpy(),
                               sc.colors.numpy(), sc.opacities.numpy(), sc.depths.numpy(), h, w,
                               sc.background.numpy(), fill_rules=sc.fill_rules.numpy(),
                               aa_widths=sc.aa_widths.numpy(), samples=sc.samples)
    assert st["edges_px"].shape != ref_b["edges_px"].shape or \
        not np.array_equal(st["edges_px"], ref_b["edges_px"])


def test_stroke_de_casteljau_matches_oracle():
    import manbo
    sc = scenes.small_stroke_scene(113)
    h, w = sc.height, sc.width
    st = oracle.render_stroke(sc.cubics_norm().numpy(), sc.seg_offsets().numpy(),
                              sc.colors.numpy(), sc.opacities.numpy(), sc.stroke_widths.numpy(),
                              sc.depths.numpy(), h, w, sc.background.numpy(),
                              aa_widths=sc.aa_widths.numpy(), samples=sc.samples,
                              flatten_method="de_casteljau")
    v_out = scenes.seeded_grad(114, h, w).numpy()
    want = oracle.stroke_backward(st, v_out)
    cn = _t(sc.cubics_norm()).requires_grad_(True)
    sw = _t(sc.stroke_widths).requires_grad_(True)
    col = _t(sc.colors).requires_grad_(True)
    out = manbo.ops.render_cubic_polyline_splat_tilelang(
        cn, _t(sc.seg_offsets()), col, _t(sc.opacities), sw, _t(sc.depths), h, w, 16, 16,
        _t(sc.background), aa_widths=_t(sc.aa_widths), distance_samples=sc.samples,
        flatten_method="de_casteljau")
    assert np.abs(_np(out) - st["image"]).max() <= 1e-6
    (out * _t(v_out)).sum().backward()
    _grad_close(_np(cn.grad), want["v_cubics_norm"], "v_cubics_norm")
    _grad_close(_np(sw.grad), want["v_stroke_widths"], "v_stroke_widths")
    _grad_close(_np(col.grad), want["v_colors"], "v_colors")


@pytest.mark.parametrize("case", ["dc_fill", "dc_stroke"])
def test_de_casteljau_api_matches_reference_golden(case):
    """Image and gradients of the public entry points with de Casteljau
    flattening against the reference's GPU renderer (make_golden.py)."""
    if not os.path.exists(os.path.join(GOLDEN, f"{case}.npz")):
        pytest.fail(f"missing fixture {case}.npz (tests/golden/make_golden.py --cases {case})")
    import manbo
    g = load_golden(case)
    h, w, s = (int(v) for v in g["hw_s"])
    cn = _t(g["cubics_norm"]).requires_grad_(True)
    col = _t(g["colors"]).requires_grad_(True)
    op = _t(g["opacities"]).requires_grad_(True)
    aw = _t(g["aa_widths"]).requires_grad_(True)
    kw = dict(aa_widths=aw, distance_samples=s, flatten_method="de_casteljau")
    if case == "dc_stroke":
        sw = _t(g["stroke_widths"]).requires_grad_(True)
        out = manbo.ops.render_cubic_polyline_splat_tilelang(
            cn, _t(g["offs"]), col, op, sw, _t(g["depths"]), h, w, 16, 16,
            _t(g["background"]), **kw)
    else:
        out = manbo.ops.render_cubic_fill_splat_tilelang(
            cn, _t(g["offs"]), col, op, _t(g["depths"]), h, w, 16, 16, _t(g["background"]),
            fill_rules=_t(g["fill_rules"]), **kw)
    assert np.abs(_np(out) - g["api_image"]).max() <= 1e-4
    (out * _t(g["v_output"])).sum().backward()
    _grad_close(_np(cn.grad), g["api_v_cubics_norm"], "v_cubics_norm")
    _grad_close(_np(col.grad), g["api_v_colors"], "v_colors")
    _grad_close(_np(op.grad), g["api_v_opacities"], "v_opacities")
    _grad_close(_np(aw.grad), g["api_v_aa_widths"], "v_aa_widths")
    if case == "dc_stroke":
        _grad_close(_np(sw.grad), g["api_v_stroke_widths"], "v_stroke_widths")
