"""Generate golden vectors by running the reference renderer itself.

This script imports the *reference* ``manbo`` package (TileLang kernels) from
an installed copy (default ``baseline/_ref``, made with ``pip install --target``
from the reference checkout) and runs it on a CUDA GPU on seeded inputs from
``repo_b200.scenes``.  Every stage output of the cubic fill / stroke pipelines,
the ring-segment conversion and the metric kernels is saved as a compressed
``.npz`` next to this file.  The fixtures pin the CPU oracle (``oracle/``) and
the CUDA path to the reference's own outputs; they are committed so that the
tests never need the reference or TileLang at run time.

It can also time the reference's training step on the 768x512 / 512-path
configuration (``--time``), which is the GPU baseline of the benchmark.

Usage (on a machine with a GPU and TileLang)::

    python tests/golden/make_golden.py --ref baseline/_ref --out tests/golden
    python tests/golden/make_golden.py --ref baseline/_ref --time --json out.json
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from repo_b200 import scenes  # noqa: E402


def _np(t):
    if t is None:
        return None
    return t.detach().cpu().contiguous().numpy()


def _save(out_dir, name, arrays):
    arrays = {k: v for k, v in arrays.items() if v is not None}
    path = os.path.join(out_dir, f"{name}.npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path}: {len(arrays)} arrays", flush=True)


def fill_case(cs, tb, scene, grad_seed, dev):
    """Run every stage of the reference fill pipeline on ``scene``."""
    h, w, s = scene.height, scene.width, scene.samples
    cubics_norm = scene.cubics_norm().to(dev)
    offs = scene.seg_offsets().to(dev)
    colors = scene.colors.to(dev)
    opac = scene.opacities.to(dev)
    depths = scene.depths.to(dev)
    rules = scene.fill_rules.to(dev)
    aa = scene.aa_widths.to(dev)
    bg = scene.background.to(dev)
    bx = by = 16
    tile_bounds = ((w + bx - 1) // bx, (h + by - 1) // by, 1)
    g = int(cubics_norm.shape[0])

    widths = torch.clamp(aa, min=1e-4)
    inv_s2 = (1.0 / torch.clamp(widths * widths, min=1e-6)).contiguous()
    seg_counts = (offs[1:] - offs[:-1]).to(torch.int64)
    support_seg = torch.repeat_interleave(widths * 3.0, seg_counts).contiguous()
    stroke_zeros = torch.zeros((g,), dtype=torch.float32, device=dev)
    cubics_px, seg_ranges, seg_hits = cs.project_cubics_2d_forward_tilelang(
        cubics_norm, stroke_zeros, support_seg, h, w, tile_bounds)
    edges_px, prim_edge_offs, _, _, _ = cs._flatten_cubics_to_edges(
        cubics_px, offs, distance_samples=s)
    prim_ranges, num_hit = cs._primitive_tile_ranges_from_segment_tile_ranges(
        seg_ranges, offs, tile_bounds)
    cum = torch.cumsum(num_hit, dim=0, dtype=torch.int32)
    isect_ids, prim_ids = cs.map_cubic_to_intersects_tilelang(prim_ranges, depths, cum, tile_bounds)
    isect_sorted, order = torch.sort(isect_ids)
    prim_sorted = torch.gather(prim_ids, 0, order)
    ranges = cs._build_fill_isect_edge_ranges(prim_sorted, prim_edge_offs, num_edges=int(edges_px.shape[0]))
    tile_bins = tb.get_tile_bin_edges_tilelang(int(cum[-1].item()), isect_sorted,
                                               num_tiles=tile_bounds[0] * tile_bounds[1], compact=True)
    img, final_ts, final_idx = cs.rasterize_cubic_fill_forward_tilelang(
        tile_bounds, (bx, by, 1), (w, h, 1), prim_sorted, tile_bins, cubics_px, offs,
        colors, opac, rules, bg, inv_sigma2s=inv_s2, edges_px=edges_px,
        isect_edge_ranges=ranges, distance_samples=s)

    v_out = scenes.seeded_grad(grad_seed, h, w).to(dev)
    v_edges = torch.zeros_like(edges_px)
    v_colors = torch.zeros_like(colors)
    v_opac = torch.zeros_like(opac)
    v_inv = torch.zeros_like(opac)
    contrib = torch.zeros_like(colors)
    isect_contrib = torch.zeros((int(prim_sorted.numel()),), dtype=torch.float32, device=dev)
    kern = cs.rasterize_cubic_fill_backward_kernel(block_x=bx, block_y=by, dtype="float32")
    kern(prim_sorted, tile_bins, edges_px, ranges, colors, opac, inv_s2, rules, bg,
         final_ts, final_idx, v_out, v_edges, v_colors, v_opac, v_inv, 1, contrib, 1, isect_contrib)
    v_cubics_px = cs._accumulate_edge_grads_to_cubics(v_edges, g, distance_samples=s)

    # end-to-end autograd through the public entry point
    cn = cubics_norm.clone().requires_grad_(True)
    col = colors.clone().requires_grad_(True)
    op = opac.clone().requires_grad_(True)
    aw = aa.clone().requires_grad_(True)
    out = cs.render_cubic_fill_splat_tilelang(cn, offs, col, op, depths, h, w, bx, by, bg,
                                              fill_rules=rules, aa_widths=aw, distance_samples=s)
    (out * v_out).sum().backward()

    return {
        "cubics_norm": _np(cubics_norm), "offs": _np(offs), "colors": _np(colors),
        "opacities": _np(opac), "depths": _np(depths), "fill_rules": _np(rules),
        "aa_widths": _np(aa), "background": _np(bg), "hw_s": np.array([h, w, s], np.int32),
        "cubics_px": _np(cubics_px), "seg_tile_ranges": _np(seg_ranges),
        "seg_num_tiles": _np(seg_hits), "edges_px": _np(edges_px),
        "prim_edge_offsets": _np(prim_edge_offs), "prim_tile_ranges": _np(prim_ranges),
        "num_tiles_hit": _np(num_hit), "isect_ids": _np(isect_ids), "prim_ids": _np(prim_ids),
        "isect_ids_sorted": _np(isect_sorted), "prim_ids_sorted": _np(prim_sorted),
        "isect_edge_ranges": _np(ranges), "tile_bins": _np(tile_bins),
        "image": _np(img), "final_Ts": _np(final_ts), "final_idx": _np(final_idx),
        "v_output": _np(v_out), "v_edges": _np(v_edges), "v_colors": _np(v_colors),
        "v_opacities": _np(v_opac), "v_inv_sigma2s": _np(v_inv),
        "curve_contrib_rgb": _np(contrib), "curve_isect_contrib": _np(isect_contrib),
        "v_cubics_px": _np(v_cubics_px),
        "api_image": _np(out), "api_v_cubics_norm": _np(cn.grad), "api_v_colors": _np(col.grad),
        "api_v_opacities": _np(op.grad), "api_v_aa_widths": _np(aw.grad),
    }


def stroke_case(cs, ps, tb, scene, grad_seed, dev):
    h, w, s = scene.height, scene.width, scene.samples
    cubics_norm = scene.cubics_norm().to(dev)
    offs = scene.seg_offsets().to(dev)
    colors = scene.colors.to(dev)
    opac = scene.opacities.to(dev)
    sw = scene.stroke_widths.to(dev)
    depths = scene.depths.to(dev)
    aa = scene.aa_widths.to(dev)
    bg = scene.background.to(dev)
    bx = by = 16
    tile_bounds = ((w + bx - 1) // bx, (h + by - 1) // by, 1)
    g = int(cubics_norm.shape[0])
    widths = torch.clamp(aa, min=1e-4)
    inv_s2 = (1.0 / torch.clamp(widths * widths, min=1e-6)).contiguous()
    seg_counts = (offs[1:] - offs[:-1]).to(torch.int64)
    support_seg = torch.repeat_interleave(widths * 3.0, seg_counts).contiguous()
    stroke_seg = torch.repeat_interleave(sw, seg_counts).contiguous()
    cubics_px, seg_ranges, seg_hits = cs.project_cubics_2d_forward_tilelang(
        cubics_norm, stroke_seg, support_seg, h, w, tile_bounds)
    edges_px, prim_edge_offs, _, _, _ = cs._flatten_cubics_to_edges(cubics_px, offs, distance_samples=s)
    prim_ranges, num_hit = cs._primitive_tile_ranges_from_segment_tile_ranges(seg_ranges, offs, tile_bounds)
    cum = torch.cumsum(num_hit, dim=0, dtype=torch.int32)
    isect_ids, prim_ids = cs.map_cubic_to_intersects_tilelang(prim_ranges, depths, cum, tile_bounds)
    isect_sorted, order = torch.sort(isect_ids)
    prim_sorted = torch.gather(prim_ids, 0, order)
    ranges = cs._build_fill_isect_edge_ranges(prim_sorted, prim_edge_offs, num_edges=int(edges_px.shape[0]))
    tile_bins = tb.get_tile_bin_edges_tilelang(int(cum[-1].item()), isect_sorted,
                                               num_tiles=tile_bounds[0] * tile_bounds[1], compact=True)
    img, final_ts, final_idx = ps.rasterize_cubic_polyline_forward_tilelang(
        tile_bounds, (bx, by, 1), (w, h, 1), prim_sorted, tile_bins, colors, opac, sw, bg,
        inv_sigma2s=inv_s2, edges_px=edges_px, isect_edge_ranges=ranges)
    v_out = scenes.seeded_grad(grad_seed, h, w).to(dev)
    v_edges = torch.zeros_like(edges_px)
    v_colors = torch.zeros_like(colors)
    v_opac = torch.zeros_like(opac)
    v_sw = torch.zeros_like(sw)
    v_inv = torch.zeros_like(opac)
    contrib = torch.zeros_like(colors)
    isect_contrib = torch.zeros((int(prim_sorted.numel()),), dtype=torch.float32, device=dev)
    kern = ps.rasterize_cubic_polyline_backward_kernel(block_x=bx, block_y=by, dtype="float32")
    kern(prim_sorted, tile_bins, edges_px, ranges, colors, opac, sw, inv_s2, bg, final_ts,
         final_idx, v_out, v_edges, v_colors, v_opac, v_sw, v_inv, 1, contrib, 1, isect_contrib)
    v_cubics_px = cs._accumulate_edge_grads_to_cubics(v_edges, g, distance_samples=s)

    cn = cubics_norm.clone().requires_grad_(True)
    col = colors.clone().requires_grad_(True)
    op = opac.clone().requires_grad_(True)
    swr = sw.clone().requires_grad_(True)
    aw = aa.clone().requires_grad_(True)
    out = ps.render_cubic_polyline_splat_tilelang(cn, offs, col, op, swr, depths, h, w, bx, by, bg,
                                                  aa_widths=aw, distance_samples=s)
    (out * v_out).sum().backward()
    return {
        "cubics_norm": _np(cubics_norm), "offs": _np(offs), "colors": _np(colors),
        "opacities": _np(opac), "stroke_widths": _np(sw), "depths": _np(depths),
        "aa_widths": _np(aa), "background": _np(bg), "hw_s": np.array([h, w, s], np.int32),
        "cubics_px": _np(cubics_px), "seg_tile_ranges": _np(seg_ranges),
        "edges_px": _np(edges_px), "prim_tile_ranges": _np(prim_ranges),
        "isect_ids_sorted": _np(isect_sorted), "prim_ids_sorted": _np(prim_sorted),
        "tile_bins": _np(tile_bins), "image": _np(img), "final_Ts": _np(final_ts),
        "final_idx": _np(final_idx), "v_output": _np(v_out), "v_edges": _np(v_edges),
        "v_colors": _np(v_colors), "v_opacities": _np(v_opac), "v_stroke_widths": _np(v_sw),
        "v_inv_sigma2s": _np(v_inv), "curve_contrib_rgb": _np(contrib),
        "curve_isect_contrib": _np(isect_contrib), "v_cubics_px": _np(v_cubics_px),
        "api_image": _np(out), "api_v_cubics_norm": _np(cn.grad), "api_v_colors": _np(col.grad),
        "api_v_opacities": _np(op.grad), "api_v_stroke_widths": _np(swr.grad),
        "api_v_aa_widths": _np(aw.grad),
    }


def ring_case(cs, dev):
    gen = torch.Generator().manual_seed(7)
    cp = (torch.rand(5, 10, 2, generator=gen) * 2.0 - 1.0).to(dev)
    cpg = cp.clone().requires_grad_(True)
    segs, offs = cs.closed_cubic_fill_segments_tilelang(cpg, subdiv=4)
    gs = (torch.rand(segs.shape, generator=gen) - 0.5).to(dev)
    (segs * gs).sum().backward()
    return {"control_points": _np(cp), "segments": _np(segs), "offsets": _np(offs),
            "grad_segments": _np(gs), "grad_control_points": _np(cpg.grad)}


def metric_case(metric, dev):
    gen = torch.Generator().manual_seed(11)
    x = torch.rand(2, 3, 40, 52, generator=gen).to(dev)
    y = torch.clamp(x + 0.1 * (torch.rand(x.shape, generator=gen) - 0.5).to(dev), 0, 1)
    xg = x.clone().requires_grad_(True)
    loss = metric.mse_loss_tilelang(xg, y)
    loss.backward()
    return {
        "x": _np(x), "y": _np(y), "mse": _np(loss.detach()), "mse_grad": _np(xg.grad),
        "psnr": _np(metric.psnr(x, y)), "ssim": _np(metric.ssim(x, y)),
        "ssim_per_image": _np(metric.ssim(x, y, size_average=False)),
    }


ADAN_VARIANTS = {
    "prox": dict(lr=0.05, weight_decay=0.02),
    "noprox": dict(lr=0.05, weight_decay=0.02, no_prox=True),
    "clip": dict(lr=0.05, max_grad_norm=0.5),
}


def adan_case(manbo, dev):
    """Three steps of the reference Adan optimiser in three variants, on one
    odd-length and one 4-aligned parameter with seeded gradients."""
    gen = torch.Generator().manual_seed(13)
    shapes = [(37, 2), (64,)]
    params0 = [torch.randn(s, generator=gen) for s in shapes]
    grads = [[torch.randn(s, generator=gen) * 0.1 for s in shapes] for _ in range(3)]
    out = {f"param0_{i}": _np(p) for i, p in enumerate(params0)}
    for t in range(3):
        for i, g in enumerate(grads[t]):
            out[f"grad{t}_{i}"] = _np(g)
    for name, kw in ADAN_VARIANTS.items():
        ps = [p.clone().to(dev).requires_grad_(True) for p in params0]
        opt = manbo.Adan(ps, **kw)
        for t in range(3):
            for p, g in zip(ps, grads[t]):
                p.grad = g.to(dev).clone()
            opt.step()
        for i, p in enumerate(ps):
            out[f"{name}_param_{i}"] = _np(p)
            for k in ("exp_avg", "exp_avg_sq", "exp_avg_diff", "neg_pre_grad"):
                out[f"{name}_{k}_{i}"] = _np(opt.state[p][k])
    return out


REG_KW = dict(num_beziers=2, bezier_degree=4, num_samples=3, lambda_proj=0.7,
              opacity_weight=0.3, boundary_bound=1.0, curvature_angle_thresh_deg=60.0)


def reg_case(manbo, dev):
    """The reference's regularisation loss and its gradients (autograd through
    its backward kernels) on seeded closed (K = 10, sampled paths) and open
    (K = 4) curves."""
    gen = torch.Generator().manual_seed(17)
    out = {}
    for mode, k in (("closed", 10), ("unclosed", 4)):
        n = 7
        cp = (torch.rand(n, k, 2, generator=gen) * 2.6 - 1.3)
        op = torch.randn(n, 1, generator=gen) * 2.0
        xyz = torch.rand(n, 2, 24, 2, generator=gen) * 2.0 - 1.0
        out[f"{mode}_cp"], out[f"{mode}_op"], out[f"{mode}_xyz"] = _np(cp), _np(op), _np(xyz)
        tcp = cp.to(dev).requires_grad_(True)
        top = op.to(dev).requires_grad_(True)
        txyz = xyz.to(dev).requires_grad_(True) if mode == "closed" else None
        loss = manbo.regularization_loss_tilelang(tcp, top, txyz, mode=mode, **REG_KW)
        loss.backward()
        out[f"{mode}_loss"] = _np(loss.detach().reshape(1))
        out[f"{mode}_g_cp"], out[f"{mode}_g_op"] = _np(tcp.grad), _np(top.grad)
        if txyz is not None:
            out[f"{mode}_g_xyz"] = _np(txyz.grad)
    return out


def ccl_case(dev):
    """The reference's 4-connected labelling (raw labels and the stats
    variant) on seeded masks."""
    from manbo.ops import connected_components as ccm
    out = {}
    for i, (shape, density) in enumerate((((13, 19), 0.5), ((64, 97), 0.6), ((40, 40), 0.0))):
        gen = torch.Generator().manual_seed(70 + i)
        mask = torch.rand(shape, generator=gen) < density
        out[f"m{i}_mask"] = _np(mask.to(torch.uint8))
        out[f"m{i}_raw"] = _np(ccm.connected_components_labels_4_tilelang(mask.to(dev)))
        n, lab, stats, cent = ccm.connected_components_with_stats_4_tilelang(mask.to(dev))
        out[f"m{i}_n"] = np.array([n], np.int32)
        out[f"m{i}_labels"], out[f"m{i}_stats"], out[f"m{i}_centers"] = \
            _np(lab), _np(stats), _np(cent)
    return out


def dc_cubics(seed: int, n: int) -> torch.Tensor:
    """Pixel-space cubics for the adaptive flatten: random ones plus straight,
    fully degenerate, closed-loop (zero chord), tiny and very large ones."""
    g = torch.Generator().manual_seed(seed)
    rnd = torch.rand(n, 4, 2, generator=g) * 200.0
    t = torch.linspace(0.0, 1.0, 4).view(4, 1)
    line = torch.tensor([[3.0, 5.0]]) + t * torch.tensor([[90.0, 40.0]])
    point = torch.full((4, 2), 17.25)
    loop = torch.tensor([[50.0, 50.0], [120.0, 10.0], [-20.0, 10.0], [50.0, 50.0]])
    tiny = torch.tensor([[10.0, 10.0], [10.1, 10.3], [10.2, 9.9], [10.4, 10.1]])
    huge = torch.tensor([[0.0, 0.0], [5000.0, 9000.0], [-4000.0, 7000.0], [3000.0, -100.0]])
    near = torch.tensor([[0.0, 0.0], [30.0, 0.49], [60.0, -0.5], [90.0, 0.0]])
    return torch.cat([rnd, torch.stack([line, point, loop, tiny, huge, near])], 0).contiguous()


def dc_flatten_case(cs):
    """The reference's adaptive de Casteljau flatten on its host branch
    (cubic_splatting.py:1729-1832, CPU tensors) for several sample counts."""
    out = {}
    cub = dc_cubics(51, 58)
    g = int(cub.shape[0])
    offs = torch.tensor([0, 5, 5, 17, 40, g], dtype=torch.int32)  # an empty primitive
    out["cubics_px"] = _np(cub)
    out["offs"] = _np(offs)
    out["flat_tol0.5"] = _np(cs.cubic_adaptive_flatness_flags_tilelang(cub, tol_px=0.5))
    out["flat_tol3"] = _np(cs.cubic_adaptive_flatness_flags_tilelang(cub, tol_px=3.0))
    left, right = cs.cubic_split_half_tilelang(cub)
    out["split_left"] = _np(left)
    out["split_right"] = _np(right)
    for s in (5, 16, 24, 33):
        edges, peo, seo, t0, t1 = cs._flatten_cubics_to_edges(
            cub, offs, distance_samples=s, flatten_method="de_casteljau")
        out[f"s{s}_edges_px"] = _np(edges)
        out[f"s{s}_prim_edge_offsets"] = _np(peo)
        out[f"s{s}_segment_edge_offsets"] = _np(seo)
        out[f"s{s}_edge_t_starts"] = _np(t0)
        out[f"s{s}_edge_t_ends"] = _np(t1)
    return out


def dc_api_case(cs, ps, scene, grad_seed, dev, stroke=False):
    """Image and gradients of the public entry point with
    flatten_method="de_casteljau" (fill or stroke)."""
    h, w, s = scene.height, scene.width, scene.samples
    cn = scene.cubics_norm().to(dev).clone().requires_grad_(True)
    offs = scene.seg_offsets().to(dev)
    col = scene.colors.to(dev).clone().requires_grad_(True)
    op = scene.opacities.to(dev).clone().requires_grad_(True)
    depths = scene.depths.to(dev)
    aw = scene.aa_widths.to(dev).clone().requires_grad_(True)
    bg = scene.background.to(dev)
    v_out = scenes.seeded_grad(grad_seed, h, w).to(dev)
    res = {"cubics_norm": _np(cn), "offs": _np(offs), "colors": _np(col), "opacities": _np(op),
           "depths": _np(depths), "aa_widths": _np(aw), "background": _np(bg),
           "hw_s": np.array([h, w, s], np.int32), "v_output": _np(v_out)}
    if stroke:
        sw = scene.stroke_widths.to(dev).clone().requires_grad_(True)
        out = ps.render_cubic_polyline_splat_tilelang(
            cn, offs, col, op, sw, depths, h, w, 16, 16, bg, aa_widths=aw, distance_samples=s,
            flatten_method="de_casteljau")
        res["stroke_widths"] = _np(sw)
    else:
        rules = scene.fill_rules.to(dev)
        out = cs.render_cubic_fill_splat_tilelang(
            cn, offs, col, op, depths, h, w, 16, 16, bg, fill_rules=rules, aa_widths=aw,
            distance_samples=s, flatten_method="de_casteljau")
        res["fill_rules"] = _np(rules)
    (out * v_out).sum().backward()
    res.update(api_image=_np(out), api_v_cubics_norm=_np(cn.grad), api_v_colors=_np(col.grad),
               api_v_opacities=_np(op.grad), api_v_aa_widths=_np(aw.grad))
    if stroke:
        res["api_v_stroke_widths"] = _np(sw.grad)
    return res


def time_config2(manbo, cs, dev, iters: int, warmup: int):
    """Reference training step at config 2: render + MSE + SSIM + backward + Adam."""
    sc = scenes.config2()
    h, w = sc.height, sc.width
    ring = sc.ring.to(dev).clone().requires_grad_(True)
    colors = sc.colors.to(dev).clone().requires_grad_(True)
    opac, depths = sc.opacities.to(dev), sc.depths.to(dev)
    rules, aa, bg = sc.fill_rules.to(dev), sc.aa_widths.to(dev), sc.background.to(dev)
    offs = sc.seg_offsets().to(dev)
    target = sc.target.to(dev)
    gidx = scenes.ring_gather_index(sc.segs_per_path).to(dev)
    half = torch.tensor([0.5 * w, 0.5 * h], device=dev)
    opt = torch.optim.Adam([{"params": [ring], "lr": 0.5}, {"params": [colors], "lr": 0.01}])

    def step():
        opt.zero_grad(set_to_none=True)
        cub = ring[:, gidx, :].reshape(-1, 4, 2)
        cn = cub / half - 1.0
        out = cs.render_cubic_fill_splat_tilelang(cn, offs, colors, opac, depths, h, w, 16, 16, bg,
                                                  fill_rules=rules, aa_widths=aa,
                                                  distance_samples=sc.samples)
        img = torch.clamp(out, 0, 1).permute(2, 0, 1).unsqueeze(0).contiguous()
        loss = manbo.mse_loss_tilelang(img, target)
        with torch.no_grad():
            s = manbo.ssim(img.detach(), target)
        loss.backward()
        opt.step()
        return loss, s

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(iters):
        loss, s = step()
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    return {"iters": iters, "seconds": dt, "iters_per_s": iters / dt,
            "final_loss": float(loss.item()), "final_ssim": float(s.item())}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.path.join(ROOT, "baseline", "_ref"))
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--time", action="store_true")
    ap.add_argument("--no-golden", action="store_true")
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--json", default=None)
    ap.add_argument("--cases", default="all",
                    help="comma-separated fixtures to (re)generate, e.g. adan; default all")
    args = ap.parse_args(argv)

    sys.path.insert(0, os.path.abspath(args.ref))
    import tilelang  # noqa: F401
    import manbo
    from manbo import metric
    from manbo.ops import cubic_polyline_splatting as ps
    from manbo.ops import cubic_splatting as cs
    from manbo.ops import tile_bins as tb

    cases = None if args.cases == "all" else set(args.cases.split(","))
    if cases == {"dc_flatten"}:  # the host branch needs no GPU
        _save(args.out, "dc_flatten", dc_flatten_case(cs))
        return
    dev = torch.device("cuda")
    info = {"torch": torch.__version__, "tilelang": getattr(tilelang, "__version__", "?"),
            "gpu": torch.cuda.get_device_name(0)}
    print(info, flush=True)
    dc_fill = lambda: dc_api_case(cs, ps, scenes.small_fill_scene(61, paths=8), 62, dev)  # noqa
    dc_stroke = lambda: dc_api_case(cs, ps, scenes.small_stroke_scene(63), 64, dev,  # noqa
                                    stroke=True)
    if not args.no_golden and cases is not None:
        if "adan" in cases:
            _save(args.out, "adan", adan_case(manbo, dev))
        if "dc_flatten" in cases:
            _save(args.out, "dc_flatten", dc_flatten_case(cs))
        if "dc_fill" in cases:
            _save(args.out, "dc_fill", dc_fill())
        if "dc_stroke" in cases:
            _save(args.out, "dc_stroke", dc_stroke())
        if "regularization" in cases:
            _save(args.out, "regularization", reg_case(manbo, dev))
        if "components" in cases:
            _save(args.out, "components", ccl_case(dev))
    elif not args.no_golden:
        _save(args.out, "dc_flatten", dc_flatten_case(cs))
        _save(args.out, "dc_fill", dc_fill())
        _save(args.out, "dc_stroke", dc_stroke())
        _save(args.out, "adan", adan_case(manbo, dev))
        _save(args.out, "regularization", reg_case(manbo, dev))
        _save(args.out, "components", ccl_case(dev))
        _save(args.out, "fill_small_a", fill_case(cs, tb, scenes.small_fill_scene(21), 31, dev))
        _save(args.out, "fill_small_b", fill_case(cs, tb, scenes.small_fill_scene(22, h=40, w=72, paths=9, samples=5), 32, dev))
        ties = scenes.small_fill_scene(23, paths=7, mixed=False)
        ties.depths = torch.full_like(ties.depths, 0.5)
        _save(args.out, "fill_ties", fill_case(cs, tb, ties, 33, dev))
        _save(args.out, "fill_config1", fill_case(cs, tb, scenes.config1(), 34, dev))
        _save(args.out, "stroke_small", stroke_case(cs, ps, tb, scenes.small_stroke_scene(41), 42, dev))
        _save(args.out, "ring_segments", ring_case(cs, dev))
        _save(args.out, "metrics", metric_case(metric, dev))
    if args.time:
        info["config2_reference_tilelang"] = time_config2(manbo, cs, dev, args.iters, 5)
        print(json.dumps(info), flush=True)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(info, f, indent=1)


if __name__ == "__main__":
    main()
