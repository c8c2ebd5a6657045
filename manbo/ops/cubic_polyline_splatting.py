"""Cubic stroke renderer operators with the reference's names and signatures
(manbo/ops/cubic_polyline_splatting.py), backed by the B200 sm_100a kernels."""
from __future__ import annotations

import torch

from repo_b200 import render as _r

from .cubic_splatting import (  # noqa: F401  (re-exported like the reference module)
    BLOCK_X,
    BLOCK_Y,
    DEFAULT_AA_WIDTH,
    DEFAULT_AABB_PAD,
    DEFAULT_CUBIC_FLATTEN_METHOD,
    DEFAULT_DISTANCE_SAMPLES,
    DEFAULT_THREADS,
    CubicProcessFn,
    CubicProcessPayload,
    _accumulate_edge_grads_to_cubics,
    _as_f32_contig,
    _as_i32_contig,
    _build_fill_isect_edge_ranges,
    _check_ranges,
    _flatten_cubics_to_edges,
    _inv_sigma2s,
    _primitive_tile_ranges_from_segment_tile_ranges,
    _run_cubic_process_fn,
    map_cubic_to_intersects_tilelang,
    normalize_cubic_flatten_method,
    project_cubics_2d_forward_tilelang,
)


def rasterize_cubic_polyline_forward_kernel(block_x: int = BLOCK_X, block_y: int = BLOCK_Y,
                                            dtype: str = "float32"):
    _r._check_block(block_x, block_y)

    def kernel(primitive_ids_sorted, tile_bins, edges_px, isect_edge_ranges, colors, opacities,
               stroke_widths, inv_sigma2s, background, out_img, final_Ts, final_idx):
        h, w = int(out_img.shape[0]), int(out_img.shape[1])
        b = _r.stage_reference_lists(primitive_ids_sorted, tile_bins, edges_px, isect_edge_ranges,
                                     colors, opacities, inv_sigma2s, None, stroke_widths, h, w)
        _r.forward_raster(b, background, h, w, outputs=(out_img, final_Ts, final_idx))
    return kernel


def rasterize_cubic_polyline_backward_kernel(block_x: int = BLOCK_X, block_y: int = BLOCK_Y,
                                             collect_curve_contrib: bool = False,
                                             collect_curve_isect_contrib: bool = False,
                                             dtype: str = "float32"):
    _r._check_block(block_x, block_y)

    def kernel(primitive_ids_sorted, tile_bins, edges_px, isect_edge_ranges, colors, opacities,
               stroke_widths, inv_sigma2s, background, final_Ts, final_idx, v_output, v_edges,
               v_colors, v_opacities, v_stroke_widths, v_inv_sigma2s, collect_curve_contrib_i32,
               curve_contrib_rgb, collect_curve_isect_contrib_i32, curve_isect_contrib):
        h, w = int(final_Ts.shape[0]), int(final_Ts.shape[1])
        b = _r.stage_reference_lists(primitive_ids_sorted, tile_bins, edges_px, isect_edge_ranges,
                                     colors, opacities, inv_sigma2s, None, stroke_widths, h, w)
        ve, vc, vo, vi, vs, cc, ci = _r.raster_backward(
            b, int(colors.shape[0]), background, final_Ts, final_idx, v_output, h, w,
            collect_contrib=bool(int(collect_curve_contrib_i32)),
            collect_isect_contrib=bool(int(collect_curve_isect_contrib_i32)))
        v_edges.add_(ve)
        v_colors.add_(vc)
        v_opacities.add_(vo)
        v_stroke_widths.add_(vs)
        v_inv_sigma2s.add_(vi)
        if cc is not None:
            curve_contrib_rgb.add_(cc)
        if ci is not None:
            curve_isect_contrib.add_(ci)
    return kernel


def rasterize_cubic_polyline_forward_tilelang(tile_bounds, block, img_size, primitive_ids_sorted,
                                              tile_bins, colors, opacities, stroke_widths,
                                              background, *, aa_widths=None, inv_sigma2s=None,
                                              edges_px, isect_edge_ranges,
                                              aa_width=DEFAULT_AA_WIDTH):
    img_w, img_h, _ = img_size
    p = int(colors.shape[0])
    ni = int(primitive_ids_sorted.shape[0])
    dev = colors.device
    out = torch.empty((img_h, img_w, 3), dtype=torch.float32, device=dev)
    fts = torch.empty((img_h, img_w), dtype=torch.float32, device=dev)
    fidx = torch.empty((img_h, img_w), dtype=torch.int32, device=dev)
    bg = background.to(device=dev, dtype=torch.float32).view(3).contiguous()
    if ni <= 0 or p <= 0 or int(edges_px.shape[0]) <= 0:
        out.copy_(bg.view(1, 1, 3).expand(img_h, img_w, 3))
        fts.fill_(1.0)
        fidx.fill_(0)
        return out, fts, fidx
    inv = _inv_sigma2s(p, dev, aa_widths, inv_sigma2s, aa_width)
    ranges = _check_ranges(isect_edge_ranges, ni)
    rasterize_cubic_polyline_forward_kernel(block[0], block[1])(
        _as_i32_contig(primitive_ids_sorted).view(-1), _as_i32_contig(tile_bins),
        _as_f32_contig(edges_px), ranges, _as_f32_contig(colors),
        _as_f32_contig(opacities).view(-1), _as_f32_contig(stroke_widths).view(-1), inv, bg, out,
        fts, fidx)
    return out, fts, fidx


def rasterize_cubic_polyline_backward_tilelang(tile_bounds, block, img_size, primitive_ids_sorted,
                                               tile_bins, cubics_px, primitive_seg_offsets, colors,
                                               opacities, stroke_widths, background, final_Ts,
                                               final_idx, v_output, *, aa_widths=None,
                                               inv_sigma2s=None, edges_px, isect_edge_ranges,
                                               segment_edge_offsets=None, edge_t_starts=None,
                                               edge_t_ends=None, aa_width=DEFAULT_AA_WIDTH,
                                               distance_samples=DEFAULT_DISTANCE_SAMPLES,
                                               flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD,
                                               curve_contrib_rgb=None, curve_isect_contrib=None):
    p = int(colors.shape[0])
    g = int(cubics_px.shape[0])
    dev = cubics_px.device
    v_colors = torch.zeros_like(colors, dtype=torch.float32)
    v_opac = torch.zeros_like(opacities.view(-1), dtype=torch.float32)
    v_sw = torch.zeros_like(stroke_widths.view(-1), dtype=torch.float32)
    v_inv = torch.zeros((p,), dtype=torch.float32, device=dev)
    v_cubics_px = torch.zeros_like(cubics_px, dtype=torch.float32)
    ni = int(primitive_ids_sorted.numel())
    if ni <= 0 or p <= 0 or g <= 0 or int(edges_px.shape[0]) <= 0:
        return v_cubics_px, v_colors, v_opac, v_sw, v_inv
    inv = _inv_sigma2s(p, dev, aa_widths, inv_sigma2s, aa_width)
    ranges = _check_ranges(isect_edge_ranges, ni)
    v_edges = torch.zeros_like(_as_f32_contig(edges_px))
    bg = background.to(device=dev, dtype=torch.float32).view(3).contiguous()
    rasterize_cubic_polyline_backward_kernel(block[0], block[1])(
        _as_i32_contig(primitive_ids_sorted).view(-1), _as_i32_contig(tile_bins),
        _as_f32_contig(edges_px), ranges, _as_f32_contig(colors),
        _as_f32_contig(opacities).view(-1), _as_f32_contig(stroke_widths).view(-1), inv, bg,
        _as_f32_contig(final_Ts), _as_i32_contig(final_idx), _as_f32_contig(v_output), v_edges,
        v_colors, v_opac, v_sw, v_inv, int(curve_contrib_rgb is not None), curve_contrib_rgb,
        int(curve_isect_contrib is not None), curve_isect_contrib)
    v_cubics_px = _accumulate_edge_grads_to_cubics(
        v_edges, g, distance_samples=distance_samples, flatten_method=flatten_method,
        segment_edge_offsets=segment_edge_offsets, edge_t_starts=edge_t_starts,
        edge_t_ends=edge_t_ends)
    return v_cubics_px, v_colors, v_opac, v_sw, v_inv


def render_cubic_polyline_splat_tilelang(cubics_norm, primitive_seg_offsets, colors, opacities,
                                         stroke_widths, depths, img_h, img_w, block_x, block_y,
                                         background, *, project_threads=DEFAULT_THREADS,
                                         map_threads=DEFAULT_THREADS, aabb_pad=DEFAULT_AABB_PAD,
                                         aniso_intersects=False, aa_widths=None,
                                         aa_width=DEFAULT_AA_WIDTH,
                                         distance_samples=DEFAULT_DISTANCE_SAMPLES,
                                         flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD,
                                         process_fn=None):
    """Render open cubic strokes into an [H, W, 3] float32 image."""
    return _r.render_cubic_polyline_splat(
        cubics_norm, primitive_seg_offsets, colors, opacities, stroke_widths, depths, img_h,
        img_w, block_x, block_y, background, project_threads=project_threads,
        map_threads=map_threads, aabb_pad=aabb_pad, aniso_intersects=aniso_intersects,
        aa_widths=aa_widths, aa_width=aa_width, distance_samples=distance_samples,
        flatten_method=flatten_method, process_fn=process_fn)


__all__ = [
    "rasterize_cubic_polyline_forward_kernel",
    "rasterize_cubic_polyline_backward_kernel",
    "rasterize_cubic_polyline_forward_tilelang",
    "rasterize_cubic_polyline_backward_tilelang",
    "render_cubic_polyline_splat_tilelang",
]
