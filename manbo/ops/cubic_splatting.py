"""Cubic fill renderer operators with the reference's names and signatures
(manbo/ops/cubic_splatting.py), backed by the B200 sm_100a kernels.

``render_cubic_fill_splat_tilelang`` is the hot-path entry point.  The
per-stage ``*_tilelang`` wrappers and the ``*_kernel`` factories reproduce the
reference's stage boundaries for callers that drive the pipeline step by step;
a ``*_kernel(...)`` factory returns a callable with the argument order of the
corresponding TileLang kernel, writing its outputs in place.
"""
from __future__ import annotations

from typing import Optional

import torch

from repo_b200 import _native as nat
from repo_b200 import render as _r
from repo_b200.ring import closed_cubic_fill_segments as _ring_segments
from repo_b200.ring import ring_basis as _ring_basis

BLOCK_X = _r.BLOCK_X
BLOCK_Y = _r.BLOCK_Y
DEFAULT_THREADS = _r.DEFAULT_THREADS
DEFAULT_AABB_PAD = _r.DEFAULT_AABB_PAD
DEFAULT_AA_WIDTH = _r.DEFAULT_AA_WIDTH
DEFAULT_DISTANCE_SAMPLES = _r.DEFAULT_DISTANCE_SAMPLES
DEFAULT_DE_CASTELJAU_FLATNESS_TOL_PX = 0.5
CUBIC_FLATTEN_METHOD_BERNSTEIN = _r.CUBIC_FLATTEN_METHOD_BERNSTEIN
CUBIC_FLATTEN_METHOD_DE_CASTELJAU = _r.CUBIC_FLATTEN_METHOD_DE_CASTELJAU
DEFAULT_CUBIC_FLATTEN_METHOD = _r.DEFAULT_CUBIC_FLATTEN_METHOD
CubicProcessPayload = _r.CubicProcessPayload
CubicProcessFn = _r.CubicProcessFn
CubicFillProcessPayload = CubicProcessPayload
CubicFillProcessFn = CubicProcessFn

normalize_cubic_flatten_method = _r.normalize_cubic_flatten_method
_run_cubic_process_fn = _r._run_process_fn
_as_f32_contig = _r._f32
_as_i32_contig = _r._i32


def _stream(t):
    return nat.stream(t.device)


# --------------------------------------------------------------------------
# closed ring segments

def _closed_fill_piecewise_basis_tensors(*, control_points_per_bezier, subdiv, device):
    return _ring_basis(control_points_per_bezier, subdiv, device)


def closed_cubic_fill_segments_tilelang(control_points, *, subdiv: int = 4,
                                        threads: int = DEFAULT_THREADS):
    return _ring_segments(control_points, subdiv=subdiv, threads=threads)


def closed_cubic_fill_segments_forward_kernel(control_points: int, subdiv: int = 4,
                                              threads: int = DEFAULT_THREADS,
                                              dtype: str = "float32"):
    k, sub = int(control_points), int(subdiv)
    if threads <= 0:
        raise ValueError("threads must be > 0")
    if k < 4 or (k - 2) % 2 != 0:
        raise ValueError("closed cubic fill expects control_points K with K>=4 and (K-2)%2==0, "
                         f"got K={k}")
    if sub <= 0:
        raise ValueError(f"subdiv must be > 0, got {sub}")

    def kernel(control_points_in, basis, deriv_basis, dt, out_segments, num_curves_i32,
               num_segments_i32):
        nat.check(nat.call("cs_ring_segments_forward", nat.ptr(control_points_in), nat.ptr(basis),
                           nat.ptr(deriv_basis), nat.ptr(dt), nat.ptr(out_segments),
                           int(num_curves_i32), k, sub, _stream(out_segments)),
                  "cs_ring_segments_forward")
    return kernel


def closed_cubic_fill_segments_backward_kernel(control_points: int, subdiv: int = 4,
                                               threads: int = DEFAULT_THREADS,
                                               dtype: str = "float32"):
    k, sub = int(control_points), int(subdiv)
    if k < 4 or (k - 2) % 2 != 0:
        raise ValueError("closed cubic fill expects control_points K with K>=4 and (K-2)%2==0, "
                         f"got K={k}")

    def kernel(grad_segments, basis, deriv_basis, dt, grad_control_points, num_curves_i32,
               num_segments_i32):
        nat.check(nat.call("cs_ring_segments_backward", nat.ptr(grad_segments), nat.ptr(basis),
                           nat.ptr(deriv_basis), nat.ptr(dt), nat.ptr(grad_control_points),
                           int(num_curves_i32), k, sub, _stream(grad_segments)),
                  "cs_ring_segments_backward")
    return kernel


# --------------------------------------------------------------------------
# projection, flattening, binning

def project_cubics_2d_forward_kernel(block_x: int = BLOCK_X, block_y: int = BLOCK_Y,
                                     threads: int = DEFAULT_THREADS,
                                     aabb_pad: float = DEFAULT_AABB_PAD,
                                     aniso_intersects: bool = False, dtype: str = "float32"):
    def kernel(cubics_norm, stroke_widths, support_radii, cubics_px, tile_ranges, num_tiles_hit,
               tile_bound_x, tile_bound_y, img_height, img_width):
        nat.check(nat.call("cs_project_cubics", nat.ptr(cubics_norm), nat.ptr(stroke_widths),
                           nat.ptr(support_radii), nat.ptr(cubics_px), nat.ptr(tile_ranges),
                           nat.ptr(num_tiles_hit), int(cubics_norm.shape[0]), int(img_height),
                           int(img_width), int(block_x), int(block_y), float(aabb_pad),
                           int(bool(aniso_intersects)), _stream(cubics_norm)), "cs_project_cubics")
    return kernel


def project_cubics_2d_forward_tilelang(cubics_norm, stroke_widths, support_radii, img_height,
                                       img_width, tile_bounds, *, block_x=BLOCK_X, block_y=BLOCK_Y,
                                       threads=DEFAULT_THREADS, aabb_pad=DEFAULT_AABB_PAD,
                                       aniso_intersects=False):
    n = int(cubics_norm.shape[0])
    dev = cubics_norm.device
    cubics_px = torch.empty((n, 4, 2), dtype=torch.float32, device=dev)
    tile_ranges = torch.empty((n, 4), dtype=torch.int32, device=dev)
    num_hit = torch.empty((n,), dtype=torch.int32, device=dev)
    if n > 0:
        project_cubics_2d_forward_kernel(block_x, block_y, threads, aabb_pad, aniso_intersects)(
            _as_f32_contig(cubics_norm), _as_f32_contig(stroke_widths).view(-1),
            _as_f32_contig(support_radii).view(-1), cubics_px, tile_ranges, num_hit,
            tile_bounds[0], tile_bounds[1], img_height, img_width)
    return cubics_px, tile_ranges, num_hit


def _flatten_cubics_to_edges(cubics_px, primitive_seg_offsets, *, distance_samples,
                             flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD):
    """Flatten cubics into edges once per frame (cubic_splatting.py:1654-1846):
    uniform Bernstein samples, or the adaptive de Casteljau split with CSR
    segment offsets and leaf parameter intervals."""
    cubics = _as_f32_contig(cubics_px)
    offs = _as_i32_contig(primitive_seg_offsets).view(-1)
    s = max(2, int(distance_samples))
    e = s - 1
    method = normalize_cubic_flatten_method(flatten_method)
    if cubics.ndim != 3 or tuple(cubics.shape[1:]) != (4, 2):
        raise ValueError(f"cubics_px must be [N,4,2], got {tuple(cubics.shape)}")
    if offs.ndim != 1 or int(offs.numel()) <= 0:
        raise ValueError(
            f"primitive_seg_offsets must be non-empty 1D tensor, got {tuple(offs.shape)}")
    g = int(cubics.shape[0])
    edge_offsets = offs.to(torch.int64).mul(e).to(torch.int32).contiguous()
    if g <= 0:
        return (torch.empty((0, 2, 2), dtype=torch.float32, device=cubics.device), edge_offsets,
                torch.zeros((1,), dtype=torch.int32, device=cubics.device), None, None)
    if method == CUBIC_FLATTEN_METHOD_DE_CASTELJAU:
        status = torch.zeros((1,), dtype=torch.int32, device=cubics.device)
        edges, peo, seg, t0, t1 = _r.flatten_de_casteljau(cubics, offs, s, status)
        n_edges, st = (int(v) for v in torch.stack([seg[-1], status[0]]).tolist())
        nat.check(st, "cs_flatten_de_casteljau")
        if int(offs[-1].item()) != g:
            raise ValueError(
                "primitive_seg_offsets end does not match segment count during flatten: "
                f"edge_offsets[-1]={int(peo[-1].item())}, expected={n_edges}")
        return edges[:n_edges], peo, seg, t0[:n_edges], t1[:n_edges]
    edges = torch.empty((g * e, 2, 2), dtype=torch.float32, device=cubics.device)
    nat.check(nat.call("cs_flatten_bernstein", nat.ptr(cubics),
                       nat.ptr(_r.bernstein_basis(s, cubics.device)), nat.ptr(edges), g, s,
                       _stream(cubics)), "cs_flatten_bernstein")
    seg_edge_offsets = torch.arange(0, (g + 1) * e, e, dtype=torch.int32, device=cubics.device)
    return edges, edge_offsets, seg_edge_offsets, None, None


def _build_fill_isect_edge_ranges(primitive_ids_sorted, primitive_edge_offsets, *, num_edges):
    pids = _as_i32_contig(primitive_ids_sorted).view(-1)
    offs = _as_i32_contig(primitive_edge_offsets).view(-1)
    out = torch.empty((int(pids.numel()), 2), dtype=torch.int32, device=pids.device)
    if pids.numel() > 0:
        nat.check(nat.call("cs_isect_edge_ranges", nat.ptr(pids), nat.ptr(offs), nat.ptr(out),
                           int(pids.numel()), _stream(pids)), "cs_isect_edge_ranges")
    return out


def primitive_tile_ranges_from_segment_ranges_kernel(threads: int = DEFAULT_THREADS):
    def kernel(segment_tile_ranges, primitive_seg_offsets, primitive_tile_ranges, num_tiles_hit,
               num_primitives_i32, num_segments_i32, tile_bound_x, tile_bound_y):
        nat.check(nat.call("cs_primitive_tile_ranges", nat.ptr(segment_tile_ranges),
                           nat.ptr(primitive_seg_offsets), nat.ptr(primitive_tile_ranges),
                           nat.ptr(num_tiles_hit), int(num_primitives_i32), int(tile_bound_x),
                           int(tile_bound_y), _stream(segment_tile_ranges)),
                  "cs_primitive_tile_ranges")
    return kernel


def _primitive_tile_ranges_from_segment_tile_ranges(segment_tile_ranges, primitive_seg_offsets,
                                                    tile_bounds):
    p = max(0, int(primitive_seg_offsets.numel()) - 1)
    dev = segment_tile_ranges.device
    if p <= 0:
        return (torch.empty((0, 4), dtype=torch.int32, device=dev),
                torch.empty((0,), dtype=torch.int32, device=dev))
    seg = _as_i32_contig(segment_tile_ranges)
    offs = _as_i32_contig(primitive_seg_offsets).view(-1)
    pr = torch.empty((p, 4), dtype=torch.int32, device=dev)
    hit = torch.empty((p,), dtype=torch.int32, device=dev)
    primitive_tile_ranges_from_segment_ranges_kernel()(seg, offs, pr, hit, p, int(seg.shape[0]),
                                                       tile_bounds[0], tile_bounds[1])
    return pr, hit


def map_cubic_to_intersects_kernel(threads: int = DEFAULT_THREADS):
    def kernel(tile_ranges, depths_i32, cum_tiles_hit, isect_ids, curve_ids, tile_bound_x,
               tile_bound_y):
        depths = depths_i32.view(torch.float32) if depths_i32.dtype == torch.int32 else depths_i32
        nat.check(nat.call("cs_map_cubic_to_intersects", nat.ptr(tile_ranges), nat.ptr(depths),
                           nat.ptr(cum_tiles_hit), nat.ptr(isect_ids), nat.ptr(curve_ids),
                           int(tile_ranges.shape[0]), int(tile_bound_x), _stream(tile_ranges)),
                  "cs_map_cubic_to_intersects")
    return kernel


def map_cubic_to_intersects_tilelang(tile_ranges, depths, cum_tiles_hit, tile_bounds, *,
                                     threads=DEFAULT_THREADS):
    n = int(cum_tiles_hit[-1].item()) if int(cum_tiles_hit.numel()) > 0 else 0
    dev = tile_ranges.device
    if n <= 0:
        return (torch.empty((0,), dtype=torch.int64, device=dev),
                torch.empty((0,), dtype=torch.int32, device=dev))
    ids = torch.empty((n,), dtype=torch.int64, device=dev)
    cids = torch.empty((n,), dtype=torch.int32, device=dev)
    map_cubic_to_intersects_kernel(threads)(_as_i32_contig(tile_ranges),
                                            _as_f32_contig(depths).view(-1),
                                            _as_i32_contig(cum_tiles_hit), ids, cids,
                                            tile_bounds[0], tile_bounds[1])
    return ids, cids


# --------------------------------------------------------------------------
# rasterisation

def _inv_sigma2s(num_primitives, device, aa_widths, inv_sigma2s, aa_width):
    if inv_sigma2s is None:
        if aa_widths is None:
            w = torch.full((num_primitives,), float(aa_width), device=device, dtype=torch.float32)
        else:
            w = aa_widths.to(device=device, dtype=torch.float32).view(-1)
            if int(w.numel()) == 1 and num_primitives > 1:
                w = w.expand(num_primitives)
            if int(w.numel()) != num_primitives:
                raise ValueError(f"aa_widths size must match num_primitives ({num_primitives}), "
                                 f"got {int(w.numel())}")
        w = torch.clamp(_as_f32_contig(w), min=1e-4)
        return (1.0 / torch.clamp(w * w, min=1e-6)).contiguous()
    t = inv_sigma2s.to(device=device, dtype=torch.float32).view(-1)
    if int(t.numel()) == 1 and num_primitives > 1:
        t = t.expand(num_primitives)
    if int(t.numel()) != num_primitives:
        raise ValueError(f"inv_sigma2s size must match num_primitives ({num_primitives}), "
                         f"got {int(t.numel())}")
    return _as_f32_contig(t)


def _check_ranges(isect_edge_ranges, num_intersects):
    r = _as_i32_contig(isect_edge_ranges)
    if r.ndim != 2 or int(r.shape[1]) != 2:
        raise ValueError(f"isect_edge_ranges must be [num_intersects,2], got {tuple(r.shape)}")
    if int(r.shape[0]) != num_intersects:
        raise ValueError("isect_edge_ranges first dim must match num_intersects "
                         f"({num_intersects}), got {int(r.shape[0])}")
    return r


def rasterize_cubic_fill_forward_kernel(block_x: int = BLOCK_X, block_y: int = BLOCK_Y,
                                        distance_samples: int = DEFAULT_DISTANCE_SAMPLES,
                                        dtype: str = "float32"):
    """Callable(primitive_ids_sorted, tile_bins, edges_px, isect_edge_ranges, colors,
    opacities, inv_sigma2s, fill_rules, background, out_img, final_Ts, final_idx)."""
    _r._check_block(block_x, block_y)

    def kernel(primitive_ids_sorted, tile_bins, edges_px, isect_edge_ranges, colors, opacities,
               inv_sigma2s, fill_rules, background, out_img, final_Ts, final_idx):
        h, w = int(out_img.shape[0]), int(out_img.shape[1])
        b = _r.stage_reference_lists(primitive_ids_sorted, tile_bins, edges_px, isect_edge_ranges,
                                     colors, opacities, inv_sigma2s, fill_rules, None, h, w)
        _r.forward_raster(b, background, h, w, outputs=(out_img, final_Ts, final_idx))
    return kernel


def rasterize_cubic_fill_forward_tilelang(tile_bounds, block, img_size, primitive_ids_sorted,
                                          tile_bins, cubics_px, primitive_seg_offsets, colors,
                                          opacities, fill_rules, background, *, aa_widths=None,
                                          inv_sigma2s=None, edges_px, isect_edge_ranges,
                                          aa_width=DEFAULT_AA_WIDTH,
                                          distance_samples=DEFAULT_DISTANCE_SAMPLES,
                                          map_threads=DEFAULT_THREADS):
    img_w, img_h, _ = img_size
    p = int(colors.shape[0])
    ni = int(primitive_ids_sorted.shape[0])
    dev = cubics_px.device
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
    rasterize_cubic_fill_forward_kernel(block[0], block[1])(
        _as_i32_contig(primitive_ids_sorted).view(-1), _as_i32_contig(tile_bins),
        _as_f32_contig(edges_px), ranges, _as_f32_contig(colors),
        _as_f32_contig(opacities).view(-1), inv, _as_i32_contig(fill_rules).view(-1), bg, out,
        fts, fidx)
    return out, fts, fidx


def rasterize_cubic_fill_backward_kernel(block_x: int = BLOCK_X, block_y: int = BLOCK_Y,
                                         distance_samples: int = DEFAULT_DISTANCE_SAMPLES,
                                         dtype: str = "float32"):
    """Callable with the argument order of the reference backward kernel; gradients
    are accumulated into the given buffers."""
    _r._check_block(block_x, block_y)

    def kernel(primitive_ids_sorted, tile_bins, edges_px, isect_edge_ranges, colors, opacities,
               inv_sigma2s, fill_rules, background, final_Ts, final_idx, v_output, v_edges,
               v_colors, v_opacities, v_inv_sigma2s, collect_curve_contrib, curve_contrib_rgb,
               collect_curve_isect_contrib, curve_isect_contrib):
        h, w = int(final_Ts.shape[0]), int(final_Ts.shape[1])
        b = _r.stage_reference_lists(primitive_ids_sorted, tile_bins, edges_px, isect_edge_ranges,
                                     colors, opacities, inv_sigma2s, fill_rules, None, h, w)
        ve, vc, vo, vi, _, cc, ci = _r.raster_backward(
            b, int(colors.shape[0]), background, final_Ts, final_idx, v_output, h, w,
            collect_contrib=bool(int(collect_curve_contrib)),
            collect_isect_contrib=bool(int(collect_curve_isect_contrib)))
        v_edges.add_(ve)
        v_colors.add_(vc)
        v_opacities.add_(vo)
        v_inv_sigma2s.add_(vi)
        if cc is not None:
            curve_contrib_rgb.add_(cc)
        if ci is not None:
            curve_isect_contrib.add_(ci)
    return kernel


def _accumulate_edge_grads_to_cubics(v_edges, num_segments, *, distance_samples,
                                     flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD,
                                     segment_edge_offsets=None, edge_t_starts=None,
                                     edge_t_ends=None, threads=DEFAULT_THREADS):
    s = max(2, int(distance_samples))
    if int(num_segments) <= 0:
        return torch.empty((0, 4, 2), dtype=torch.float32, device=v_edges.device)
    if normalize_cubic_flatten_method(flatten_method) == CUBIC_FLATTEN_METHOD_DE_CASTELJAU:
        if segment_edge_offsets is None or edge_t_starts is None or edge_t_ends is None:
            raise ValueError("de_casteljau flatten backward requires CSR metadata "
                             "(segment_edge_offsets, edge_t_starts, edge_t_ends)")
        seg = _as_i32_contig(segment_edge_offsets).view(-1)
        if int(seg.numel()) != int(num_segments) + 1:
            raise ValueError("segment_edge_offsets size mismatch: "
                             f"got {int(seg.numel())}, expected {int(num_segments) + 1}")
        first, last = (int(v) for v in seg[[0, -1]].tolist())
        if first != 0:
            raise ValueError(f"segment_edge_offsets must start at 0, got {first}")
        if last != int(v_edges.shape[0]) or last != int(edge_t_starts.numel()) or \
                last != int(edge_t_ends.numel()):
            raise ValueError("de_casteljau edge metadata size mismatch: "
                             f"offsets end at {last}, v_edges {int(v_edges.shape[0])}, "
                             f"t starts {int(edge_t_starts.numel())}, "
                             f"t ends {int(edge_t_ends.numel())}")
        return _r.edge_grads_to_cubics_csr(_as_f32_contig(v_edges), seg,
                                           _as_f32_contig(edge_t_starts).view(-1),
                                           _as_f32_contig(edge_t_ends).view(-1), int(num_segments))
    expected = int(num_segments) * (s - 1)
    if int(v_edges.shape[0]) != expected:
        raise ValueError(f"v_edges size mismatch: got {int(v_edges.shape[0])}, expected {expected}")
    return _r.edge_grads_to_cubics(_as_f32_contig(v_edges), int(num_segments), s)


def rasterize_cubic_fill_backward_tilelang(tile_bounds, block, img_size, primitive_ids_sorted,
                                           tile_bins, cubics_px, primitive_seg_offsets, colors,
                                           opacities, fill_rules, background, final_Ts, final_idx,
                                           v_output, *, aa_widths=None, inv_sigma2s=None,
                                           edges_px, isect_edge_ranges, segment_edge_offsets=None,
                                           edge_t_starts=None, edge_t_ends=None,
                                           aa_width=DEFAULT_AA_WIDTH,
                                           distance_samples=DEFAULT_DISTANCE_SAMPLES,
                                           flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD,
                                           map_threads=DEFAULT_THREADS, curve_contrib_rgb=None,
                                           curve_isect_contrib=None):
    p = int(colors.shape[0])
    g = int(cubics_px.shape[0])
    dev = cubics_px.device
    v_colors = torch.zeros_like(colors, dtype=torch.float32)
    v_opac = torch.zeros_like(opacities.view(-1), dtype=torch.float32)
    v_inv = torch.zeros((p,), dtype=torch.float32, device=dev)
    v_cubics_px = torch.zeros_like(cubics_px, dtype=torch.float32)
    ni = int(primitive_ids_sorted.numel())
    if ni <= 0 or p <= 0 or g <= 0 or int(edges_px.shape[0]) <= 0:
        return v_cubics_px, v_colors, v_opac, v_inv
    inv = _inv_sigma2s(p, dev, aa_widths, inv_sigma2s, aa_width)
    ranges = _check_ranges(isect_edge_ranges, ni)
    if curve_contrib_rgb is not None and curve_contrib_rgb.shape != colors.shape:
        raise ValueError("curve_contrib_rgb must match colors shape "
                         f"{tuple(colors.shape)}, got {tuple(curve_contrib_rgb.shape)}")
    if curve_isect_contrib is not None:
        if curve_isect_contrib.ndim != 1:
            raise ValueError("curve_isect_contrib must be a 1D tensor")
        if int(curve_isect_contrib.numel()) != ni:
            raise ValueError("curve_isect_contrib size must match primitive_ids_sorted")
    v_edges = torch.zeros_like(_as_f32_contig(edges_px))
    bg = background.to(device=dev, dtype=torch.float32).view(3).contiguous()
    rasterize_cubic_fill_backward_kernel(block[0], block[1])(
        _as_i32_contig(primitive_ids_sorted).view(-1), _as_i32_contig(tile_bins),
        _as_f32_contig(edges_px), ranges, _as_f32_contig(colors),
        _as_f32_contig(opacities).view(-1), inv, _as_i32_contig(fill_rules).view(-1), bg,
        _as_f32_contig(final_Ts), _as_i32_contig(final_idx), _as_f32_contig(v_output), v_edges,
        v_colors, v_opac, v_inv, int(curve_contrib_rgb is not None), curve_contrib_rgb,
        int(curve_isect_contrib is not None), curve_isect_contrib)
    v_cubics_px = _accumulate_edge_grads_to_cubics(
        v_edges, g, distance_samples=distance_samples, flatten_method=flatten_method,
        segment_edge_offsets=segment_edge_offsets, edge_t_starts=edge_t_starts,
        edge_t_ends=edge_t_ends)
    return v_cubics_px, v_colors, v_opac, v_inv


def render_cubic_fill_splat_tilelang(cubics_norm, primitive_seg_offsets, colors, opacities,
                                     depths, img_h, img_w, block_x, block_y, background, *,
                                     fill_rules=None, project_threads=DEFAULT_THREADS,
                                     map_threads=DEFAULT_THREADS, aabb_pad=DEFAULT_AABB_PAD,
                                     aniso_intersects=False, aa_widths=None,
                                     aa_width=DEFAULT_AA_WIDTH,
                                     distance_samples=DEFAULT_DISTANCE_SAMPLES,
                                     flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD,
                                     process_fn: Optional[CubicFillProcessFn] = None):
    """Render closed cubic fills into an [H, W, 3] float32 image, differentiable
    in cubics_norm, colors, opacities and aa_widths."""
    return _r.render_cubic_fill_splat(
        cubics_norm, primitive_seg_offsets, colors, opacities, depths, img_h, img_w, block_x,
        block_y, background, fill_rules=fill_rules, project_threads=project_threads,
        map_threads=map_threads, aabb_pad=aabb_pad, aniso_intersects=aniso_intersects,
        aa_widths=aa_widths, aa_width=aa_width, distance_samples=distance_samples,
        flatten_method=flatten_method, process_fn=process_fn)


def cubic_adaptive_flatness_flags_tilelang(cubics, *, tol_px, force_flat=False,
                                           threads=DEFAULT_THREADS):
    """Per-cubic flatness flags [N] uint8 of the adaptive flatten
    (cubic_splatting.py:1915-1957)."""
    c = _as_f32_contig(cubics)
    nat.require_cuda(c, "cubics")
    n = int(c.shape[0])
    out = torch.empty((n,), dtype=torch.uint8, device=c.device)
    if n > 0:
        nat.check(nat.call("cs_cubic_flatness_flags", nat.ptr(c), nat.ptr(out), n,
                           float(tol_px), int(bool(force_flat)), _stream(c)),
                  "cs_cubic_flatness_flags")
    return out


def cubic_split_half_tilelang(cubics, *, threads=DEFAULT_THREADS):
    """Split cubics at t = 1/2 into left / right halves (cubic_splatting.py:2031-2068)."""
    c = _as_f32_contig(cubics)
    nat.require_cuda(c, "cubics")
    n = int(c.shape[0])
    left = torch.empty((n, 4, 2), dtype=torch.float32, device=c.device)
    right = torch.empty((n, 4, 2), dtype=torch.float32, device=c.device)
    if n > 0:
        nat.check(nat.call("cs_cubic_split_half", nat.ptr(c), nat.ptr(left), nat.ptr(right), n,
                           _stream(c)), "cs_cubic_split_half")
    return left, right


__all__ = [
    "BLOCK_X", "BLOCK_Y", "DEFAULT_AA_WIDTH", "DEFAULT_AABB_PAD", "DEFAULT_DISTANCE_SAMPLES",
    "CUBIC_FLATTEN_METHOD_BERNSTEIN", "CUBIC_FLATTEN_METHOD_DE_CASTELJAU",
    "DEFAULT_CUBIC_FLATTEN_METHOD", "DEFAULT_THREADS", "normalize_cubic_flatten_method",
    "closed_cubic_fill_segments_forward_kernel", "closed_cubic_fill_segments_backward_kernel",
    "closed_cubic_fill_segments_tilelang", "map_cubic_to_intersects_kernel",
    "map_cubic_to_intersects_tilelang", "project_cubics_2d_forward_kernel",
    "project_cubics_2d_forward_tilelang", "rasterize_cubic_fill_forward_kernel",
    "rasterize_cubic_fill_forward_tilelang", "rasterize_cubic_fill_backward_kernel",
    "rasterize_cubic_fill_backward_tilelang", "render_cubic_fill_splat_tilelang",
]
