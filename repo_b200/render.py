"""Host side of the B200 cubic renderer: binning, autograd functions, entry points.

Mirrors the reference's operator API for the hot path
(``render_cubic_fill_splat_tilelang``, manbo/ops/cubic_splatting.py:3128-3229;
``render_cubic_polyline_splat_tilelang``, manbo/ops/cubic_polyline_splatting.py:1341-1432)
with the same argument meaning, validation messages, empty-scene behaviour and
``process_fn`` hook stages.  All device work runs in the sm_100a kernels behind
the C ABI (``repo_b200._native``); there is no CPU path.

Each autograd stage is one call into the torch binding (``repo_b200._ext``,
csrc/torch_api.cpp), which launches the stage's kernels on the current stream.

Differences from the reference, by design:
  * binning is the fused count -> scan -> scatter -> per-tile sort pipeline
    with intersect buffers sized from the previous frame of the same shape:
    a forward enqueues all of its launches and then reads the counts back
    once (the reference synchronises three or more times); a frame that
    outgrew the cached size is binned again, and under CUDA graph capture
    nothing is read back (an overflow then leaves the image NaN);
  * ties in depth are ordered by primitive id (the order of a stable sort of
    the reference's keys).
"""
from __future__ import annotations

from typing import Any, Callable, Mapping, MutableMapping, Optional

import torch

from . import _ext
from . import _native as nat

BLOCK_X = 16
BLOCK_Y = 16
DEFAULT_THREADS = 256
DEFAULT_AABB_PAD = 1.0
DEFAULT_AA_WIDTH = 1.0
DEFAULT_DISTANCE_SAMPLES = 24
CUBIC_FLATTEN_METHOD_BERNSTEIN = "bernstein"
CUBIC_FLATTEN_METHOD_DE_CASTELJAU = "de_casteljau"
DEFAULT_CUBIC_FLATTEN_METHOD = CUBIC_FLATTEN_METHOD_BERNSTEIN
_FLATTEN_ALIASES = {
    "bernstein": CUBIC_FLATTEN_METHOD_BERNSTEIN,
    "de_casteljau": CUBIC_FLATTEN_METHOD_DE_CASTELJAU,
    "decasteljau": CUBIC_FLATTEN_METHOD_DE_CASTELJAU,
    "de-casteljau": CUBIC_FLATTEN_METHOD_DE_CASTELJAU,
}
DE_CASTELJAU_TOL_PX = 0.5  # DEFAULT_DE_CASTELJAU_FLATNESS_TOL_PX (cubic_splatting.py:18)

CubicProcessPayload = MutableMapping[str, Any]
CubicProcessFn = Callable[[str, CubicProcessPayload], Optional[Mapping[str, Any]]]


def normalize_cubic_flatten_method(method: object) -> str:
    raw = str(method).strip().lower()
    key = _FLATTEN_ALIASES.get(raw, raw)
    if key not in (CUBIC_FLATTEN_METHOD_BERNSTEIN, CUBIC_FLATTEN_METHOD_DE_CASTELJAU):
        raise ValueError(
            "flatten_method must be one of "
            f"{sorted(_FLATTEN_ALIASES.keys())}, got {method!r}")
    return key


def _run_process_fn(process_fn, stage, payload):
    if process_fn is None:
        return payload
    updates = process_fn(stage, payload)
    if updates:
        payload.update(updates)
    return payload


def _f32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.float32:
        return t if t.is_contiguous() else t.contiguous()
    return t.contiguous().to(torch.float32)


def _i32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.int32:
        return t if t.is_contiguous() else t.contiguous()
    return t.contiguous().to(torch.int32)


_BASIS_CACHE: dict = {}


def bernstein_basis(samples: int, device: torch.device) -> torch.Tensor:
    """[4, S] cubic Bernstein weights at linspace(0, 1, S), computed with torch on
    the host exactly as the reference writes them (cubic_splatting.py:1710-1716)."""
    s = max(2, int(samples))
    key = (s, device.type, device.index)
    b = _BASIS_CACHE.get(key)
    if b is None:
        t = torch.linspace(0.0, 1.0, s, dtype=torch.float32)
        omt = 1.0 - t
        b = torch.stack([omt * omt * omt, 3.0 * omt * omt * t, 3.0 * omt * t * t, t * t * t], 0)
        b = b.contiguous().to(device)
        _BASIS_CACHE[key] = b
    return b


def tile_bounds_for(img_h: int, img_w: int) -> tuple[int, int, int]:
    return ((int(img_w) + BLOCK_X - 1) // BLOCK_X, (int(img_h) + BLOCK_Y - 1) // BLOCK_Y, 1)


def _check_block(block_x: int, block_y: int) -> None:
    if int(block_x) != BLOCK_X or int(block_y) != BLOCK_Y:
        raise ValueError(f"the B200 renderer uses 16x16 tiles, got block {block_x}x{block_y}")


class _LazyFrame:
    """``Binning`` is the binding's Frame type (loaded on first use)."""

    def __call__(self, **fields):
        f = _ext.load().Frame()
        for k, v in fields.items():
            setattr(f, k, v)
        return f

    def __instancecheck__(self, obj):
        return isinstance(obj, _ext.load().Frame)


# A binned and staged frame: reference-format intersect list (tile_bins,
# prim_ids_sorted, isect_ids_sorted) plus the per-tile raster input (near-edge
# records, per-intersect records, row offsets, dispatch and visit lists).
Binning = _LazyFrame()


def replace_binning(b, **changes):
    """A shallow copy of a frame with some fields replaced (the tensors are
    shared, as dataclasses.replace shares them)."""
    c = b.copy()
    for k, v in changes.items():
        setattr(c, k, v)
    return c


def flatten_de_casteljau(cubics_px: torch.Tensor, offs: torch.Tensor, samples: int,
                         status: Optional[torch.Tensor] = None, tol_px: float = DE_CASTELJAU_TOL_PX):
    """Adaptive de Casteljau flatten on the device, without a host
    synchronisation: edges [cap, 2, 2], prim_edge_offsets [P + 1],
    segment_edge_offsets [G + 1], edge t starts / ends [cap], where cap bounds
    the edge count E = segment_edge_offsets[-1]."""
    dev = cubics_px.device
    g = int(cubics_px.shape[0])
    p = max(0, int(offs.numel()) - 1)
    s = max(2, int(samples))
    cap = int(nat.call("cs_de_casteljau_edge_capacity", g, s))
    edges = torch.empty((max(cap, 1), 2, 2), dtype=torch.float32, device=dev)
    t0 = torch.empty((max(cap, 1),), dtype=torch.float32, device=dev)
    t1 = torch.empty((max(cap, 1),), dtype=torch.float32, device=dev)
    seg = torch.empty((g + 1,), dtype=torch.int32, device=dev)
    prim = torch.empty((p + 1,), dtype=torch.int32, device=dev)
    nat.check(nat.call("cs_flatten_de_casteljau", nat.ptr(cubics_px), nat.ptr(offs), g, p, s,
                       float(tol_px), nat.ptr(edges), nat.ptr(prim), nat.ptr(seg), nat.ptr(t0),
                       nat.ptr(t1), cap, nat.ptr(status), nat.stream(dev)),
              "cs_flatten_de_casteljau")
    return edges, prim, seg, t0, t1


def bin_primitives(cubics_norm: torch.Tensor, offs: torch.Tensor, depths: torch.Tensor,
                   aa_widths: torch.Tensor, img_h: int, img_w: int, samples: int, *,
                   colors: torch.Tensor, opacities: torch.Tensor, inv_sigma2s: torch.Tensor,
                   fill_rules: Optional[torch.Tensor] = None,
                   stroke_widths: Optional[torch.Tensor] = None,
                   aabb_pad: float = DEFAULT_AABB_PAD, aniso: bool = False,
                   tile_rows: Optional[tuple] = None,
                   flatten_method: str = CUBIC_FLATTEN_METHOD_BERNSTEIN):
    """Project, bound, flatten, bin, sort and stage all primitives (fused B200
    pipeline, one read-back of the counts).

    The intersect list equals the reference's K3 + flatten + K4 + cumsum + K5 +
    sort + K6 (cubic_splatting.py:2815-2908): tile_bins [T, 2] of [start, end)
    into prim_ids_sorted / isect_ids_sorted, front (small depth) first.
    stroke_widths selects stroke mode.  flatten_method "de_casteljau" flattens
    adaptively (cs_flatten_de_casteljau) before the counts instead of the
    uniform Bernstein flatten inside cs_bin_count.
    """
    s = max(2, int(samples))
    r0, r1 = (0, -1) if tile_rows is None else (int(tile_rows[0]), int(tile_rows[1]))
    return _ext.load().bin_frame(
        cubics_norm, _i32(offs), _f32(depths), _f32(aa_widths), _f32(inv_sigma2s), _f32(colors),
        _f32(opacities), None if fill_rules is None else _i32(fill_rules),
        None if stroke_widths is None else _f32(stroke_widths),
        bernstein_basis(s, cubics_norm.device), int(img_h), int(img_w), s, float(aabb_pad),
        bool(aniso), r0, r1, flatten_method == CUBIC_FLATTEN_METHOD_DE_CASTELJAU)


def stage_reference_lists(prim_ids_sorted, tile_bins, edges_px, isect_edge_ranges, colors,
                          opacities, inv_sigma2s, fill_rules, stroke_widths, img_h, img_w,
                          prim_edge_offsets=None) -> Binning:
    """Stage a reference-format sorted intersect list for the raster kernels
    (per-stage API).  Costs one host synchronisation to size the records."""
    dev = edges_px.device
    tbx, tby, _ = tile_bounds_for(img_h, img_w)
    nt = tbx * tby
    n = int(prim_ids_sorted.numel())
    stroke = stroke_widths is not None
    if isect_edge_ranges is not None:
        slots = int((isect_edge_ranges[:, 1] - isect_edge_ranges[:, 0]).clamp_min(0).sum().item())
    else:
        eo = prim_edge_offsets.to(torch.int64)
        pid = prim_ids_sorted.to(torch.int64)
        slots = int((eo[pid + 1] - eo[pid]).clamp_min(0).sum().item())
    bound = 4 * slots  # every strip of a tile has room for all of the tile's edge slots
    tile_dlist = torch.empty((nt, 2), dtype=torch.int32, device=dev)
    counters = torch.zeros((4,), dtype=torch.int32, device=dev)
    imeta = torch.empty((max(n, 1), 12), dtype=torch.int32, device=dev)
    rowoff = None if stroke else torch.empty((max(n, 1), 16), dtype=torch.int32, device=dev)
    dlist = torch.empty((max(bound, 1), 8), dtype=torch.float32, device=dev)
    istrips = torch.empty((max(n, 1), 4, 2), dtype=torch.int32, device=dev)
    unit_order = torch.empty((int(nat.call("cs_unit_lists_size", nt)) // 4,), dtype=torch.int32,
                             device=dev)
    ws = torch.empty((int(nat.call("cs_stage_workspace_size", nt)),), dtype=torch.uint8,
                     device=dev)
    nat.check(nat.call("cs_tile_stage", nat.ptr(prim_ids_sorted), nat.ptr(tile_bins),
                       nat.ptr(edges_px), nat.ptr(isect_edge_ranges), nat.ptr(prim_edge_offsets),
                       nat.ptr(colors), nat.ptr(opacities), nat.ptr(inv_sigma2s),
                       nat.ptr(fill_rules), nat.ptr(stroke_widths), nat.ptr(tile_dlist),
                       nat.ptr(imeta), nat.ptr(rowoff), nat.ptr(istrips), nat.ptr(dlist),
                       nat.ptr(unit_order), nat.ptr(counters), ws.data_ptr(), max(bound, 1),
                       int(img_h), int(img_w), nat.stream(dev)),
              "cs_tile_stage")
    return Binning(edges_px=edges_px, prim_edge_offsets=prim_edge_offsets, tile_bins=tile_bins,
                   prim_ids_sorted=prim_ids_sorted, num_intersects=n, isect_capacity=max(n, 1),
                   tile_bounds=(tbx, tby, 1), samples=0, tile_rows=(0, tby),
                   tile_dlist=tile_dlist, imeta=imeta, rowoff=rowoff, dlist=dlist,
                   counters=counters, stroke=stroke, isect_strips=istrips, unit_order=unit_order)


def _aa_widths(raw: torch.Tensor):
    """Clamped anti-aliasing widths and 1/sigma^2 in one launch
    (cs_aa_widths_forward): clamp(aa, min=1e-4), 1 / clamp(w^2, min=1e-6)."""
    return _ext.load().aa_widths_forward(raw)


def _aa_widths_grad(raw: torch.Tensor, widths: torch.Tensor, v_inv: torch.Tensor):
    """Gradient of the raw anti-aliasing widths: -2 v_inv / clamp(w^3, 1e-12)
    through the clamp(aa, min=1e-4) of the entry (cs_aa_widths_backward)."""
    return _ext.load().aa_widths_backward(raw, widths, v_inv)


def _inv_sigma2(widths: torch.Tensor) -> torch.Tensor:
    return (1.0 / torch.clamp(widths * widths, min=1e-6)).contiguous()


def forward_raster(b, background, img_h: int, img_w: int, out_chw=None, outputs=None):
    """Forward rasteriser over staged tiles: image [H, W, 3], final_Ts, final_idx
    (written into ``outputs`` when given)."""
    o = (None, None, None) if outputs is None else tuple(outputs)
    return _ext.load().raster_forward(b, background, int(img_h), int(img_w), out_chw, *o)


def raster_backward(b, num_primitives: int, background, final_ts, final_idx, v_output,
                    img_h, img_w, *, collect_contrib: bool = False,
                    collect_isect_contrib: bool = False, out_img=None, target_chw=None,
                    mse_scale=None):
    """Backward rasteriser.  Returns v_edges, v_colors, v_opacities, v_inv_sigma2s,
    v_stroke_widths (stroke only), curve_contrib_rgb, curve_isect_contrib."""
    return tuple(_ext.load().raster_backward(
        b, int(num_primitives), background, final_ts, final_idx, v_output, int(img_h),
        int(img_w), bool(collect_contrib), bool(collect_isect_contrib), out_img, target_chw,
        mse_scale))


def edge_grads_to_cubics_csr(v_edges: torch.Tensor, segment_edge_offsets: torch.Tensor,
                             edge_t_starts: torch.Tensor, edge_t_ends: torch.Tensor,
                             num_segments: int, scale=(1.0, 1.0)) -> torch.Tensor:
    """Edge gradients of a de Casteljau flattening -> cubic gradients."""
    dev = v_edges.device
    out = torch.empty((num_segments, 4, 2), dtype=torch.float32, device=dev)
    if num_segments > 0:
        nat.check(nat.call("cs_edge_grads_to_cubics_csr", nat.ptr(v_edges),
                           nat.ptr(edge_t_starts), nat.ptr(edge_t_ends),
                           nat.ptr(segment_edge_offsets), nat.ptr(out), int(num_segments),
                           float(scale[0]), float(scale[1]), nat.stream(dev)),
                  "cs_edge_grads_to_cubics_csr")
    return out


def binning_edge_grads(b, v_edges: torch.Tensor, num_segments: int,
                       scale=(1.0, 1.0)) -> torch.Tensor:
    """Cubic gradients from edge gradients with the binning's flatten method."""
    return _ext.load().edge_grads(b, v_edges, int(num_segments), float(scale[0]),
                                  float(scale[1]))


def edge_grads_to_cubics(v_edges: torch.Tensor, num_segments: int, samples: int,
                         scale=(1.0, 1.0)) -> torch.Tensor:
    dev = v_edges.device
    e = max(2, int(samples)) - 1
    out = torch.empty((num_segments, 4, 2), dtype=torch.float32, device=dev)
    if num_segments > 0:
        nat.check(nat.call("cs_edge_grads_to_cubics", nat.ptr(v_edges), nat.ptr(out),
                           int(num_segments), e, float(scale[0]), float(scale[1]),
                           nat.stream(dev)), "cs_edge_grads_to_cubics")
    return out


# --------------------------------------------------------------------------
# autograd functions

def _empty_image(bg: torch.Tensor, img_h: int, img_w: int) -> torch.Tensor:
    return bg.view(1, 1, 3).expand(int(img_h), int(img_w), 3).clone()


def _validate_common(num_primitives, num_segments, offs, colors, opacities, depths,
                     stroke_widths=None):
    """The entries' size checks in the reference's order (the stroke entry
    checks stroke widths before depths, cubic_polyline_splatting.py:1371-1387)."""
    if int(colors.shape[0]) != num_primitives:
        raise ValueError(
            f"colors first dim must match primitive count ({num_primitives}), got {int(colors.shape[0])}")
    if int(opacities.reshape(-1).shape[0]) != num_primitives:
        raise ValueError(
            f"opacities size must match primitive count ({num_primitives}), got {int(opacities.reshape(-1).shape[0])}")
    if stroke_widths is not None and int(stroke_widths.reshape(-1).shape[0]) != num_primitives:
        raise ValueError(
            f"stroke_widths size must match primitive count ({num_primitives}), got {int(stroke_widths.reshape(-1).shape[0])}")
    if int(depths.reshape(-1).shape[0]) != num_primitives:
        raise ValueError(
            f"depths size must match primitive count ({num_primitives}), got {int(depths.reshape(-1).shape[0])}")


def _background(background, device) -> torch.Tensor:
    bg = background
    if bg.device != device or bg.dtype != torch.float32:
        bg = bg.to(device=device, dtype=torch.float32)
    return bg.reshape(3) if bg.is_contiguous() else bg.contiguous().reshape(3)


def _backward_common(ctx, grad_out, colors, opac, raw, widths, bg, fts, fidx, extra_post=None):
    """Backward of both renderers: one binding call without a process_fn;
    with one, the reference's pre/post hook stages around the raster
    backward (cubic_splatting.py:3014-3091)."""
    b = ctx.binning
    p = int(colors.shape[0])
    half_w, half_h = 0.5 * float(ctx.img_w), 0.5 * float(ctx.img_h)
    process_fn = ctx.process_fn
    if process_fn is None:
        v_cubics_norm, v_colors, v_opac, v_aa, v_sw = _ext.load().render_backward(
            b, p, ctx.num_segments, bg, fts, fidx, grad_out, raw, widths, ctx.img_h, ctx.img_w,
            half_w, half_h)
        return v_cubics_norm, v_colors, v_opac, v_aa, v_sw
    pre = _run_process_fn(process_fn, "pre_backward_rasterize", {
        "collect_curve_contrib_rgb": False,
        "collect_curve_isect_contrib": False,
        "num_primitives": p,
        "colors": colors,
    })
    cc = bool(pre.get("collect_curve_contrib_rgb", False))
    ci = bool(pre.get("collect_curve_isect_contrib", False))
    v_edges, v_colors, v_opac, v_inv, v_sw, contrib, icontrib = raster_backward(
        b, p, bg, fts, fidx, grad_out, ctx.img_h, ctx.img_w, collect_contrib=cc,
        collect_isect_contrib=ci)
    v_cubics_px = binning_edge_grads(b, v_edges, ctx.num_segments)
    payload = {
        "v_cubics_px": v_cubics_px, "v_colors": v_colors, "v_opacity": v_opac,
        "curve_contrib_rgb": contrib, "curve_isect_contrib": icontrib,
        "primitive_ids_sorted": b.prim_ids_sorted, "tile_bins": b.tile_bins,
        "colors": colors, "opacities": opac, "primitive_seg_offsets": ctx.offs,
    }
    if extra_post:
        payload.update(extra_post(v_sw))
    post = _run_process_fn(process_fn, "post_backward_rasterize", payload)
    v_cubics_px = post["v_cubics_px"]
    v_colors = post["v_colors"]
    v_opac = post["v_opacity"]
    if b.stroke:
        v_sw = post["v_stroke"]
    v_cubics_norm = torch.empty(v_cubics_px.shape, dtype=torch.float32, device=v_cubics_px.device)
    v_cubics_norm[..., 0] = v_cubics_px[..., 0] * half_w
    v_cubics_norm[..., 1] = v_cubics_px[..., 1] * half_h
    v_aa = _aa_widths_grad(raw, widths, v_inv)
    return v_cubics_norm, v_colors, v_opac, v_aa, v_sw


def _forward_common(ctx, cubics_norm, offs, col, op, depths, rules, sw, raw, background, img_h,
                    img_w, aabb_pad, aniso, distance_samples, method, process_fn, tile_rows):
    dev = cubics_norm.device
    bg = _background(background, dev)
    h, w = int(img_h), int(img_w)
    ctx.img_h, ctx.img_w = h, w
    s = max(2, int(distance_samples))
    r0, r1 = (0, -1) if tile_rows is None else (int(tile_rows[0]), int(tile_rows[1]))
    out, fts, fidx, b, widths, _ = _ext.load().render_forward(
        cubics_norm, offs, col, op, depths, rules, sw, raw, bg, bernstein_basis(s, dev), h, w, s,
        float(aabb_pad), bool(aniso), r0, r1, method == CUBIC_FLATTEN_METHOD_DE_CASTELJAU)
    if b.num_intersects == 0:
        ctx.empty = True
        return out, None
    ctx.empty = False
    ctx.binning = b
    ctx.process_fn = process_fn
    ctx.num_segments = int(cubics_norm.shape[0])
    ctx.offs = offs
    return out, (widths, bg, fts, fidx)


class CubicFillSplatFunction(torch.autograd.Function):
    """Closed-fill renderer (mirrors _CubicFillSplatFunction, cubic_splatting.py:2750-3125).
    ``_checked`` (internal) marks arguments already validated and coerced by
    ``render_cubic_fill_splat``."""

    @staticmethod
    def forward(ctx, cubics_norm, primitive_seg_offsets, colors, opacities, depths, fill_rules,
                img_h, img_w, block_x, block_y, background, project_threads, map_threads,
                aabb_pad, aniso_intersects, aa_widths, distance_samples,
                flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD, process_fn=None, tile_rows=None,
                _checked=False):
        if _checked:
            method, offs, col, op, rules, raw = (flatten_method, primitive_seg_offsets, colors,
                                                 opacities, fill_rules, aa_widths)
            dep = depths
        else:
            nat.require_cuda(cubics_norm, "cubics_norm")
            method = normalize_cubic_flatten_method(flatten_method)
            _check_block(block_x, block_y)
            num_segments = int(cubics_norm.shape[0])
            offs = _i32(primitive_seg_offsets).view(-1)
            num_primitives = max(0, int(offs.numel()) - 1)
            if num_primitives <= 0:
                ctx.empty = True
                return _empty_image(_background(background, cubics_norm.device), img_h, img_w)
            _validate_common(num_primitives, num_segments, offs, colors, opacities, depths)
            if int(fill_rules.reshape(-1).shape[0]) != num_primitives:
                raise ValueError(
                    f"fill_rules size must match primitive count ({num_primitives}), got {int(fill_rules.reshape(-1).shape[0])}")
            raw = _f32(aa_widths.to(device=cubics_norm.device, dtype=torch.float32).reshape(-1))
            if int(raw.numel()) != num_primitives:
                raise ValueError(
                    f"aa_widths size must match primitive count ({num_primitives}), got {int(raw.numel())}")
            col = _f32(colors)
            op = _f32(opacities).view(-1)
            rules = _i32(fill_rules).view(-1)
            dep = _f32(depths.reshape(-1))
        out, keep = _forward_common(ctx, cubics_norm, offs, col, op, dep, rules, None, raw,
                                    background, img_h, img_w, aabb_pad, aniso_intersects,
                                    distance_samples, method, process_fn, tile_rows)
        if keep is not None:
            widths, bg, fts, fidx = keep
            ctx.save_for_backward(col, op, raw, widths, bg, fts, fidx)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if getattr(ctx, "empty", False):
            return (None,) * 21
        colors, opac, raw, widths, bg, fts, fidx = ctx.saved_tensors
        v_cubics_norm, v_colors, v_opac, v_aa, _ = _backward_common(
            ctx, grad_out, colors, opac, raw, widths, bg, fts, fidx)
        out = [None] * 21
        out[0] = v_cubics_norm
        out[2] = v_colors
        out[3] = v_opac.view_as(opac)
        out[4] = torch.zeros_like(opac) if ctx.needs_input_grad[4] else None
        out[15] = v_aa
        return tuple(out)


class CubicPolylineSplatFunction(torch.autograd.Function):
    """Open-stroke renderer (mirrors _CubicPolylineSplatFunction,
    cubic_polyline_splatting.py:962-1338)."""

    @staticmethod
    def forward(ctx, cubics_norm, primitive_seg_offsets, colors, opacities, stroke_widths, depths,
                img_h, img_w, block_x, block_y, background, project_threads, map_threads,
                aabb_pad, aniso_intersects, aa_widths, distance_samples,
                flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD, process_fn=None, tile_rows=None,
                _checked=False):
        if _checked:
            method, offs, col, op, sw, raw = (flatten_method, primitive_seg_offsets, colors,
                                              opacities, stroke_widths, aa_widths)
            dep = depths
        else:
            nat.require_cuda(cubics_norm, "cubics_norm")
            method = normalize_cubic_flatten_method(flatten_method)
            _check_block(block_x, block_y)
            num_segments = int(cubics_norm.shape[0])
            offs = _i32(primitive_seg_offsets).view(-1)
            num_primitives = max(0, int(offs.numel()) - 1)
            if num_primitives <= 0:
                ctx.empty = True
                return _empty_image(_background(background, cubics_norm.device), img_h, img_w)
            _validate_common(num_primitives, num_segments, offs, colors, opacities, depths,
                             stroke_widths=stroke_widths)
            raw = _f32(aa_widths.to(device=cubics_norm.device, dtype=torch.float32).reshape(-1))
            if int(raw.numel()) != num_primitives:
                raise ValueError(
                    f"aa_widths size must match primitive count ({num_primitives}), got {int(raw.numel())}")
            sw = _f32(stroke_widths).view(-1)
            col = _f32(colors)
            op = _f32(opacities).view(-1)
            dep = _f32(depths.reshape(-1))
        out, keep = _forward_common(ctx, cubics_norm, offs, col, op, dep, None, sw, raw,
                                    background, img_h, img_w, aabb_pad, aniso_intersects,
                                    distance_samples, method, process_fn, tile_rows)
        if keep is not None:
            widths, bg, fts, fidx = keep
            ctx.save_for_backward(col, op, sw, raw, widths, bg, fts, fidx)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if getattr(ctx, "empty", False):
            return (None,) * 21
        colors, opac, sw, raw, widths, bg, fts, fidx = ctx.saved_tensors
        v_cubics_norm, v_colors, v_opac, v_aa, v_sw = _backward_common(
            ctx, grad_out, colors, opac, raw, widths, bg, fts, fidx,
            extra_post=lambda v: {"v_stroke": v, "stroke_widths": sw})
        out = [None] * 21
        out[0] = v_cubics_norm
        out[2] = v_colors
        out[3] = v_opac.view_as(opac)
        out[4] = v_sw.view_as(sw)
        out[5] = torch.zeros_like(opac) if ctx.needs_input_grad[5] else None
        out[15] = v_aa
        return tuple(out)


# --------------------------------------------------------------------------
# public entry points (reference signatures)

def _prim_param(value, default, num_primitives, device, dtype, name):
    if value is None:
        return torch.full((num_primitives,), float(default), device=device, dtype=dtype)
    t = value.to(device=device, dtype=dtype).reshape(-1)
    if int(t.numel()) == 1 and num_primitives > 1:
        t = t.expand(num_primitives)
    if int(t.numel()) != num_primitives:
        raise ValueError(
            f"{name} size must match primitive count ({num_primitives}), got {int(t.numel())}")
    return t


def render_cubic_fill_splat(cubics_norm, primitive_seg_offsets, colors, opacities, depths, img_h,
                            img_w, block_x, block_y, background, *, fill_rules=None,
                            project_threads=DEFAULT_THREADS, map_threads=DEFAULT_THREADS,
                            aabb_pad=DEFAULT_AABB_PAD, aniso_intersects=False, aa_widths=None,
                            aa_width=DEFAULT_AA_WIDTH, distance_samples=DEFAULT_DISTANCE_SAMPLES,
                            flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD, process_fn=None,
                            tile_rows=None):
    """Render closed cubic fills, [H, W, 3] float32 (render_cubic_fill_splat_tilelang,
    cubic_splatting.py:3128-3229).  ``tile_rows`` restricts rendering to a band of
    tile rows (multi-GPU partition); rows outside it are left unwritten."""
    num_segments = int(cubics_norm.shape[0])
    offs = _i32(primitive_seg_offsets).view(-1)
    num_primitives = max(0, int(offs.numel()) - 1)
    if num_primitives <= 0:
        bg = background.to(device=cubics_norm.device, dtype=torch.float32).view(1, 1, 3)
        return bg.expand(int(img_h), int(img_w), 3).clone()
    _validate_common(num_primitives, num_segments, offs, colors, opacities, depths)
    dev = cubics_norm.device
    rules = _prim_param(fill_rules, 1, num_primitives, dev, torch.int32, "fill_rules")
    # raw widths: the Function clamps them (min 1e-4) and masks their gradient
    widths = _f32(_prim_param(aa_widths, aa_width, num_primitives, dev, torch.float32,
                              "aa_widths"))
    method = normalize_cubic_flatten_method(flatten_method)
    nat.require_cuda(cubics_norm, "cubics_norm")
    _check_block(block_x, block_y)
    return CubicFillSplatFunction.apply(
        cubics_norm, offs, _f32(colors), _f32(opacities.reshape(-1)), _f32(depths.reshape(-1)),
        _i32(rules), int(img_h), int(img_w), int(block_x), int(block_y), background,
        int(project_threads), int(map_threads), float(aabb_pad), bool(aniso_intersects), widths,
        int(distance_samples), method, process_fn, tile_rows, True)


def render_cubic_polyline_splat(cubics_norm, primitive_seg_offsets, colors, opacities,
                                stroke_widths, depths, img_h, img_w, block_x, block_y, background,
                                *, project_threads=DEFAULT_THREADS, map_threads=DEFAULT_THREADS,
                                aabb_pad=DEFAULT_AABB_PAD, aniso_intersects=False, aa_widths=None,
                                aa_width=DEFAULT_AA_WIDTH,
                                distance_samples=DEFAULT_DISTANCE_SAMPLES,
                                flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD, process_fn=None,
                                tile_rows=None):
    """Render open cubic strokes, [H, W, 3] float32 (render_cubic_polyline_splat_tilelang,
    cubic_polyline_splatting.py:1341-1432)."""
    num_segments = int(cubics_norm.shape[0])
    offs = _i32(primitive_seg_offsets).view(-1)
    num_primitives = max(0, int(offs.numel()) - 1)
    if num_primitives <= 0:
        bg = background.to(device=cubics_norm.device, dtype=torch.float32).view(1, 1, 3)
        return bg.expand(int(img_h), int(img_w), 3).clone()
    _validate_common(num_primitives, num_segments, offs, colors, opacities, depths,
                     stroke_widths=stroke_widths)
    dev = cubics_norm.device
    # raw widths: the Function clamps them (min 1e-4) and masks their gradient
    widths = _f32(_prim_param(aa_widths, aa_width, num_primitives, dev, torch.float32,
                              "aa_widths"))
    method = normalize_cubic_flatten_method(flatten_method)
    nat.require_cuda(cubics_norm, "cubics_norm")
    _check_block(block_x, block_y)
    return CubicPolylineSplatFunction.apply(
        cubics_norm, offs, _f32(colors), _f32(opacities.reshape(-1)),
        _f32(stroke_widths.reshape(-1)), _f32(depths.reshape(-1)), int(img_h), int(img_w),
        int(block_x), int(block_y), background, int(project_threads), int(map_threads),
        float(aabb_pad), bool(aniso_intersects), widths, int(distance_samples), method,
        process_fn, tile_rows, True)
