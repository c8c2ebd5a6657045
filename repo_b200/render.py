"""Host side of the B200 cubic renderer: binning, autograd functions, entry points.

Mirrors the reference's operator API for the hot path
(``render_cubic_fill_splat_tilelang``, manbo/ops/cubic_splatting.py:3128-3229;
``render_cubic_polyline_splat_tilelang``, manbo/ops/cubic_polyline_splatting.py:1341-1432)
with the same argument meaning, validation messages, empty-scene behaviour and
``process_fn`` hook stages.  All device work runs in the sm_100a kernels behind
the C ABI (``repo_b200._native``); there is no CPU path.

Differences from the reference, by design:
  * binning is the fused count -> scan -> scatter -> per-tile sort pipeline,
    which costs one host synchronisation per forward (to size the intersect
    list) instead of the reference's three or more;
  * ties in depth are ordered by primitive id (the order of a stable sort of
    the reference's keys).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Callable, Mapping, MutableMapping, Optional

import torch

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
INT64_MAX = (1 << 63) - 1
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
    key = (s, str(device))
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


@dataclass
class Binning:
    """Binned and staged frame: reference-format intersect list plus the per-tile
    raster input (near-edge records, per-intersect records, row offsets)."""
    cubics_px: torch.Tensor
    edges_px: torch.Tensor
    prim_edge_offsets: torch.Tensor
    prim_tile_ranges: torch.Tensor
    num_tiles_hit: torch.Tensor
    tile_bins: torch.Tensor
    prim_ids_sorted: torch.Tensor
    isect_ids_sorted: torch.Tensor
    num_intersects: int
    tile_bounds: tuple
    samples: int
    tile_rows: tuple
    tile_dlist: torch.Tensor
    imeta: torch.Tensor
    rowoff: Optional[torch.Tensor]
    dlist: torch.Tensor
    counters: torch.Tensor
    stroke: bool
    isect_strips: torch.Tensor                  # [I, 4, 2] per-strip record ranges
    unit_order: Optional[torch.Tensor] = None   # strip dispatch lists (staged work)
    unit_order_bwd: Optional[torch.Tensor] = None  # strip dispatch lists (forward's work)
    visit_lists: Optional[torch.Tensor] = None  # per strip: intersects that composited a pixel
    visit_winners: Optional[torch.Tensor] = None  # per listed visit and lane: closest-record codes
    flatten_method: str = CUBIC_FLATTEN_METHOD_BERNSTEIN
    segment_edge_offsets: Optional[torch.Tensor] = None  # de Casteljau CSR [G + 1]
    edge_t_starts: Optional[torch.Tensor] = None         # de Casteljau leaf intervals [E]
    edge_t_ends: Optional[torch.Tensor] = None


def _offsets_error(offs: torch.Tensor, num_segments: int) -> ValueError:
    o = offs.detach().to("cpu")
    return ValueError(
        "primitive_seg_offsets must start at 0 and end at num_segments "
        f"(got start={int(o[0])}, end={int(o[-1])}, num_segments={num_segments})")


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
                   flatten_method: str = CUBIC_FLATTEN_METHOD_BERNSTEIN) -> Binning:
    """Project, bound, flatten, bin, sort and stage all primitives (fused B200
    pipeline, one host synchronisation to size the intersect list).

    The intersect list equals the reference's K3 + flatten + K4 + cumsum + K5 +
    sort + K6 (cubic_splatting.py:2815-2908): tile_bins [T, 2] of [start, end)
    into prim_ids_sorted / isect_ids_sorted, front (small depth) first.
    stroke_widths selects stroke mode.  flatten_method "de_casteljau" flattens
    adaptively (cs_flatten_de_casteljau) before the counts instead of the
    uniform Bernstein flatten inside cs_bin_count.
    """
    dev = cubics_norm.device
    s = max(2, int(samples))
    g = int(cubics_norm.shape[0])
    p = int(offs.numel()) - 1
    tbx, tby, _ = tile_bounds_for(img_h, img_w)
    nt = tbx * tby
    r0, r1 = (0, tby) if tile_rows is None else (int(tile_rows[0]), int(tile_rows[1]))
    stroke = stroke_widths is not None
    cubics_px = torch.empty((g, 4, 2), dtype=torch.float32, device=dev)
    dc = flatten_method == CUBIC_FLATTEN_METHOD_DE_CASTELJAU
    prim_ranges = torch.empty((p, 4), dtype=torch.int32, device=dev)
    num_hit = torch.empty((p,), dtype=torch.int32, device=dev)
    tile_bins = torch.empty((nt, 2), dtype=torch.int32, device=dev)
    tile_dlist = torch.empty((nt, 2), dtype=torch.int32, device=dev)
    counters = torch.zeros((4,), dtype=torch.int32, device=dev)
    ws = _cached_workspace(_BIN_WS, dev, int(nat.call("cs_bin_workspace_size", nt)))
    st = nat.stream(dev)
    cn = _f32(cubics_norm)
    aw = _f32(aa_widths)
    sw = None if stroke_widths is None else _f32(stroke_widths)
    basis = bernstein_basis(s, dev)
    peo = seg_eo = t0 = t1 = None
    edge_offs = None
    if dc:
        nat.check(nat.call("cs_project_cubics", nat.ptr(cn), None, None, nat.ptr(cubics_px), None,
                           None, g, int(img_h), int(img_w), 16, 16, 0.0, 0, st),
                  "cs_project_cubics")
        edges, peo, seg_eo, t0, t1 = flatten_de_casteljau(cubics_px, offs, s, counters[1:2])
    else:
        edges = torch.empty((g * (s - 1), 2, 2), dtype=torch.float32, device=dev)
        edge_offs = torch.empty((p + 1,), dtype=torch.int32, device=dev)
    nat.check(nat.call("cs_bin_count", nat.ptr(cn), nat.ptr(offs), nat.ptr(aw), nat.ptr(sw),
                       nat.ptr(basis), nat.ptr(cubics_px), nat.ptr(edges), nat.ptr(peo),
                       nat.ptr(edge_offs), nat.ptr(prim_ranges),
                       nat.ptr(num_hit), nat.ptr(tile_bins), nat.ptr(tile_dlist),
                       nat.ptr(counters), ws.data_ptr(), p, g, INT64_MAX, INT64_MAX, s,
                       int(img_h), int(img_w), r0, r1, float(aabb_pad), int(bool(aniso)), None,
                       0, st),
              "cs_bin_count")
    # the one host synchronisation of the forward: sizes + status
    n_isect, status, n_dbound, _ = (int(v) for v in counters.tolist())
    if status == nat.CS_ERR_ARG:
        raise _offsets_error(offs, g)
    nat.check(status, "cs_bin_count")
    if dc:
        edge_offs = peo
    # per-frame buffers are sized in a few classes (_size_class), so that the
    # caching allocator reuses blocks from frame to frame; the sorted lists
    # are exact-length views
    ci, cd = _size_class(n_isect), _size_class(n_dbound)
    prim_sorted = torch.empty((ci,), dtype=torch.int32, device=dev)[:n_isect]
    isect_sorted = torch.empty((ci,), dtype=torch.int64, device=dev)[:n_isect]
    imeta = torch.empty((ci, 12), dtype=torch.int32, device=dev)
    rowoff = None if stroke else torch.empty((ci, 16), dtype=torch.int32, device=dev)
    dlist = torch.empty((cd, 8), dtype=torch.float32, device=dev)
    istrips = torch.empty((ci, 4, 2), dtype=torch.int32, device=dev)
    unit_order = torch.empty((int(nat.call("cs_unit_lists_size", max(1, r1 - r0) * tbx)) // 4,),
                             dtype=torch.int32, device=dev)
    if n_isect > 0:
        nat.check(nat.call("cs_bin_sort", nat.ptr(prim_ranges), nat.ptr(_f32(depths)),
                           nat.ptr(tile_bins), nat.ptr(prim_sorted), nat.ptr(isect_sorted),
                           nat.ptr(counters), ws.data_ptr(), p, n_isect, int(img_h), int(img_w),
                           r0, r1, nat.ptr(edges), nat.ptr(edge_offs), nat.ptr(colors),
                           nat.ptr(opacities), nat.ptr(inv_sigma2s), nat.ptr(fill_rules),
                           nat.ptr(sw), nat.ptr(tile_dlist), nat.ptr(imeta), nat.ptr(rowoff),
                           nat.ptr(istrips), nat.ptr(dlist), max(n_dbound, 1),
                           nat.ptr(unit_order), st), "cs_bin_sort")
    return Binning(cubics_px, edges, edge_offs, prim_ranges, num_hit, tile_bins, prim_sorted,
                   isect_sorted, n_isect, (tbx, tby, 1), s, (r0, r1), tile_dlist, imeta, rowoff,
                   dlist, counters, stroke, istrips, unit_order if n_isect > 0 else None,
                   flatten_method=flatten_method, segment_edge_offsets=seg_eo,
                   edge_t_starts=t0, edge_t_ends=t1)


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
    return Binning(None, edges_px, prim_edge_offsets, None, None, tile_bins, prim_ids_sorted,
                   None, n, (tbx, tby, 1), 0, (0, tby), tile_dlist, imeta, rowoff, dlist, counters,
                   stroke, istrips, unit_order)


def _size_class(n: int) -> int:
    """Smallest allocation size class >= max(n, 1): multiples of 1/16 of the
    power of two below n (at most 6.25% over), and at least 4096."""
    n = max(int(n), 1)
    if n <= 4096:
        return 4096
    step = 1 << (n.bit_length() - 5)
    return (n + step - 1) // step * step


_RASTER_WS: dict = {}
_BIN_WS: dict = {}


def _cached_workspace(cache: dict, device: torch.device, nbytes: int) -> torch.Tensor:
    """Workspace per device and exact size, zeroed when allocated and left
    zeroed by every launch that uses it, so launches in stream order share it.
    Keyed by size because its layout depends on the tile count: a buffer laid
    out for another grid would put the counters where that grid left data."""
    key = (str(device), int(nbytes))
    buf = cache.get(key)
    if buf is None:
        buf = torch.zeros((max(nbytes, 256),), dtype=torch.uint8, device=device)
        cache[key] = buf
    return buf


def _bwd_lists(b: "Binning"):
    """Dispatch lists for the backward: the forward's (measured work) when the
    forward filled them, else the staging pass's."""
    return b.unit_order_bwd if b.unit_order_bwd is not None else b.unit_order


def raster_workspace(device: torch.device, num_tiles: int) -> torch.Tensor:
    """Per-device workspace of the raster kernels (dispatch counter, completion
    ticket, per-strip loss partials).  It is zeroed when allocated and every
    launch leaves it zeroed, so launches in stream order share it."""
    key = str(device)
    need = int(nat.call("cs_raster_workspace_size", int(num_tiles)))
    buf = _RASTER_WS.get(key)
    if buf is None or buf.numel() < need:
        buf = torch.zeros((need,), dtype=torch.uint8, device=device)
        _RASTER_WS[key] = buf
    return buf


def _aa_widths(raw: torch.Tensor):
    """Clamped anti-aliasing widths and 1/sigma^2 in one launch
    (cs_aa_widths_forward): clamp(aa, min=1e-4), 1 / clamp(w^2, min=1e-6)."""
    n = int(raw.numel())
    buf = torch.empty((2, n), dtype=torch.float32, device=raw.device)
    nat.check(nat.call("cs_aa_widths_forward", nat.ptr(raw), nat.ptr(buf[0]), nat.ptr(buf[1]), n,
                       nat.stream(raw.device)), "cs_aa_widths_forward")
    return buf[0], buf[1]


def _aa_widths_grad(raw: torch.Tensor, widths: torch.Tensor, v_inv: torch.Tensor):
    """Gradient of the raw anti-aliasing widths: -2 v_inv / clamp(w^3, 1e-12)
    through the clamp(aa, min=1e-4) of the entry (cs_aa_widths_backward)."""
    n = int(widths.numel())
    out = torch.empty((n,), dtype=torch.float32, device=widths.device)
    nat.check(nat.call("cs_aa_widths_backward", nat.ptr(raw), nat.ptr(widths), nat.ptr(v_inv),
                       nat.ptr(out), n, nat.stream(widths.device)), "cs_aa_widths_backward")
    return out


def _inv_sigma2(widths: torch.Tensor) -> torch.Tensor:
    return (1.0 / torch.clamp(widths * widths, min=1e-6)).contiguous()


def _zeros_views(dev, *shapes):
    total = sum(math.prod(sh) for sh in shapes)
    buf = torch.zeros((max(total, 1),), dtype=torch.float32, device=dev)
    out, o = [], 0
    for sh in shapes:
        n = math.prod(sh)
        out.append(buf[o:o + n].view(sh))
        o += n
    return out


def forward_raster(b: Binning, background, img_h: int, img_w: int, out_chw=None, outputs=None):
    """Forward rasteriser over staged tiles: image [H, W, 3], final_Ts, final_idx
    (written into ``outputs`` when given)."""
    dev = b.tile_bins.device
    if outputs is None:
        out = torch.empty((img_h, img_w, 3), dtype=torch.float32, device=dev)
        fts = torch.empty((img_h, img_w), dtype=torch.float32, device=dev)
        fidx = torch.empty((img_h, img_w), dtype=torch.int32, device=dev)
    else:
        out, fts, fidx = outputs
    if b.num_intersects <= 0:
        out.copy_(background.view(1, 1, 3).expand(img_h, img_w, 3))
        fts.fill_(1.0)
        fidx.fill_(0)
        return out, fts, fidx
    st = nat.stream(dev)
    status = b.counters[1:2]
    ws = raster_workspace(dev, b.tile_bounds[0] * b.tile_bounds[1])
    if b.unit_order is not None and b.unit_order_bwd is None:
        b.unit_order_bwd = torch.empty_like(b.unit_order)
    if b.visit_lists is None:
        nt = b.tile_bounds[0] * b.tile_bounds[1]
        nbytes = int(nat.call("cs_visit_lists_size", int(b.num_intersects), nt))
        b.visit_lists = torch.empty((nbytes // 4,), dtype=torch.int32, device=dev)
        if not b.stroke:  # closest-record codes: fills only
            wbytes = int(nat.call("cs_visit_winners_size", int(b.num_intersects), nt))
            b.visit_winners = torch.empty((wbytes // 2,), dtype=torch.int16, device=dev)
    if not b.stroke:
        nat.check(nat.call("cs_fill_forward", nat.ptr(b.prim_ids_sorted), nat.ptr(b.tile_bins),
                           nat.ptr(b.tile_dlist), nat.ptr(b.imeta), nat.ptr(b.isect_strips),
                           nat.ptr(b.rowoff), nat.ptr(b.dlist), nat.ptr(b.unit_order),
                           nat.ptr(b.unit_order_bwd), nat.ptr(b.visit_lists),
                           nat.ptr(b.visit_winners), nat.ptr(background),
                           nat.ptr(out), nat.ptr(fts), nat.ptr(fidx),
                           nat.ptr(out_chw), None, None, nat.ptr(status), ws.data_ptr(),
                           img_h, img_w, b.tile_rows[0], b.tile_rows[1], st), "cs_fill_forward")
    else:
        nat.check(nat.call("cs_stroke_forward", nat.ptr(b.prim_ids_sorted), nat.ptr(b.tile_bins),
                           nat.ptr(b.tile_dlist), nat.ptr(b.imeta), nat.ptr(b.isect_strips),
                           nat.ptr(b.dlist), nat.ptr(b.unit_order), nat.ptr(b.unit_order_bwd),
                           nat.ptr(b.visit_lists), nat.ptr(b.visit_winners),
                           nat.ptr(background), nat.ptr(out), nat.ptr(fts), nat.ptr(fidx),
                           nat.ptr(out_chw), None,
                           None, nat.ptr(status), ws.data_ptr(), img_h, img_w,
                           b.tile_rows[0], b.tile_rows[1], st), "cs_stroke_forward")
    return out, fts, fidx


def raster_backward(b: Binning, num_primitives: int, background, final_ts, final_idx, v_output,
                    img_h, img_w, *, collect_contrib: bool = False,
                    collect_isect_contrib: bool = False, out_img=None, target_chw=None,
                    mse_scale=None):
    """Backward rasteriser.  Returns v_edges, v_colors, v_opacities, v_inv_sigma2s,
    v_stroke_widths (stroke only), curve_contrib_rgb, curve_isect_contrib."""
    dev = b.tile_bins.device
    p = int(num_primitives)
    ne = int(b.edges_px.shape[0])
    ni = int(b.num_intersects)
    shapes = [(ne, 2, 2), (p, 3), (p,), (p,)]
    if b.stroke:
        shapes.append((p,))
    if collect_contrib:
        shapes.append((p, 3))
    if collect_isect_contrib:
        shapes.append((ni,))
    views = _zeros_views(dev, *shapes)
    v_edges, v_colors, v_opac, v_inv = views[:4]
    i = 4
    v_sw = None
    if b.stroke:
        v_sw = views[i]
        i += 1
    contrib = None
    if collect_contrib:
        contrib = views[i]
        i += 1
    icontrib = views[i] if collect_isect_contrib else None
    if ni > 0 and ne > 0:
        st = nat.stream(dev)
        vo = None if v_output is None else _f32(v_output)
        status = b.counters[1:2]
        ws = raster_workspace(dev, b.tile_bounds[0] * b.tile_bounds[1])
        if not b.stroke:
            nat.check(nat.call("cs_fill_backward", nat.ptr(b.prim_ids_sorted), nat.ptr(b.tile_bins),
                               nat.ptr(b.tile_dlist), nat.ptr(b.imeta),
                               nat.ptr(b.isect_strips), nat.ptr(b.rowoff), nat.ptr(b.dlist),
                               nat.ptr(_bwd_lists(b)), nat.ptr(b.visit_lists),
                               nat.ptr(b.visit_winners), nat.ptr(background), nat.ptr(final_ts),
                               nat.ptr(final_idx), nat.ptr(vo), nat.ptr(out_img),
                               nat.ptr(target_chw), nat.ptr(mse_scale), nat.ptr(v_edges),
                               nat.ptr(v_colors), nat.ptr(v_opac), nat.ptr(v_inv),
                               nat.ptr(contrib), nat.ptr(icontrib), nat.ptr(status),
                               ws.data_ptr(), img_h, img_w, b.tile_rows[0], b.tile_rows[1], st),
                      "cs_fill_backward")
        else:
            nat.check(nat.call("cs_stroke_backward", nat.ptr(b.prim_ids_sorted),
                               nat.ptr(b.tile_bins), nat.ptr(b.tile_dlist), nat.ptr(b.imeta),
                               nat.ptr(b.isect_strips), nat.ptr(b.dlist),
                               nat.ptr(_bwd_lists(b)), nat.ptr(b.visit_lists),
                               nat.ptr(b.visit_winners), nat.ptr(background), nat.ptr(final_ts),
                               nat.ptr(final_idx), nat.ptr(vo), nat.ptr(out_img),
                               nat.ptr(target_chw), nat.ptr(mse_scale), nat.ptr(v_edges),
                               nat.ptr(v_colors), nat.ptr(v_opac), nat.ptr(v_sw), nat.ptr(v_inv),
                               nat.ptr(contrib), nat.ptr(icontrib), nat.ptr(status),
                               ws.data_ptr(), img_h, img_w, b.tile_rows[0], b.tile_rows[1], st),
                      "cs_stroke_backward")
    return v_edges, v_colors, v_opac, v_inv, v_sw, contrib, icontrib


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


def binning_edge_grads(b: Binning, v_edges: torch.Tensor, num_segments: int,
                       scale=(1.0, 1.0)) -> torch.Tensor:
    """Cubic gradients from edge gradients with the binning's flatten method."""
    if b.flatten_method == CUBIC_FLATTEN_METHOD_DE_CASTELJAU:
        return edge_grads_to_cubics_csr(v_edges, b.segment_edge_offsets, b.edge_t_starts,
                                        b.edge_t_ends, num_segments, scale)
    return edge_grads_to_cubics(v_edges, num_segments, b.samples, scale)


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


class CubicFillSplatFunction(torch.autograd.Function):
    """Closed-fill renderer (mirrors _CubicFillSplatFunction, cubic_splatting.py:2750-3125)."""

    @staticmethod
    def forward(ctx, cubics_norm, primitive_seg_offsets, colors, opacities, depths, fill_rules,
                img_h, img_w, block_x, block_y, background, project_threads, map_threads,
                aabb_pad, aniso_intersects, aa_widths, distance_samples,
                flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD, process_fn=None, tile_rows=None):
        nat.require_cuda(cubics_norm, "cubics_norm")
        method = normalize_cubic_flatten_method(flatten_method)
        _check_block(block_x, block_y)
        num_segments = int(cubics_norm.shape[0])
        offs = _i32(primitive_seg_offsets).view(-1)
        num_primitives = max(0, int(offs.numel()) - 1)
        bg = background.to(device=cubics_norm.device, dtype=torch.float32).view(3).contiguous()
        ctx.img_h, ctx.img_w = int(img_h), int(img_w)
        if num_primitives <= 0:
            ctx.empty = True
            return _empty_image(bg, img_h, img_w)
        _validate_common(num_primitives, num_segments, offs, colors, opacities, depths)
        if int(fill_rules.reshape(-1).shape[0]) != num_primitives:
            raise ValueError(
                f"fill_rules size must match primitive count ({num_primitives}), got {int(fill_rules.reshape(-1).shape[0])}")
        raw = _f32(aa_widths.to(device=cubics_norm.device, dtype=torch.float32).reshape(-1))
        if int(raw.numel()) != num_primitives:
            raise ValueError(
                f"aa_widths size must match primitive count ({num_primitives}), got {int(raw.numel())}")
        widths, inv_s2 = _aa_widths(raw)
        col = _f32(colors)
        op = _f32(opacities).view(-1)
        rules = _i32(fill_rules).view(-1)
        b = bin_primitives(cubics_norm, offs, depths.reshape(-1), widths, int(img_h), int(img_w),
                           int(distance_samples), colors=col, opacities=op, inv_sigma2s=inv_s2,
                           fill_rules=rules, aabb_pad=float(aabb_pad),
                           aniso=bool(aniso_intersects), tile_rows=tile_rows,
                           flatten_method=method)
        if b.num_intersects <= 0:
            ctx.empty = True
            return _empty_image(bg, img_h, img_w)
        out, fts, fidx = forward_raster(b, bg, int(img_h), int(img_w))
        ctx.empty = False
        ctx.binning = b
        ctx.process_fn = process_fn
        ctx.num_segments = num_segments
        ctx.save_for_backward(cubics_norm, offs, col, op, rules, raw, widths, inv_s2, bg, fts, fidx)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        nones = (None,) * 20
        if getattr(ctx, "empty", False):
            return nones
        cubics_norm, offs, colors, opac, rules, raw, widths, inv_s2, bg, fts, fidx = \
            ctx.saved_tensors
        b: Binning = ctx.binning
        process_fn = ctx.process_fn
        pre = _run_process_fn(process_fn, "pre_backward_rasterize", {
            "collect_curve_contrib_rgb": False,
            "collect_curve_isect_contrib": False,
            "num_primitives": int(colors.shape[0]),
            "colors": colors,
        })
        cc = bool(pre.get("collect_curve_contrib_rgb", False))
        ci = bool(pre.get("collect_curve_isect_contrib", False))
        v_edges, v_colors, v_opac, v_inv, _, contrib, icontrib = raster_backward(
            b, int(colors.shape[0]), bg, fts, fidx, grad_out, ctx.img_h, ctx.img_w,
            collect_contrib=cc, collect_isect_contrib=ci)
        half_w, half_h = 0.5 * float(ctx.img_w), 0.5 * float(ctx.img_h)
        if process_fn is None:
            v_cubics_norm = binning_edge_grads(b, v_edges, ctx.num_segments,
                                               (half_w, half_h))
        else:
            v_cubics_px = binning_edge_grads(b, v_edges, ctx.num_segments)
            post = _run_process_fn(process_fn, "post_backward_rasterize", {
                "v_cubics_px": v_cubics_px, "v_colors": v_colors, "v_opacity": v_opac,
                "curve_contrib_rgb": contrib, "curve_isect_contrib": icontrib,
                "primitive_ids_sorted": b.prim_ids_sorted, "tile_bins": b.tile_bins,
                "colors": colors, "opacities": opac, "primitive_seg_offsets": offs,
            })
            v_cubics_px = post["v_cubics_px"]
            v_colors = post["v_colors"]
            v_opac = post["v_opacity"]
            v_cubics_norm = torch.empty_like(cubics_norm, dtype=torch.float32)
            v_cubics_norm[..., 0] = v_cubics_px[..., 0] * half_w
            v_cubics_norm[..., 1] = v_cubics_px[..., 1] * half_h
        v_aa = _aa_widths_grad(raw, widths, v_inv)
        out = [None] * 20
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
                flatten_method=DEFAULT_CUBIC_FLATTEN_METHOD, process_fn=None, tile_rows=None):
        nat.require_cuda(cubics_norm, "cubics_norm")
        method = normalize_cubic_flatten_method(flatten_method)
        _check_block(block_x, block_y)
        num_segments = int(cubics_norm.shape[0])
        offs = _i32(primitive_seg_offsets).view(-1)
        num_primitives = max(0, int(offs.numel()) - 1)
        bg = background.to(device=cubics_norm.device, dtype=torch.float32).view(3).contiguous()
        ctx.img_h, ctx.img_w = int(img_h), int(img_w)
        if num_primitives <= 0:
            ctx.empty = True
            return _empty_image(bg, img_h, img_w)
        _validate_common(num_primitives, num_segments, offs, colors, opacities, depths,
                         stroke_widths=stroke_widths)
        raw = _f32(aa_widths.to(device=cubics_norm.device, dtype=torch.float32).reshape(-1))
        if int(raw.numel()) != num_primitives:
            raise ValueError(
                f"aa_widths size must match primitive count ({num_primitives}), got {int(raw.numel())}")
        widths, inv_s2 = _aa_widths(raw)
        sw = _f32(stroke_widths).view(-1)
        col = _f32(colors)
        op = _f32(opacities).view(-1)
        b = bin_primitives(cubics_norm, offs, depths.reshape(-1), widths, int(img_h), int(img_w),
                           int(distance_samples), colors=col, opacities=op, inv_sigma2s=inv_s2,
                           stroke_widths=sw, aabb_pad=float(aabb_pad),
                           aniso=bool(aniso_intersects), tile_rows=tile_rows,
                           flatten_method=method)
        if b.num_intersects <= 0:
            ctx.empty = True
            return _empty_image(bg, img_h, img_w)
        out, fts, fidx = forward_raster(b, bg, int(img_h), int(img_w))
        ctx.empty = False
        ctx.binning = b
        ctx.process_fn = process_fn
        ctx.num_segments = num_segments
        ctx.save_for_backward(cubics_norm, offs, col, op, sw, raw, widths, inv_s2, bg, fts, fidx)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        nones = (None,) * 20
        if getattr(ctx, "empty", False):
            return nones
        cubics_norm, offs, colors, opac, sw, raw, widths, inv_s2, bg, fts, fidx = \
            ctx.saved_tensors
        b: Binning = ctx.binning
        process_fn = ctx.process_fn
        pre = _run_process_fn(process_fn, "pre_backward_rasterize", {
            "collect_curve_contrib_rgb": False,
            "collect_curve_isect_contrib": False,
            "num_primitives": int(colors.shape[0]),
            "colors": colors,
        })
        cc = bool(pre.get("collect_curve_contrib_rgb", False))
        ci = bool(pre.get("collect_curve_isect_contrib", False))
        v_edges, v_colors, v_opac, v_inv, v_sw, contrib, icontrib = raster_backward(
            b, int(colors.shape[0]), bg, fts, fidx, grad_out, ctx.img_h, ctx.img_w,
            collect_contrib=cc, collect_isect_contrib=ci)
        half_w, half_h = 0.5 * float(ctx.img_w), 0.5 * float(ctx.img_h)
        if process_fn is None:
            v_cubics_norm = binning_edge_grads(b, v_edges, ctx.num_segments,
                                               (half_w, half_h))
        else:
            v_cubics_px = binning_edge_grads(b, v_edges, ctx.num_segments)
            post = _run_process_fn(process_fn, "post_backward_rasterize", {
                "v_cubics_px": v_cubics_px, "v_colors": v_colors, "v_opacity": v_opac,
                "v_stroke": v_sw, "curve_contrib_rgb": contrib, "curve_isect_contrib": icontrib,
                "primitive_ids_sorted": b.prim_ids_sorted, "tile_bins": b.tile_bins,
                "colors": colors, "opacities": opac, "stroke_widths": sw,
                "primitive_seg_offsets": offs,
            })
            v_cubics_px = post["v_cubics_px"]
            v_colors = post["v_colors"]
            v_opac = post["v_opacity"]
            v_sw = post["v_stroke"]
            v_cubics_norm = torch.empty_like(cubics_norm, dtype=torch.float32)
            v_cubics_norm[..., 0] = v_cubics_px[..., 0] * half_w
            v_cubics_norm[..., 1] = v_cubics_px[..., 1] * half_h
        v_aa = _aa_widths_grad(raw, widths, v_inv)
        out = [None] * 20
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
    return CubicFillSplatFunction.apply(
        cubics_norm, offs.contiguous(), colors.contiguous(), opacities.reshape(-1).contiguous(),
        depths.reshape(-1).contiguous(), rules.contiguous(), int(img_h), int(img_w), int(block_x),
        int(block_y), background, int(project_threads), int(map_threads), float(aabb_pad),
        bool(aniso_intersects), widths, int(distance_samples), method, process_fn, tile_rows)


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
    return CubicPolylineSplatFunction.apply(
        cubics_norm, offs.contiguous(), colors.contiguous(), opacities.reshape(-1).contiguous(),
        stroke_widths.reshape(-1).contiguous(), depths.reshape(-1).contiguous(), int(img_h),
        int(img_w), int(block_x), int(block_y), background, int(project_threads),
        int(map_threads), float(aabb_pad), bool(aniso_intersects), widths,
        int(distance_samples), method, process_fn, tile_rows)
