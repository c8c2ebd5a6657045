/*
 * cubicsplat_b200.h -- C ABI of the B200 (sm_100a) CubicSplat hot path.
 *
 * Every entry point takes raw device pointers, element counts and a
 * cudaStream_t passed as void* (the caller's current stream), launches its
 * kernels on that stream and returns a status code.  No entry point allocates
 * device memory; the ones that need scratch take a caller-provided workspace
 * whose size is reported by a *_workspace_size function.  Nothing is
 * synchronised: results are ready when the stream reaches them.
 *
 * Reference interfaces are cited by file:line inside the reference project
 * (manbo/ops/cubic_splatting.py, manbo/ops/cubic_polyline_splatting.py,
 * manbo/ops/tile_bins.py, manbo/ops/metric.py, manbo/metric.py,
 * manbo/ops/optim.py).  Tiles are
 * 16x16 pixels as in the reference default (BLOCK_X = BLOCK_Y = 16); other
 * block sizes return CS_ERR_UNSUPPORTED.  Images are [H, W, 3] float32
 * (HWC) as the reference renderer returns them; metric inputs are [N, C, H, W].
 */
#ifndef CUBICSPLAT_B200_H
#define CUBICSPLAT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CS_API __attribute__((visibility("default")))
#else
#define CS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define CS_OK 0
#define CS_ERR_ARG 1          /* bad size, null pointer or unsupported tile size */
#define CS_ERR_CAPACITY 2     /* intersect count exceeded the caller's capacity */
#define CS_ERR_CUDA 3         /* a kernel launch failed */
#define CS_ERR_UNSUPPORTED 4  /* valid but unsupported configuration */
#define CS_ERR_TIMEOUT 5      /* a bounded device-side wait gave up (reported on the device) */

/* Library version string and the list of exported entry points (for checks). */
CS_API const char *cs_version(void);

/* --------------------------------------------------------------------------
 * Projection, flattening and binning
 * ------------------------------------------------------------------------ */

/* Normalised cubic -> pixel space (p = fma(n, W/2, W/2)), exact cubic AABB from
 * the roots of B'(t), padded by max(aabb_pad, support) + half stroke width (or
 * the chord-anisotropic pad), tile rectangle [min, max) clamped to the grid.
 * Replaces project_cubics_2d_forward_kernel, cubic_splatting.py:546-747.
 * cubics_norm/cubics_px: [n, 4, 2]; stroke_widths, support_radii: [n] (NULL
 * reads as 0); tile_ranges: [n, 4]; num_tiles_hit: [n] (may be NULL).  With
 * tile_ranges NULL only cubics_px is written (projection only). */
CS_API int cs_project_cubics(const float *cubics_norm, const float *stroke_widths,
                      const float *support_radii, float *cubics_px, int32_t *tile_ranges,
                      int32_t *num_tiles_hit, int64_t num_curves, int32_t img_height,
                      int32_t img_width, int32_t block_x, int32_t block_y, float aabb_pad,
                      int32_t aniso, void *stream);

/* Uniform S-point Bernstein flattening of each cubic into S-1 straight edges.
 * basis: [4, S] cubic Bernstein weights at linspace(0, 1, S).
 * Replaces _flatten_cubics_to_edges (bernstein), cubic_splatting.py:1709-1728.
 * cubics_px: [n, 4, 2] -> edges_px: [n*(S-1), 2, 2]. */
CS_API int cs_flatten_bernstein(const float *cubics_px, const float *basis, float *edges_px,
                         int64_t num_segments, int32_t samples, void *stream);

/* Adaptive de Casteljau flattening (flatten_method "de_casteljau"): each
 * cubic is split at t = 1/2 until its inner control points lie within tol_px
 * (floored at 1e-4) of its chord, at most max_depth = ceil(log2(S - 1)) times;
 * each leaf becomes one edge (its first and last control points), ordered by
 * segment then t.  Outputs: edges_px [E, 2, 2], segment_edge_offsets [n + 1]
 * and (optional, from prim_seg_offsets [P + 1]) prim_edge_offsets [P + 1] CSR
 * offsets, edge_t_starts / edge_t_ends [E] leaf parameter intervals.  E is at
 * most n << max_depth (cs_de_casteljau_edge_capacity); the buffers hold that
 * many edges and E = segment_edge_offsets[n].  Works on the device without a
 * host synchronisation; status (device int, may be NULL) receives
 * CS_ERR_CAPACITY if edge_capacity is too small for the leaves written, and
 * CS_ERR_ARG for segment offsets out of range.
 * Replaces the de_casteljau branch of _flatten_cubics_to_edges,
 * cubic_splatting.py:1729-1832, with cubic_adaptive_flatness_flags_kernel
 * (:1863-1957) and cubic_split_half_kernel (:1960-2068). */
CS_API int32_t cs_de_casteljau_max_depth(int32_t samples);
CS_API int64_t cs_de_casteljau_edge_capacity(int64_t num_segments, int32_t samples);
CS_API int cs_flatten_de_casteljau(const float *cubics_px, const int32_t *prim_seg_offsets,
                                   int64_t num_segments, int64_t num_primitives,
                                   int32_t samples, float tol_px, float *edges_px,
                                   int32_t *prim_edge_offsets, int32_t *segment_edge_offsets,
                                   float *edge_t_starts, float *edge_t_ends,
                                   int64_t edge_capacity, int32_t *status, void *stream);

/* The two steps of the adaptive flatten on their own: per-cubic flatness flag
 * (1 = inner control points within tol_px, floored at 1e-4, of the chord; all
 * 1 with force_flat) and the midpoint split into left / right halves, each
 * [n, 4, 2].  Replace cubic_adaptive_flatness_flags_kernel and
 * cubic_split_half_kernel, cubic_splatting.py:1863-2068. */
CS_API int cs_cubic_flatness_flags(const float *cubics, uint8_t *out_flat, int64_t num_cubics,
                                   float tol_px, int32_t force_flat, void *stream);
CS_API int cs_cubic_split_half(const float *cubics, float *left, float *right,
                               int64_t num_cubics, void *stream);

/* Union of segment tile rectangles per primitive (CSR offsets over segments).
 * Replaces primitive_tile_ranges_from_segment_ranges_kernel,
 * cubic_splatting.py:2071-2137. */
CS_API int cs_primitive_tile_ranges(const int32_t *seg_tile_ranges, const int32_t *prim_seg_offsets,
                             int32_t *prim_tile_ranges, int32_t *num_tiles_hit,
                             int64_t num_primitives, int32_t tile_bound_x, int32_t tile_bound_y,
                             void *stream);

/* Intersect keys (tile << 32 | sortable depth bits) and primitive ids,
 * primitive-major and row-major over each primitive's tile rectangle;
 * cum_tiles_hit is the inclusive prefix sum of num_tiles_hit.
 * Replaces map_cubic_to_intersects_kernel, cubic_splatting.py:750-819. */
CS_API int cs_map_cubic_to_intersects(const int32_t *tile_ranges, const float *depths,
                               const int32_t *cum_tiles_hit, int64_t *isect_ids,
                               int32_t *prim_ids, int64_t num_primitives, int32_t tile_bound_x,
                               void *stream);

/* Per-tile [start, end) of sorted keys; tile_bins [num_tiles, 2] is zeroed
 * first, so empty tiles read [0, 0].
 * Replaces get_tile_bin_edges_kernel, tile_bins.py:10-60 (compact=True). */
CS_API int cs_tile_bin_edges(const int64_t *isect_ids_sorted, int64_t num_intersects,
                      int32_t *tile_bins, int64_t num_tiles, void *stream);

/* ranges[i] = (edge_offsets[pid], edge_offsets[pid + 1]) for pid = prim_ids[i].
 * Replaces _build_fill_isect_edge_ranges, cubic_splatting.py:1849-1860. */
CS_API int cs_isect_edge_ranges(const int32_t *prim_ids_sorted, const int32_t *prim_edge_offsets,
                         int32_t *isect_edge_ranges, int64_t num_intersects, void *stream);

/* Fused B200 binning, stage 1 of 2: projection + AABB + flattening of every
 * segment, per-primitive tile rectangles, per-tile intersect and edge-slot
 * counts restricted to tile rows [tile_row_begin, tile_row_end), and their
 * exclusive scans: tile_bins [T, 2] (intersect [start, end)) and tile_dlist
 * [T, 2] (first staged record of the tile, per-strip record capacity c: the
 * tile's 4 strip lists start at first + s c).  counters is a device int32[4]:
 * [0] intersect total, [1] status, [2] staged-record bound, [3] unused.
 * stroke_widths may be NULL (fill mode: zero stroke width); aniso selects the
 * chord-anisotropic padding of the reference's aniso_intersects.  If a total
 * exceeds its capacity (pass INT64_MAX to size buffers from the counters
 * afterwards) every tile range is written empty and counters[1] is set to
 * CS_ERR_CAPACITY, so no later kernel reads past the caller's buffers.
 * Offsets that do not start at 0, end at num_segments and increase set
 * counters[1] to CS_ERR_ARG (the primitive is treated as empty).  With ring
 * (closed paths as ring points [P, 3G, 2] in pixels, G = ring_segs_per_path)
 * the control points are read from the ring, normalised exactly as
 * cs_ring_to_cubics does, and cubics_norm may be NULL.  For a band
 * (rows other than the whole grid), tiles outside it read as empty and the
 * edges of primitives whose tile rows miss the band are not written.
 * prim_edge_offsets [P + 1] (may be NULL) selects pre-flattened edges: edges_px
 * then holds edges already written (e.g. by cs_flatten_de_casteljau) with
 * these CSR offsets, is only read by later stages, and the edge-slot counts
 * use each primitive's own edge count.  Otherwise prim_edge_offsets_out [P + 1]
 * (may be NULL) receives the uniform flatten's offsets offs * (S - 1).
 * With cs_bin_sort this replaces project (K3) + flatten + K4 + cumsum + K5 +
 * torch.sort + K6 of _CubicFillSplatFunction.forward, cubic_splatting.py:2815-2908.
 * Workspace: cs_bin_workspace_size(num_tiles) bytes, zeroed before its first
 * use; every call leaves it zeroed again (cs_bin_sort reads the cursors it
 * holds, so a call's cs_bin_sort must follow it before the next cs_bin_count
 * on the same workspace). */
CS_API size_t cs_bin_workspace_size(int64_t num_tiles);
CS_API int cs_bin_count(const float *cubics_norm, const int32_t *prim_seg_offsets,
                 const float *aa_widths, const float *stroke_widths, const float *basis,
                 float *cubics_px, float *edges_px, const int32_t *prim_edge_offsets,
                 int32_t *prim_edge_offsets_out, int32_t *prim_tile_ranges, int32_t *num_tiles_hit, int32_t *tile_bins,
                 int32_t *tile_dlist, int32_t *counters, void *workspace, int64_t num_primitives,
                 int64_t num_segments, int64_t isect_capacity, int64_t dlist_capacity,
                 int32_t samples, int32_t img_height, int32_t img_width, int32_t tile_row_begin,
                 int32_t tile_row_end, float aabb_pad, int32_t aniso, const float *ring,
                 int32_t ring_segs_per_path, void *stream);

/* Fused B200 binning, stage 2 of 2: scatter each (primitive, tile) pair into
 * its tile's range and sort every tile's pairs by (depth key, primitive id),
 * the order of a stable sort of the reference's keys.  Writes prim_ids_sorted
 * and isect_ids_sorted (reference key format; also used as scratch) [capacity].
 * When imeta is not NULL the same per-tile pass also stages the raster input.
 * A tile is rasterised as 4 strips of 4 pixel rows ("units", unit id =
 * 4 * (band tile index) + strip).  Per intersect: a 48-byte record (imeta
 * [I]), per strip its (first record, record count) in that strip's list
 * (isect_strips [I, 4, 2]) and, in fill mode, packed per-row winding offsets
 * (rowoff [I, 16]); per strip the near-edge records (dlist [dlist_capacity]
 * of 32 bytes, at the offsets tile_dlist gives).  unit_order (may be NULL;
 * cs_unit_lists_size(band tiles) bytes) receives the band's units in 64
 * buckets of their staged work, heaviest first, which the raster entry
 * points use as their dispatch order.  stroke_widths non-NULL selects stroke
 * mode (fill_rules, rowoff unused).  Work stops at the device when counters
 * report an overflow. */
CS_API size_t cs_unit_lists_size(int64_t num_tiles);
CS_API int cs_bin_sort(const int32_t *prim_tile_ranges, const float *depths,
                const int32_t *tile_bins, int32_t *prim_ids_sorted, int64_t *isect_ids_sorted,
                int32_t *counters, void *workspace, int64_t num_primitives,
                int64_t isect_capacity, int32_t img_height, int32_t img_width,
                int32_t tile_row_begin, int32_t tile_row_end, const float *edges_px,
                const int32_t *prim_edge_offsets, const float *colors, const float *opacities,
                const float *inv_sigma2s, const int32_t *fill_rules, const float *stroke_widths,
                int32_t *tile_dlist, void *imeta, int32_t *rowoff, int32_t *isect_strips,
                void *dlist, int64_t dlist_capacity, int32_t *unit_order, void *stream);

/* Staging of a reference-format sorted intersect list (primitive_ids_sorted,
 * tile_bins and isect_edge_ranges [I, 2] or prim_edge_offsets [P + 1]) into
 * the raster input described for cs_bin_sort; used by the per-stage API.
 * counters: device int32[4] as for cs_bin_count ([2] receives the record
 * bound; CS_ERR_CAPACITY in [1] if it exceeds dlist_capacity).
 * Workspace: cs_stage_workspace_size(num_tiles). */
CS_API size_t cs_stage_workspace_size(int64_t num_tiles);
CS_API int cs_tile_stage(const int32_t *prim_ids_sorted, const int32_t *tile_bins,
                  const float *edges_px, const int32_t *isect_edge_ranges,
                  const int32_t *prim_edge_offsets, const float *colors, const float *opacities,
                  const float *inv_sigma2s, const int32_t *fill_rules, const float *stroke_widths,
                  int32_t *tile_dlist, void *imeta, int32_t *rowoff, int32_t *isect_strips,
                  void *dlist, int32_t *unit_order, int32_t *counters, void *workspace,
                  int64_t dlist_capacity, int32_t img_height, int32_t img_width, void *stream);

/* --------------------------------------------------------------------------
 * Rasterisation (one warp per 4 x 16-pixel strip, front-to-back compositing)
 * ------------------------------------------------------------------------ */

/* Closed-fill forward: per pixel, winding number / crossing parity and the
 * minimum distance to the primitive's polyline, sigmoid soft coverage, then
 * front-to-back alpha compositing with early termination.  Input is the
 * staged data of cs_bin_sort / cs_tile_stage (tile_dlist, imeta,
 * isect_strips, rowoff, dlist; unit_order may be NULL).  unit_order_bwd (may
 * be NULL; cs_unit_lists_size bytes) receives the same units bucketed by the
 * work this launch measured, the better dispatch order for the backward.
 * visit_lists (may be NULL; cs_visit_lists_size bytes) receives, per 4-row
 * strip, the ids of the intersects that composited at least one of its
 * pixels; given to the backward, it walks only those (exactly the ones that
 * can carry a gradient) instead of every intersect of the tile.
 * visit_winners (may be NULL; cs_visit_winners_size bytes; used only with
 * visit_lists) receives, per listed visit and lane, each of the lane's two
 * pixels' closest record (relative to the intersect's first, 7 bits) and
 * inside state (1 bit); given to the backward, it evaluates only that record
 * per pixel instead of walking all of the intersect's records.
 * out_chw_clamped
 * [3, H, W] (may be NULL) also receives clamp(out, 0, 1) channel-major, the
 * image the training loss sees (the reference does torch.clamp + permute,
 * manbo/gaussian_trace/render.py:1309-1310).  status (device int, may be NULL)
 * receives CS_ERR_TIMEOUT if a bounded wait gave up.  When target_chw
 * [3, H, W] is given the same launch also computes the MSE loss of the
 * clamped image: loss_out[0] = sum of squared differences over the band,
 * loss_out[1] = that / (3 H W), reduced in a fixed order.  workspace:
 * cs_raster_workspace_size(num_tiles) bytes, zeroed before its first use; the
 * launch leaves it ready for the next one (launches sharing a workspace must
 * be ordered on one stream).  Tile rows outside [tile_row_begin, tile_row_end)
 * are not touched.
 * Replaces rasterize_cubic_fill_forward_kernel, cubic_splatting.py:918-1194,
 * and (with target_chw) mse_partial_sum_kernel + reduce_sum_partial_kernel,
 * manbo/ops/metric.py:18-163. */
CS_API size_t cs_raster_workspace_size(int64_t num_tiles);
CS_API size_t cs_visit_lists_size(int64_t isect_capacity, int64_t num_tiles);
CS_API size_t cs_visit_winners_size(int64_t isect_capacity, int64_t num_tiles);
CS_API int cs_fill_forward(const int32_t *prim_ids_sorted, const int32_t *tile_bins,
                    const int32_t *tile_dlist, const void *imeta, const int32_t *isect_strips,
                    const int32_t *rowoff, const void *dlist, const int32_t *unit_order,
                    int32_t *unit_order_bwd, int32_t *visit_lists, uint16_t *visit_winners,
                    const float *background, float *out_img,
                    float *final_Ts, int32_t *final_idx, float *out_chw_clamped,
                    const float *target_chw, float *loss_out, int32_t *status,
                    void *workspace, int32_t img_height, int32_t img_width,
                    int32_t tile_row_begin, int32_t tile_row_end, void *stream);

/* Closed-fill backward: reverse compositing from final_idx, gradients of the
 * colours, opacities, 1/sigma^2 and edge endpoints (closest edge only).
 * Outputs are accumulated (+=) into caller-zeroed buffers.  curve_contrib_rgb
 * [P, 3] and curve_isect_contrib [I] are optional (NULL = not collected).
 * v_output [H, W, 3] is the upstream image gradient; when it is NULL the MSE
 * gradient is computed in the kernel instead: v = scale * (clamp(out) - target)
 * masked to 0 <= out <= 1, with out_img [H, W, 3], target_chw [3, H, W] and
 * *mse_scale (device scalar, e.g. 2/N * dLoss).  v_opacities and
 * v_inv_sigma2s may be NULL (not accumulated).  workspace as for the forward.
 * visit_lists (may be NULL: every intersect up to final_idx is walked) is the
 * forward's output of the same frame; a list that does not fit the tile bins
 * sets CS_ERR_ARG in status and its strip is skipped.  visit_winners (may be
 * NULL) likewise; a code past its intersect's records sets CS_ERR_ARG.
 * Replaces rasterize_cubic_fill_backward_kernel, cubic_splatting.py:1197-1651. */
CS_API int cs_fill_backward(const int32_t *prim_ids_sorted, const int32_t *tile_bins,
                     const int32_t *tile_dlist, const void *imeta, const int32_t *isect_strips,
                     const int32_t *rowoff, const void *dlist, const int32_t *unit_order,
                     const int32_t *visit_lists, const uint16_t *visit_winners,
                     const float *background, const float *final_Ts, const int32_t *final_idx,
                     const float *v_output, const float *out_img, const float *target_chw,
                     const float *mse_scale, float *v_edges, float *v_colors,
                     float *v_opacities, float *v_inv_sigma2s, float *curve_contrib_rgb,
                     float *curve_isect_contrib, int32_t *status, void *workspace,
                     int32_t img_height, int32_t img_width, int32_t tile_row_begin,
                     int32_t tile_row_end, void *stream);

/* Stroke forward: coverage exp(-1/2 max(0, d - w/2)^2 / sigma^2).
 * Replaces rasterize_cubic_polyline_forward_kernel,
 * cubic_polyline_splatting.py:33-249. */
CS_API int cs_stroke_forward(const int32_t *prim_ids_sorted, const int32_t *tile_bins,
                      const int32_t *tile_dlist, const void *imeta, const int32_t *isect_strips,
                      const void *dlist, const int32_t *unit_order, int32_t *unit_order_bwd,
                      int32_t *visit_lists, uint16_t *visit_winners, const float *background,
                      float *out_img, float *final_Ts,
                      int32_t *final_idx, float *out_chw_clamped, const float *target_chw,
                      float *loss_out,
                      int32_t *status, void *workspace, int32_t img_height, int32_t img_width,
                      int32_t tile_row_begin, int32_t tile_row_end, void *stream);

/* Stroke backward (adds d/d stroke width).
 * Replaces rasterize_cubic_polyline_backward_kernel,
 * cubic_polyline_splatting.py:252-660. */
CS_API int cs_stroke_backward(const int32_t *prim_ids_sorted, const int32_t *tile_bins,
                       const int32_t *tile_dlist, const void *imeta, const int32_t *isect_strips,
                       const void *dlist, const int32_t *unit_order,
                       const int32_t *visit_lists, const uint16_t *visit_winners,
                       const float *background, const float *final_Ts, const int32_t *final_idx,
                       const float *v_output,
                       const float *out_img, const float *target_chw, const float *mse_scale,
                       float *v_edges, float *v_colors, float *v_opacities,
                       float *v_stroke_widths, float *v_inv_sigma2s, float *curve_contrib_rgb,
                       float *curve_isect_contrib, int32_t *status, void *workspace,
                       int32_t img_height, int32_t img_width, int32_t tile_row_begin,
                       int32_t tile_row_end, void *stream);

/* Edge endpoint gradients -> cubic control-point gradients with the Bernstein
 * weights at t = e / (S-1); optional scale (sx, sy) applied to the result
 * (pass 1, 1 for pixel space, W/2, H/2 for normalised space).
 * Replaces _accumulate_edge_grads_to_cubics_kernel, cubic_splatting.py:2308-2396
 * and the epilogue scaling of cubic_splatting.py:3096-3100. */
CS_API int cs_edge_grads_to_cubics(const float *v_edges, float *v_cubics, int64_t num_segments,
                            int32_t edges_per_segment, float scale_x, float scale_y,
                            void *stream);

/* Edge gradients of a de Casteljau flattening -> cubic control-point
 * gradients: v_P_k = sum over the segment's edges of gs B_k(t0) + ge B_k(t1),
 * then the optional per-axis scale.  segment_edge_offsets [n + 1] and
 * edge_t_starts / edge_t_ends as written by cs_flatten_de_casteljau.
 * Replaces _accumulate_edge_grads_to_cubics_csr_kernel,
 * cubic_splatting.py:2399-2487. */
CS_API int cs_edge_grads_to_cubics_csr(const float *v_edges, const float *edge_t_starts,
                                       const float *edge_t_ends,
                                       const int32_t *segment_edge_offsets, float *v_cubics,
                                       int64_t num_segments, float scale_x, float scale_y,
                                       void *stream);

/* Anti-aliasing widths of the renderer: widths_clamped = clamp(aa, min=1e-4)
 * and inv_sigma2s = 1 / clamp(w^2, min=1e-6) (cubic_splatting.py:2820-2821);
 * backward v_aa = -2 v_inv / clamp(w^3, min=1e-12) (:3101-3104), and with
 * aa_widths (may be NULL) also the entry clamp's backward: 0 where
 * !(aa >= 1e-4).  [n] each; NaN propagates as through torch.clamp. */
CS_API int cs_aa_widths_forward(const float *aa_widths, float *widths_clamped,
                                float *inv_sigma2s, int64_t n, void *stream);
CS_API int cs_aa_widths_backward(const float *aa_widths, const float *widths_clamped,
                                 const float *v_inv_sigma2s, float *v_aa_widths, int64_t n,
                                 void *stream);

/* Ring parameterisation of closed paths (the B200 training step's
 * parameters): ring [P, 3G, 2] pixel-space points; segment k of a path is
 * (r[3k], r[3k+1], r[3k+2], r[3k+3 mod 3G]).  cubics_norm [P*G, 4, 2] =
 * point / (W/2, H/2) - 1, the normalisation the reference's renderer inverts
 * (cubic_splatting.py:588-595). */
CS_API int cs_ring_to_cubics(const float *ring, float *cubics_norm, int64_t num_paths,
                      int32_t segs_per_path, int32_t img_height, int32_t img_width, void *stream);

/* Edge endpoint gradients [P*G*E, 2, 2] -> ring point gradients [P, 3G, 2]
 * (written, not accumulated): the per-segment Bernstein accumulation of
 * cs_edge_grads_to_cubics in normalised space, then the derivative of the
 * normalisation, summed over the control points that share a ring point.
 * clear_edges != 0 zeroes v_edges after reading it.  G <= 128.  With
 * prim_tile_ranges [P, 4] (may be NULL) a path whose tile rectangle misses the
 * tile rows [tile_row_begin, tile_row_end) gets zero gradients without its
 * edges being read (a band renders only its rows). */
CS_API int cs_edge_grads_to_ring(float *v_edges, float *v_ring, int64_t num_paths,
                          int32_t segs_per_path, int32_t edges_per_segment, int32_t img_height,
                          int32_t img_width, int32_t clear_edges,
                          const int32_t *prim_tile_ranges, int32_t tile_row_begin,
                          int32_t tile_row_end, void *stream);

/* Adam step over one flat fp32 parameter buffer, elements [0, n_first) with
 * lr_first and the rest with lr_rest; step (device int32) holds the number of
 * steps taken and is advanced on the device.  clear_grads != 0 zeroes the
 * gradient after use.  Workspace: cs_adam_workspace_size() bytes, zeroed once. */
CS_API size_t cs_adam_workspace_size(void);
CS_API int cs_adam_step(float *params, float *grads, float *exp_avg, float *exp_avg_sq, int64_t n,
                 int64_t n_first, float lr_first, float lr_rest, float beta1, float beta2,
                 float eps, int32_t *step, void *workspace, int32_t clear_grads, void *stream);

/* --------------------------------------------------------------------------
 * Closed control polygon -> ring of piecewise-Hermite cubics
 * ------------------------------------------------------------------------ */

/* control_points [N, K, 2] -> segments [N*2*subdiv, 4, 2]; basis [subdiv+1, Kb],
 * deriv_basis [subdiv+1, Kb-1], dt [subdiv] with Kb = (K+2)/2.
 * Replaces closed_cubic_fill_segments_forward_kernel, cubic_splatting.py:137-268. */
CS_API int cs_ring_segments_forward(const float *control_points, const float *basis,
                             const float *deriv_basis, const float *dt, float *segments,
                             int64_t num_curves, int32_t k, int32_t subdiv, void *stream);

/* Adjoint of the above, accumulated (+=) into grad_control_points.
 * Replaces closed_cubic_fill_segments_backward_kernel, cubic_splatting.py:271-397. */
CS_API int cs_ring_segments_backward(const float *grad_segments, const float *basis,
                              const float *deriv_basis, const float *dt,
                              float *grad_control_points, int64_t num_curves, int32_t k,
                              int32_t subdiv, void *stream);

/* --------------------------------------------------------------------------
 * Metrics
 * ------------------------------------------------------------------------ */

/* Sum of squared differences in one launch (block partials, last block
 * reduces them in a fixed order).  Writes *out_sse and *out_mse = sse / n
 * (device scalars; either may be NULL).  Workspace: cs_mse_workspace_size(n).
 * Replaces mse_partial_sum_kernel + the reduce_sum_partial_kernel loop,
 * manbo/ops/metric.py:18-163, 344-382 and _mse_forward_tilelang,
 * manbo/metric.py:102-130. */
CS_API size_t cs_mse_workspace_size(int64_t n);
CS_API int cs_mse_forward(const float *x, const float *y, int64_t n, float *out_sse, float *out_mse,
                   void *workspace, void *stream);

/* grad = s * (lhs - rhs) with s = (*scale) * factor, scale read on the
 * device (no host sync), or s = factor when scale is NULL.
 * Replaces mse_backward_diff_kernel, manbo/ops/metric.py:166-202. */
CS_API int cs_mse_backward(const float *lhs, const float *rhs, const float *scale, float factor,
                           float *grad, int64_t n, void *stream);

/* SSIM with a separable Gaussian window g [win] (win odd, win2d = outer(g, g)),
 * valid-window semantics, per plane (N*C planes of H x W).  Writes the mean
 * SSIM of every plane to plane_means [planes] and, when ssim_map is not NULL,
 * the map [planes, H-win+1, W-win+1].  One launch; per-block sums are
 * reduced by the last block.  win <= 15.
 * Workspace: cs_ssim_workspace_size(planes, h, w, win) bytes, zeroed once.
 * Replaces ssim_map_kernel + the mean of manbo/metric.py:215-273
 * (manbo/ops/metric.py:205-341). */
CS_API size_t cs_ssim_workspace_size(int64_t planes, int32_t h, int32_t w, int32_t win);
CS_API int cs_ssim(const float *x, const float *y, const float *gauss, int64_t planes, int32_t h,
            int32_t w, int32_t win, float c1, float c2, float *plane_means, float *ssim_map,
            void *workspace, void *stream);

/* Largest planes * ceil((h-win+1)/32) * ceil((w-win+1)/32) that
 * cs_ssim_noalloc accepts: e.g. 3 planes of up to about 4700 x 4700 pixels. */
#define CS_SSIM_NOALLOC_MAX_PARTIALS 65536

/* cs_ssim without a workspace argument, for callers that cannot hand the
 * library device memory: a plain C host with no device allocator or memory
 * pool of its own, or a host that has reserved its whole memory budget up
 * front and must not call cudaMalloc/cudaFree (which also synchronise the
 * device) once its loop runs.  This entry point has no counterpart in the
 * reference; it computes exactly what cs_ssim computes, with the same
 * arguments minus the workspace.
 *
 * Its scratch (a 256-byte completion ticket and
 * CS_SSIM_NOALLOC_MAX_PARTIALS per-block partial sums, 256 KB + 256 B) is a
 * fixed array in the library's device memory, one per GPU.  The first call on
 * each device looks up that array's address (cudaGetSymbolAddress, with the
 * calling thread's current device); make that first call on each device
 * before any stream capture.  Every call clears the ticket with
 * cudaMemsetAsync on `stream` before its launch, so nothing needs to be
 * zeroed by the caller.  Nothing is allocated or freed, on the host or the
 * device.
 *
 * Limits: planes * tiles above CS_SSIM_NOALLOC_MAX_PARTIALS returns
 * CS_ERR_CAPACITY without launching; devices with ordinal >= 64 return
 * CS_ERR_UNSUPPORTED.  Because the scratch is shared, two calls on the same
 * device whose executions overlap (different streams with no ordering between
 * them, or several host threads) race on it and give wrong results; order
 * them on one stream, or use cs_ssim with a workspace per stream.  The
 * looked-up address is kept for the life of the process: cudaDeviceReset (or
 * anything else that destroys the device's primary context) reloads the
 * library's device memory, possibly elsewhere, so a process that resets a
 * device must not call cs_ssim_noalloc on that device afterwards. */
CS_API int cs_ssim_noalloc(const float *x, const float *y, const float *gauss, int64_t planes,
            int32_t h, int32_t w, int32_t win, float c1, float c2, float *plane_means,
            float *ssim_map, void *stream);

/* --------------------------------------------------------------------------
 * Optimiser
 * ------------------------------------------------------------------------ */

/* One Adan step in place from a gradient, element by element over numel
 * float32 values: m (exp_avg), n (exp_avg_sq), d (exp_avg_diff) and the
 * negated previous gradient are updated, then the parameter, with decoupled
 * (no_prox != 0) or proximal weight decay; the gradient is scaled by
 * clip_global_grad_norm first and step == 1 starts the gradient difference at
 * zero.  Arguments as the reference kernel's, in its order.
 * Replaces adan_step_from_grad_kernel, manbo/ops/optim.py:8-106. */
CS_API int cs_adan_step(float *param, const float *grad, float *exp_avg, float *exp_avg_sq,
                 float *exp_avg_diff, float *neg_pre_grad, int64_t numel, int32_t step,
                 float beta1, float beta2, float beta3, float bias_correction1,
                 float bias_correction2, float bias_correction3_sqrt, float lr,
                 float weight_decay, float eps, float clip_global_grad_norm, int32_t no_prox,
                 void *stream);

/* --------------------------------------------------------------------------
 * Regularisation loss of the curve model
 * (manbo/regularization.py:65-250, manbo/ops/regularization.py)
 *
 * L = lambda_proj / N * sum phi(alpha)  +  opacity_weight * mean |sigmoid(op) - 1|
 *   + [closed] masked second-difference energy / (N * ceil(2M / stride))
 *   + [closed] joint hinge sum / (N * ceil(K / boundary_degree) * 2)
 *
 * control_points [N, K, 2]; opacity [num_opacity]; xyz [N, 2, M, 2] sampled
 * paths (closed only, M = points_per_side).  Open mode projects the middle
 * points onto p[0] -> p[K-1]; closed mode onto p[0] -> p[split_idx] (the
 * shape degree + 1) and skips p[split_idx].  curvature_cos_thresh is
 * cos(angle threshold).  N >= 1.
 * ------------------------------------------------------------------------ */
/* Workspace: cs_regularization_workspace_size() bytes, zeroed once. */
CS_API size_t cs_regularization_workspace_size(void);
/* The scalar loss into *loss (device). */
CS_API int cs_regularization_forward(const float *control_points, const float *opacity,
                              const float *xyz, int64_t num_curves, int64_t num_ctrl,
                              int64_t num_opacity, int64_t points_per_side, int32_t closed,
                              int32_t split_idx, int32_t boundary_degree, float boundary_bound,
                              int32_t curvature_stride, float curvature_cos_thresh,
                              float lambda_proj, float opacity_weight, float *loss,
                              void *workspace, void *stream);
/* Gradients times *grad_output (device scalar; NULL = 1): grad_control_points
 * [N, K, 2] and grad_xyz [N, 2, M, 2] are overwritten (zeroed, then the terms'
 * atomics), grad_opacity [num_opacity] written; any output may be NULL. */
CS_API int cs_regularization_backward(const float *control_points, const float *opacity,
                               const float *xyz, int64_t num_curves, int64_t num_ctrl,
                               int64_t num_opacity, int64_t points_per_side, int32_t closed,
                               int32_t split_idx, int32_t boundary_degree, float boundary_bound,
                               int32_t curvature_stride, float curvature_cos_thresh,
                               float lambda_proj, float opacity_weight, const float *grad_output,
                               float *grad_control_points, float *grad_opacity, float *grad_xyz,
                               void *stream);

/* --------------------------------------------------------------------------
 * 4-connected component labelling of a uint8 mask [H, W]
 * (manbo/ops/connected_components.py:98-236)
 *
 * cs_ccl_labels_4: raw labels [H, W] int32, each component labelled with its
 * smallest linear index + 1, background 0 (the reference's relaxation result).
 * cs_ccl_compact_4 (after it, on its labels, same workspace): components
 * renumbered 1.. in raster order of their first pixel, their count into
 * *num_components (device).  cs_ccl_stats_4 (after that, same workspace):
 * stats [n, 5] int32 (x, y, width, height, area) and centers [n, 2] float32
 * (mean x, mean y) of the n = num_components components.  status (device
 * int32) records a union that exceeded its retry bound or a label outside
 * [0, H*W].  H * W < 2^31 - 1.
 * ------------------------------------------------------------------------ */
CS_API size_t cs_ccl_workspace_size(int64_t num_pixels);
CS_API int cs_ccl_labels_4(const uint8_t *mask, int32_t height, int32_t width, int32_t *labels,
                    int32_t *status, void *workspace, void *stream);
CS_API int cs_ccl_compact_4(const int32_t *labels, int32_t height, int32_t width,
                     int32_t *labels_compact, int32_t *num_components, int32_t *status,
                     void *workspace, void *stream);
CS_API int cs_ccl_stats_4(int32_t height, int32_t width, int32_t num_components, int32_t *stats,
                   float *centers, void *workspace, void *stream);

/* --------------------------------------------------------------------------
 * Peer-memory exchange for one image split across GPUs in tile-row bands
 * (no counterpart in the reference, which renders an image on one GPU; these
 * replace a library all-reduce and all-gather in the band-parallel step)
 *
 * Pointer arrays (flag_ptrs, grad_ptrs) are device arrays of `world` device
 * addresses, entry q pointing into rank q's buffer as mapped in the calling
 * process (e.g. symmetric memory).  Flag words are uint32 step numbers, laid
 * out [slot][world]: word slot * world + q of a rank's array is written by
 * rank q.  `epoch` is a device int32 (the optimiser's completed-step count);
 * a signal stores *epoch + epoch_add, a wait waits for at least that value.
 * Waits poll at most spin_limit times and then record CS_ERR_TIMEOUT in
 * *status and skip their work; they never hang.  Kernels that wait on another
 * rank must run on different GPUs at the same time (one process per GPU).
 *
 * cs_peer_signal: after the stream's earlier work, store the step into word
 * slot * world + rank of every rank's flags (or only of rank only_peer >= 0),
 * with release semantics at system scope.
 * cs_peer_wait_copy: wait for rank from_rank's word in this rank's flags, then
 * (src != NULL) copy `planes` blocks of plane_elems floats from src (plane
 * stride src_plane_stride, e.g. a peer's buffer) to dst (dst_plane_stride).
 * cs_allreduce_adam: wait for every rank's word in slot flag_slot, then
 * params[0:n) take one Adam step (two learning rates: lr_first below n_first)
 * with the gradient sum over ranks of grad_ptrs[q][0:n) (summed in rank order,
 * so every rank computes identical parameters); the n_tail values after the
 * gradients are summed into tail_out; clear_buf[0:n + n_tail) is zeroed (this
 * rank's gradient buffer of the next step); *step is incremented.  With n a
 * multiple of 4 every buffer must be 16-byte aligned to take the vector path.
 * ------------------------------------------------------------------------ */
CS_API size_t cs_allreduce_adam_workspace_size(void);
CS_API int cs_peer_signal(const uint64_t *flag_ptrs, int32_t rank, int32_t world, int32_t slot,
                          const int32_t *epoch, int32_t epoch_add, int32_t only_peer,
                          void *stream);
CS_API int cs_peer_wait_copy(const uint32_t *flags, int32_t slot, int32_t world,
                             int32_t from_rank, const int32_t *epoch, int32_t epoch_add,
                             int64_t spin_limit, int32_t *status, const float *src,
                             int64_t src_plane_stride, float *dst, int64_t dst_plane_stride,
                             int64_t plane_elems, int32_t planes, void *stream);
CS_API int cs_allreduce_adam(const uint64_t *grad_ptrs, int32_t world, float *params,
                             float *exp_avg, float *exp_avg_sq, int64_t n, int64_t n_first,
                             int32_t n_tail, float *tail_out, float *clear_buf, float lr_first,
                             float lr_rest, float beta1, float beta2, float eps, int32_t *step,
                             const uint32_t *flags, int32_t flag_slot, int64_t spin_limit,
                             int32_t *status, void *workspace, void *stream);

/* --------------------------------------------------------------------------
 * Graph-capture helpers (no counterpart in the reference, whose renderer reads
 * intersect counts back to the host every frame and cannot be captured)
 *
 * cs_stream_is_capturing: 1 if the stream is capturing a CUDA graph, 0 if not,
 * -1 if the query failed.  cs_poison_on_status: when *status (device int32) is
 * not CS_OK, every element of data [n] becomes NaN; a frame captured with a
 * fixed intersect capacity uses it so that an overflow cannot pass unnoticed.
 * ------------------------------------------------------------------------ */
CS_API int cs_stream_is_capturing(void *stream);
CS_API int cs_poison_on_status(const int32_t *status, float *data, int64_t n, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CUBICSPLAT_B200_H */
