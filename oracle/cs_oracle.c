/*
 * CPU oracle for the CubicSplat render/optimise hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain C and IEEE float32,
 * the algorithm of the reference's TileLang kernels so that the CUDA product
 * can be checked against it.  Only tests, the smoke check and the CPU-baseline
 * leg of the benchmark may load it; the product never calls it.
 *
 * Arithmetic rules: compile with -ffp-contract=off (no implicit FMA); every
 * expression is evaluated in the order the reference writes it, and the one
 * fused multiply-add the reference's compiled projection is known to use
 * (pixel = n * W/2 + W/2, pinned bit for bit by the golden vectors) is written
 * out with fmaf.  The one deliberate departure is exp(): the reference uses the fast-math hardware
 * exponential, this file uses cso_expf below (Cody-Waite reduction + degree-7
 * Taylor polynomial), the same published method the CUDA kernels use, so the
 * two agree bit for bit.  The reference's fast-math ulps are therefore not
 * reproduced; parity against the reference itself is carried by tolerances on
 * golden vectors produced by the reference.
 *
 * Reference files are cited by path inside the reference project.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ALPHA_CAP 0.999f
#define ALPHA_MIN ((float)(1.0 / 255.0))
#define TRANS_STOP 1e-4f
#define EPS_F 1e-6f

static inline float fminf_(float a, float b) { return fminf(a, b); }
static inline float fmaxf_(float a, float b) { return fmaxf(a, b); }
static inline int imin_(int a, int b) { return a < b ? a : b; }
static inline int imax_(int a, int b) { return a > b ? a : b; }

/* float -> int32 truncation with the saturating semantics of cvt.rzi.s32.f32
   (NaN -> 0), which is what the reference's T.Cast(int32, float) compiles to. */
static inline int32_t f2i_trunc_sat(float v) {
    if (v != v) return 0;
    if (v >= 2147483648.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return (int32_t)v;
}

/* exp(x): x = k*ln2 + r with ln2 split into a short high part and a low part
   (Cody & Waite), exp(r) by its Taylor series to degree 7 in Horner form with
   fused multiply-adds, then scaled by 2^k.  |r| <= ln2/2 keeps the truncation
   error below 3e-9 relative.  x below -87 returns 0 (no subnormal results). */
float cso_expf(float x) {
    if (x != x) return x;
    if (x > 88.5f) return INFINITY;
    if (x < -87.0f) return 0.0f;
    const float log2e = 1.44269504088896341f;
    const float ln2_hi = 0.693145751953125f;       /* 0x3F317200: 16 significant bits */
    const float ln2_lo = 1.42860676533018708e-06f; /* ln2 - ln2_hi */
    float kf = rintf(x * log2e);
    float r = fmaf(kf, -ln2_hi, x);
    r = fmaf(kf, -ln2_lo, r);
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return ldexpf(p, (int)kf);
}

/* ------------------------------------------------------------------------ */
/* projection + exact cubic AABB + padded tile rectangle
   (manbo/ops/cubic_splatting.py:588-745, project_cubics_2d_forward_kernel) */

static void axis_extrema(float a, float b, float c, float d, float *mn, float *mx) {
    const float zero = 0.0f, one = 1.0f, two = 2.0f, four = 4.0f, eps = EPS_F;
    float q2 = 3.0f * a;
    float q1 = two * b;
    float q0 = c;
    if ((q2 > eps) | (q2 < -eps)) {
        float disc = q1 * q1 - four * q2 * q0;
        if (disc >= -eps) {
            float sq = sqrtf(fmaxf_(disc, zero));
            float inv2q2 = one / (two * q2);
            float t0 = (-q1 - sq) * inv2q2;
            float t1 = (-q1 + sq) * inv2q2;
            if ((t0 > zero) & (t0 < one)) {
                float v = ((a * t0 + b) * t0 + c) * t0 + d;
                *mn = fminf_(*mn, v);
                *mx = fmaxf_(*mx, v);
            }
            if ((t1 > zero) & (t1 < one)) {
                float v = ((a * t1 + b) * t1 + c) * t1 + d;
                *mn = fminf_(*mn, v);
                *mx = fmaxf_(*mx, v);
            }
        }
    } else if ((q1 > eps) | (q1 < -eps)) {
        float t = -q0 / q1;
        if ((t > zero) & (t < one)) {
            float v = ((a * t + b) * t + c) * t + d;
            *mn = fminf_(*mn, v);
            *mx = fmaxf_(*mx, v);
        }
    }
}

void cso_project_cubics(int64_t num_curves, const float *cubics_norm, const float *stroke_widths,
                        const float *support_radii, int img_h, int img_w, int block_x, int block_y,
                        float aabb_pad, int aniso, float *cubics_px, int32_t *tile_ranges,
                        int32_t *num_tiles_hit) {
    const float half_w = 0.5f * (float)img_w;
    const float half_h = 0.5f * (float)img_h;
    const int tbx = (img_w + block_x - 1) / block_x;
    const int tby = (img_h + block_y - 1) / block_y;
    const float bxf = (float)block_x, byf = (float)block_y;
    for (int64_t g = 0; g < num_curves; ++g) {
        const float *cn = cubics_norm + g * 8;
        float p[8];
        for (int k = 0; k < 4; ++k) {
            /* the reference's n * half + half compiles to one fused multiply-add
               (verified bit for bit against its golden vectors) */
            p[2 * k] = fmaf(cn[2 * k], half_w, half_w);
            p[2 * k + 1] = fmaf(cn[2 * k + 1], half_h, half_h);
        }
        memcpy(cubics_px + g * 8, p, sizeof(p));
        float p0x = p[0], p0y = p[1], p1x = p[2], p1y = p[3], p2x = p[4], p2y = p[5], p3x = p[6], p3y = p[7];
        float ax = -p0x + 3.0f * p1x - 3.0f * p2x + p3x;
        float bx = 3.0f * p0x - 6.0f * p1x + 3.0f * p2x;
        float cx = -3.0f * p0x + 3.0f * p1x;
        float dx = p0x;
        float ay = -p0y + 3.0f * p1y - 3.0f * p2y + p3y;
        float by = 3.0f * p0y - 6.0f * p1y + 3.0f * p2y;
        float cy = -3.0f * p0y + 3.0f * p1y;
        float dy = p0y;
        float min_x = fminf_(p0x, p3x), max_x = fmaxf_(p0x, p3x);
        float min_y = fminf_(p0y, p3y), max_y = fmaxf_(p0y, p3y);
        axis_extrema(ax, bx, cx, dx, &min_x, &max_x);
        axis_extrema(ay, by, cy, dy, &min_y, &max_y);
        float half_sw = fmaxf_(0.0f, stroke_widths[g]) * 0.5f;
        float support = fmaxf_(0.0f, support_radii[g]);
        if (aniso) {
            float chx = p3x - p0x, chy = p3y - p0y;
            float chord2 = chx * chx + chy * chy;
            float inv_chord = 1.0f / sqrtf(fmaxf_(chord2, EPS_F));
            float nx0 = fabsf(chy) * inv_chord;
            float ny0 = fabsf(chx) * inv_chord;
            float nx = fmaxf_(0.20f, nx0), ny = fmaxf_(0.20f, ny0);
            float radial = half_sw + support;
            float pad_x = aabb_pad + radial * nx;
            float pad_y = aabb_pad + radial * ny;
            min_x = min_x - pad_x;
            max_x = max_x + pad_x;
            min_y = min_y - pad_y;
            max_y = max_y + pad_y;
        } else {
            float pad_i = fmaxf_(aabb_pad, support);
            min_x = min_x - half_sw - pad_i;
            min_y = min_y - half_sw - pad_i;
            max_x = max_x + half_sw + pad_i;
            max_y = max_y + half_sw + pad_i;
        }
        int tminx = imin_(imax_(f2i_trunc_sat(min_x / bxf), 0), tbx);
        int tminy = imin_(imax_(f2i_trunc_sat(min_y / byf), 0), tby);
        int tmaxx = imin_(imax_(f2i_trunc_sat(max_x / bxf + 1.0f), 0), tbx);
        int tmaxy = imin_(imax_(f2i_trunc_sat(max_y / byf + 1.0f), 0), tby);
        tile_ranges[g * 4 + 0] = tminx;
        tile_ranges[g * 4 + 1] = tminy;
        tile_ranges[g * 4 + 2] = tmaxx;
        tile_ranges[g * 4 + 3] = tmaxy;
        num_tiles_hit[g] = imax_(0, (tmaxx - tminx) * (tmaxy - tminy));
    }
}

/* Bernstein flatten (manbo/ops/cubic_splatting.py:1709-1719): basis holds
   b0[S], b1[S], b2[S], b3[S] computed by torch exactly as the reference does;
   points are (((c0*b0 + c1*b1) + c2*b2) + c3*b3), edges join consecutive points. */
void cso_flatten_bernstein(int64_t num_segments, int samples, const float *cubics_px,
                           const float *basis, float *edges_px) {
    const int S = samples, E = samples - 1;
    for (int64_t g = 0; g < num_segments; ++g) {
        const float *c = cubics_px + g * 8;
        float prevx = 0.f, prevy = 0.f;
        for (int s = 0; s < S; ++s) {
            float b0 = basis[s], b1 = basis[S + s], b2 = basis[2 * S + s], b3 = basis[3 * S + s];
            float x = c[0] * b0 + c[2] * b1;
            x = x + c[4] * b2;
            x = x + c[6] * b3;
            float y = c[1] * b0 + c[3] * b1;
            y = y + c[5] * b2;
            y = y + c[7] * b3;
            if (s > 0) {
                float *e = edges_px + (g * E + (s - 1)) * 4;
                e[0] = prevx; e[1] = prevy; e[2] = x; e[3] = y;
            }
            prevx = x; prevy = y;
        }
    }
}

/* union of segment tile rectangles per primitive
   (manbo/ops/cubic_splatting.py:2098-2135) */
void cso_prim_tile_ranges(int64_t num_prims, const int32_t *seg_offs, const int32_t *seg_ranges,
                          int tbx, int tby, int32_t *prim_ranges, int32_t *num_hit) {
    for (int64_t p = 0; p < num_prims; ++p) {
        int s0 = seg_offs[p], s1 = seg_offs[p + 1];
        if (s1 > s0) {
            int mnx = tbx, mny = tby, mxx = 0, mxy = 0;
            for (int s = s0; s < s1; ++s) {
                mnx = imin_(mnx, seg_ranges[s * 4 + 0]);
                mny = imin_(mny, seg_ranges[s * 4 + 1]);
                mxx = imax_(mxx, seg_ranges[s * 4 + 2]);
                mxy = imax_(mxy, seg_ranges[s * 4 + 3]);
            }
            prim_ranges[p * 4 + 0] = mnx; prim_ranges[p * 4 + 1] = mny;
            prim_ranges[p * 4 + 2] = mxx; prim_ranges[p * 4 + 3] = mxy;
            num_hit[p] = imax_(0, mxx - mnx) * imax_(0, mxy - mny);
        } else {
            prim_ranges[p * 4 + 0] = prim_ranges[p * 4 + 1] = 0;
            prim_ranges[p * 4 + 2] = prim_ranges[p * 4 + 3] = 0;
            num_hit[p] = 0;
        }
    }
}

/* intersect keys (manbo/ops/cubic_splatting.py:792-817): primitive-major,
   row-major over the primitive's tile rectangle; key = tile<<32 | sortable depth */
int64_t cso_map_intersects(int64_t num_prims, const int32_t *prim_ranges, const int32_t *depth_bits,
                           int tbx, int64_t *isect_ids, int32_t *prim_ids) {
    int64_t out = 0;
    for (int64_t p = 0; p < num_prims; ++p) {
        int x0 = prim_ranges[p * 4 + 0], y0 = prim_ranges[p * 4 + 1];
        int x1 = prim_ranges[p * 4 + 2], y1 = prim_ranges[p * 4 + 3];
        int w = x1 - x0, h = y1 - y0;
        if (w * h <= 0) continue;
        int32_t mask = (depth_bits[p] >> 31) | (int32_t)0x80000000;
        uint64_t dk = (uint64_t)(uint32_t)(depth_bits[p] ^ mask);
        for (int r = 0; r < h; ++r)
            for (int c = 0; c < w; ++c) {
                int64_t tile = (int64_t)(y0 + r) * tbx + x0 + c;
                isect_ids[out] = (int64_t)(((uint64_t)tile << 32) | dk);
                prim_ids[out] = (int32_t)p;
                ++out;
            }
    }
    return out;
}

/* stable ascending sort of (key, value) pairs: merge sort */
void cso_stable_sort_pairs(int64_t n, int64_t *keys, int32_t *vals) {
    if (n <= 1) return;
    int64_t *k2 = (int64_t *)malloc(sizeof(int64_t) * n);
    int32_t *v2 = (int32_t *)malloc(sizeof(int32_t) * n);
    int64_t *ka = keys, *kb = k2;
    int32_t *va = vals, *vb = v2;
    for (int64_t width = 1; width < n; width *= 2) {
        for (int64_t lo = 0; lo < n; lo += 2 * width) {
            int64_t mid = lo + width < n ? lo + width : n;
            int64_t hi = lo + 2 * width < n ? lo + 2 * width : n;
            int64_t i = lo, j = mid, o = lo;
            while (i < mid && j < hi) {
                if (ka[j] < ka[i]) { kb[o] = ka[j]; vb[o++] = va[j++]; }
                else { kb[o] = ka[i]; vb[o++] = va[i++]; }
            }
            while (i < mid) { kb[o] = ka[i]; vb[o++] = va[i++]; }
            while (j < hi) { kb[o] = ka[j]; vb[o++] = va[j++]; }
        }
        int64_t *tk = ka; ka = kb; kb = tk;
        int32_t *tv = va; va = vb; vb = tv;
    }
    if (ka != keys) {
        memcpy(keys, ka, sizeof(int64_t) * n);
        memcpy(vals, va, sizeof(int32_t) * n);
    }
    free(k2);
    free(v2);
}

/* per-tile [start, end) of sorted keys (manbo/ops/tile_bins.py:24-41); rows
   of empty tiles stay zero */
void cso_tile_bins(int64_t n, const int64_t *ids_sorted, int num_tiles, int32_t *tile_bins) {
    memset(tile_bins, 0, sizeof(int32_t) * 2 * (size_t)num_tiles);
    for (int64_t i = 0; i < n; ++i) {
        int cur = (int)(ids_sorted[i] >> 32);
        if (i == 0) tile_bins[cur * 2] = 0;
        if (i == n - 1) tile_bins[cur * 2 + 1] = (int32_t)n;
        if (i > 0) {
            int prev = (int)(ids_sorted[i - 1] >> 32);
            if (prev != cur) {
                tile_bins[prev * 2 + 1] = (int32_t)i;
                tile_bins[cur * 2] = (int32_t)i;
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* per-pixel geometry shared by the fill forward and backward restatements   */

/* Squared distance from the pixel centre (px, py) to edge (x0, y0) + t (vx, vy),
   t in [0, 1]: the reference's proj = (w . v) / max(|v|^2, eps) clamped to
   [0, 1], closest point c = p0 + proj v, d2 = |c - p|^2
   (cubic_splatting.py:1095-1110, :1451-1470).  The dot product, the closest
   point and the squared length are each evaluated with one fused
   multiply-add (fmaf), as the B200 kernels do. */
static inline float edge_d2(float x0, float y0, float vx, float vy, float inv_vv, float px, float py,
                            float *proj, float *cx, float *cy) {
    float wx = px - x0, wy = py - y0;
    float pr = fmaf(wx, vx, wy * vy) * inv_vv;
    pr = fmaxf_(0.0f, fminf_(1.0f, pr));
    *cx = fmaf(pr, vx, x0);
    *cy = fmaf(pr, vy, y0);
    float dx = *cx - px, dy = *cy - py;
    *proj = pr;
    return fmaf(dx, dx, dy * dy);
}

typedef struct {
    float min_d2, best_proj, best_cx, best_cy;
    int best_eid, parity, winding;
} fill_geom;

/* distance to the primitive's polyline and crossing parity / winding for the
   pixel centre (px, py) (cubic_splatting.py:1095-1134 forward, :1451-1501
   backward; the argmin keeps the first minimum, strict <) */
static inline void fill_pixel_geom(const float *edges, int e0, int e1, float px, float py, fill_geom *g) {
    g->min_d2 = 1e30f;
    g->best_eid = -1;
    g->best_proj = 0.f; g->best_cx = 0.f; g->best_cy = 0.f;
    g->parity = 0; g->winding = 0;
    for (int e = e0; e < e1; ++e) {
        const float *ed = edges + (int64_t)e * 4;
        float x0 = ed[0], y0 = ed[1], x1 = ed[2], y1 = ed[3];
        float vx = x1 - x0, vy = y1 - y0;
        float vv = vx * vx + vy * vy;
        float inv_vv = 1.0f / fmaxf_(vv, EPS_F);
        float proj, cx, cy;
        float d2 = edge_d2(x0, y0, vx, vy, inv_vv, px, py, &proj, &cx, &cy);
        if (d2 < g->min_d2) {
            g->min_d2 = d2; g->best_eid = e; g->best_proj = proj; g->best_cx = cx; g->best_cy = cy;
        }
        int cross = ((y0 <= py) & (y1 > py)) | ((y0 > py) & (y1 <= py));
        if (cross) {
            float lhs = x0 * vy + (py - y0) * vx;
            float rhs = px * vy;
            int hit = (vy > 0.0f) ? (lhs > rhs) : (lhs < rhs);
            g->parity ^= hit;
            g->winding += hit * ((vy > 0.0f) ? 1 : -1);
        }
    }
}

static inline float fill_cov(const fill_geom *g, int rule, float inv_sigma2_raw, float *out_sign,
                             float *out_dist, float *out_inv_sigma) {
    int inside = (rule == 0) ? (g->parity != 0) : (g->winding != 0);
    float dist = sqrtf(fmaxf_(g->min_d2, 0.0f));
    float inv_sigma = sqrtf(fmaxf_(inv_sigma2_raw, EPS_F));
    float sign = inside ? -1.0f : 1.0f;
    float logit = sign * dist * inv_sigma * 2.0f;
    logit = fmaxf_(-60.0f, fminf_(60.0f, logit));
    *out_sign = sign; *out_dist = dist; *out_inv_sigma = inv_sigma;
    return 1.0f / (1.0f + cso_expf(logit));
}

/* fill forward (manbo/ops/cubic_splatting.py:1036-1192) */
void cso_fill_forward(int img_h, int img_w, int block_x, int block_y, const int32_t *prim_ids_sorted,
                      const int32_t *tile_bins, const float *edges, const int32_t *isect_edge_ranges,
                      const float *colors, const float *opac, const float *inv_sigma2s,
                      const int32_t *rules, const float *bg, float *out, float *final_ts,
                      int32_t *final_idx) {
    const int tbx = (img_w + block_x - 1) / block_x;
    const int tby = (img_h + block_y - 1) / block_y;
    const int ntiles = tbx * tby;
#pragma omp parallel for schedule(dynamic, 1)
    for (int t = 0; t < ntiles; ++t) {
        int tx = t % tbx, ty = t / tbx;
        int rs = tile_bins[2 * t], re = tile_bins[2 * t + 1];
        for (int ly = 0; ly < block_y; ++ly)
            for (int lx = 0; lx < block_x; ++lx) {
                int i = ty * block_y + ly, j = tx * block_x + lx;
                if (i >= img_h || j >= img_w) continue;
                float px = (float)j + 0.5f, py = (float)i + 0.5f;
                float T = 1.0f, c0 = 0.f, c1 = 0.f, c2 = 0.f;
                int cur = 0;
                for (int k = rs; k < re; ++k) {
                    int pid = prim_ids_sorted[k];
                    fill_geom g;
                    fill_pixel_geom(edges, isect_edge_ranges[2 * k], isect_edge_ranges[2 * k + 1], px, py, &g);
                    float sign, dist, inv_sigma;
                    float cov = fill_cov(&g, rules[pid], inv_sigma2s[pid], &sign, &dist, &inv_sigma);
                    float alpha = fminf_(ALPHA_CAP, opac[pid] * cov);
                    if (alpha < ALPHA_MIN) continue;
                    float next_T = T * (1.0f - alpha);
                    float vis = alpha * T;
                    c0 += colors[3 * pid] * vis;
                    c1 += colors[3 * pid + 1] * vis;
                    c2 += colors[3 * pid + 2] * vis;
                    T = next_T;
                    cur = k;
                    if (next_T <= TRANS_STOP) break;
                }
                int64_t pix = (int64_t)i * img_w + j;
                final_ts[pix] = T;
                final_idx[pix] = cur;
                out[3 * pix] = c0 + T * bg[0];
                out[3 * pix + 1] = c1 + T * bg[1];
                out[3 * pix + 2] = c2 + T * bg[2];
            }
    }
}

/* Per-thread gradient accumulators, reduced in thread order at the end. */
typedef struct {
    float *v_edges, *v_colors, *v_opac, *v_inv, *v_extra, *contrib, *isect_contrib;
} grad_bufs;

static void grad_alloc(grad_bufs *b, int64_t nedges, int64_t nprims, int64_t nisect, int extra,
                       int want_contrib, int want_isect) {
    b->v_edges = (float *)calloc((size_t)nedges * 4, sizeof(float));
    b->v_colors = (float *)calloc((size_t)nprims * 3, sizeof(float));
    b->v_opac = (float *)calloc((size_t)nprims, sizeof(float));
    b->v_inv = (float *)calloc((size_t)nprims, sizeof(float));
    b->v_extra = extra ? (float *)calloc((size_t)nprims, sizeof(float)) : NULL;
    b->contrib = want_contrib ? (float *)calloc((size_t)nprims * 3, sizeof(float)) : NULL;
    b->isect_contrib = want_isect ? (float *)calloc((size_t)(nisect > 0 ? nisect : 1), sizeof(float)) : NULL;
}

static void grad_free(grad_bufs *b) {
    free(b->v_edges); free(b->v_colors); free(b->v_opac); free(b->v_inv);
    free(b->v_extra); free(b->contrib); free(b->isect_contrib);
}

static void grad_reduce(grad_bufs *bufs, int nb, int64_t nedges, int64_t nprims, int64_t nisect,
                        float *v_edges, float *v_colors, float *v_opac, float *v_inv, float *v_extra,
                        float *contrib, float *isect_contrib) {
    for (int b = 0; b < nb; ++b) {
        for (int64_t i = 0; i < nedges * 4; ++i) v_edges[i] += bufs[b].v_edges[i];
        for (int64_t i = 0; i < nprims * 3; ++i) v_colors[i] += bufs[b].v_colors[i];
        for (int64_t i = 0; i < nprims; ++i) { v_opac[i] += bufs[b].v_opac[i]; v_inv[i] += bufs[b].v_inv[i]; }
        if (v_extra) for (int64_t i = 0; i < nprims; ++i) v_extra[i] += bufs[b].v_extra[i];
        if (contrib) for (int64_t i = 0; i < nprims * 3; ++i) contrib[i] += bufs[b].contrib[i];
        if (isect_contrib) for (int64_t i = 0; i < nisect; ++i) isect_contrib[i] += bufs[b].isect_contrib[i];
    }
}

static int oracle_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static int oracle_thread_id(void) {
#ifdef _OPENMP
    return omp_get_thread_num();
#else
    return 0;
#endif
}

/* fill backward (manbo/ops/cubic_splatting.py:1339-1649): reverse compositing
   from final_idx, T <- T/(1-alpha), geometry grads to the closest edge only,
   opacity / softness / geometry grads gated by alpha < 0.999.  Outputs are
   accumulated (+=) into the caller's zero-initialised buffers. */
void cso_fill_backward(int img_h, int img_w, int block_x, int block_y, int64_t num_edges,
                       int64_t num_prims, int64_t num_isect, const int32_t *prim_ids_sorted,
                       const int32_t *tile_bins, const float *edges, const int32_t *isect_edge_ranges,
                       const float *colors, const float *opac, const float *inv_sigma2s,
                       const int32_t *rules, const float *bg, const float *final_ts,
                       const int32_t *final_idx, const float *v_out, float *v_edges, float *v_colors,
                       float *v_opac, float *v_inv, float *contrib_rgb, float *isect_contrib) {
    const int tbx = (img_w + block_x - 1) / block_x;
    const int tby = (img_h + block_y - 1) / block_y;
    const int ntiles = tbx * tby;
    const int collect = (contrib_rgb != NULL) | (isect_contrib != NULL);
    const int nb = oracle_threads();
    grad_bufs *bufs = (grad_bufs *)calloc((size_t)nb, sizeof(grad_bufs));
    for (int b = 0; b < nb; ++b)
        grad_alloc(&bufs[b], num_edges, num_prims, num_isect, 0, contrib_rgb != NULL, isect_contrib != NULL);
#pragma omp parallel for schedule(static, 1)
    for (int t = 0; t < ntiles; ++t) {
        grad_bufs *B = &bufs[oracle_thread_id()];
        int tx = t % tbx, ty = t / tbx;
        int rs = tile_bins[2 * t], re = tile_bins[2 * t + 1];
        for (int ly = 0; ly < block_y; ++ly)
            for (int lx = 0; lx < block_x; ++lx) {
                int i = ty * block_y + ly, j = tx * block_x + lx;
                if (i >= img_h || j >= img_w) continue;
                int64_t pix = (int64_t)i * img_w + j;
                float px = (float)j + 0.5f, py = (float)i + 0.5f;
                int bin_final = final_idx[pix];
                float T = final_ts[pix];
                const float T_final = T;
                float vo0 = v_out[3 * pix], vo1 = v_out[3 * pix + 1], vo2 = v_out[3 * pix + 2];
                float bg_dot = bg[0] * vo0 + bg[1] * vo1 + bg[2] * vo2;
                float buf0 = 0.f, buf1 = 0.f, buf2 = 0.f;
                for (int k = re - 1; k >= rs; --k) {
                    if (k > bin_final) continue;
                    int pid = prim_ids_sorted[k];
                    float rgb0 = colors[3 * pid], rgb1 = colors[3 * pid + 1], rgb2 = colors[3 * pid + 2];
                    float op = opac[pid];
                    fill_geom g;
                    fill_pixel_geom(edges, isect_edge_ranges[2 * k], isect_edge_ranges[2 * k + 1], px, py, &g);
                    float sign, dist, inv_sigma;
                    float cov = fill_cov(&g, rules[pid], inv_sigma2s[pid], &sign, &dist, &inv_sigma);
                    float alpha = fminf_(ALPHA_CAP, op * cov);
                    if (!(alpha >= ALPHA_MIN)) continue;
                    float ra = 1.0f / (1.0f - alpha);
                    T = T * ra;
                    float fac = alpha * T;
                    B->v_colors[3 * pid] += fac * vo0;
                    B->v_colors[3 * pid + 1] += fac * vo1;
                    B->v_colors[3 * pid + 2] += fac * vo2;
                    if (collect) {
                        float cr0 = fac * rgb0, cr1 = fac * rgb1, cr2 = fac * rgb2;
                        if (B->contrib) {
                            B->contrib[3 * pid] += cr0; B->contrib[3 * pid + 1] += cr1; B->contrib[3 * pid + 2] += cr2;
                        }
                        if (B->isect_contrib) B->isect_contrib[k] += cr0 + cr1 + cr2;
                    }
                    float v_alpha = 0.0f;
                    v_alpha = v_alpha + (rgb0 * T - buf0 * ra) * vo0;
                    v_alpha = v_alpha + (rgb1 * T - buf1 * ra) * vo1;
                    v_alpha = v_alpha + (rgb2 * T - buf2 * ra) * vo2;
                    v_alpha = v_alpha + T_final * ra * (0.0f - bg_dot);
                    buf0 = buf0 + rgb0 * fac;
                    buf1 = buf1 + rgb1 * fac;
                    buf2 = buf2 + rgb2 * fac;
                    if (alpha < ALPHA_CAP) {
                        B->v_opac[pid] += cov * v_alpha;
                        float v_cov = op * v_alpha;
                        float v_logit = -v_cov * cov * (1.0f - cov);
                        float v_inv_sigma = v_logit * sign * dist * 2.0f;
                        B->v_inv[pid] += v_inv_sigma * 0.5f / fmaxf_(inv_sigma, EPS_F);
                        if ((dist > EPS_F) & (g.best_eid >= 0)) {
                            float v_dist = v_logit * sign * inv_sigma * 2.0f;
                            float gx = v_dist * (g.best_cx - px) / dist;
                            float gy = v_dist * (g.best_cy - py) / dist;
                            float *ve = B->v_edges + (int64_t)g.best_eid * 4;
                            ve[0] += (1.0f - g.best_proj) * gx;
                            ve[1] += (1.0f - g.best_proj) * gy;
                            ve[2] += g.best_proj * gx;
                            ve[3] += g.best_proj * gy;
                        }
                    }
                }
            }
    }
    grad_reduce(bufs, nb, num_edges, num_prims, num_isect, v_edges, v_colors, v_opac, v_inv, NULL,
                contrib_rgb, isect_contrib);
    for (int b = 0; b < nb; ++b) grad_free(&bufs[b]);
    free(bufs);
}

/* edge endpoint grads -> cubic control-point grads with Bernstein weights at
   t = e / E (manbo/ops/cubic_splatting.py:2335-2394) */
void cso_edge_grads_to_cubics(int64_t num_segments, int edges_per_segment, const float *v_edges,
                              float *v_cubics) {
    const float inv_e = 1.0f / (float)edges_per_segment;
    for (int64_t g = 0; g < num_segments; ++g) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int e = 0; e < edges_per_segment; ++e) {
            float t0 = (float)e * inv_e, t1 = (float)(e + 1) * inv_e;
            float omt0 = 1.0f - t0, omt1 = 1.0f - t1;
            float omt0_2 = omt0 * omt0, omt1_2 = omt1 * omt1;
            float t0_2 = t0 * t0, t1_2 = t1 * t1;
            float b00 = omt0_2 * omt0, b01 = 3.0f * omt0_2 * t0, b02 = 3.0f * omt0 * t0_2, b03 = t0_2 * t0;
            float b10 = omt1_2 * omt1, b11 = 3.0f * omt1_2 * t1, b12 = 3.0f * omt1 * t1_2, b13 = t1_2 * t1;
            const float *v = v_edges + (g * edges_per_segment + e) * 4;
            float gsx = v[0], gsy = v[1], gex = v[2], gey = v[3];
            acc[0] = acc[0] + gsx * b00 + gex * b10;
            acc[1] = acc[1] + gsy * b00 + gey * b10;
            acc[2] = acc[2] + gsx * b01 + gex * b11;
            acc[3] = acc[3] + gsy * b01 + gey * b11;
            acc[4] = acc[4] + gsx * b02 + gex * b12;
            acc[5] = acc[5] + gsy * b02 + gey * b12;
            acc[6] = acc[6] + gsx * b03 + gex * b13;
            acc[7] = acc[7] + gsy * b03 + gey * b13;
        }
        memcpy(v_cubics + g * 8, acc, sizeof(acc));
    }
}

/* ------------------------------------------------------------------------ */
/* adaptive de Casteljau flattening, restated breadth-first as the reference  */
/* runs it (manbo/ops/cubic_splatting.py:1729-1832): per depth, flatness      */
/* flags (:1925-1953, its host branch :1924-1946), split of the non-flat      */
/* cubics at t = 1/2 (:2000-2028), leaves sorted by (segment, t0).            */

static inline float dc_max(float a, float b) { /* torch.maximum: NaN wins */
    if (a != a) return a;
    if (b != b) return b;
    return a > b ? a : b;
}

static inline float dc_clamp_min(float a, float lo) { return a != a ? a : (a < lo ? lo : a); }

static int dc_is_flat(const float *c, float tol) {
    const float lx = c[6] - c[0], ly = c[7] - c[1];
    const float chord2 = lx * lx + ly * ly;
    const float chord = sqrtf(dc_clamp_min(chord2, 1e-6f));
    const float v1x = c[2] - c[0], v1y = c[3] - c[1], v2x = c[4] - c[0], v2y = c[5] - c[1];
    const float cross1 = fabsf(lx * v1y - ly * v1x);
    const float cross2 = fabsf(lx * v2y - ly * v2x);
    float dmax = dc_max(cross1 / chord, cross2 / chord);
    if (chord2 <= 1e-6f) {
        const float n1 = sqrtf(dc_clamp_min(v1x * v1x + v1y * v1y, 0.0f));
        const float n2 = sqrtf(dc_clamp_min(v2x * v2x + v2y * v2y, 0.0f));
        dmax = dc_max(n1, dc_max(n2, sqrtf(dc_clamp_min(chord2, 0.0f))));
    }
    return dmax <= tol;
}

typedef struct { float c[8]; int64_t sid; float t0, t1; } dc_node;

static int64_t dc_key_base;
static int dc_cmp(const void *a, const void *b) {
    const dc_node *x = (const dc_node *)a, *y = (const dc_node *)b;
    const int64_t kx = x->sid * (dc_key_base + 1) + (int64_t)rintf(x->t0 * (float)dc_key_base);
    const int64_t ky = y->sid * (dc_key_base + 1) + (int64_t)rintf(y->t0 * (float)dc_key_base);
    return kx < ky ? -1 : (kx > ky ? 1 : 0);
}

/* Returns the number of edges E; edges [E, 2, 2], t0/t1 [E], seg_offs
   [nseg + 1].  The output buffers hold nseg << max_depth edges. */
int64_t cso_flatten_de_casteljau(int64_t nseg, int samples, float tol, const float *cubics,
                                 float *edges, float *t0o, float *t1o, int32_t *seg_offs) {
    const int e_per = (samples < 2 ? 2 : samples) - 1;
    const int max_depth = (int)ceil(log2((double)(e_per > 1 ? e_per : 1)));
    if (tol < 1e-4f) tol = 1e-4f;
    const int64_t cap = nseg << max_depth;
    dc_node *active = (dc_node *)malloc(sizeof(dc_node) * (size_t)(cap > 0 ? cap : 1));
    dc_node *next = (dc_node *)malloc(sizeof(dc_node) * (size_t)(cap > 0 ? cap : 1));
    dc_node *leaves = (dc_node *)malloc(sizeof(dc_node) * (size_t)(cap > 0 ? cap : 1));
    int64_t na = nseg, nl = 0;
    for (int64_t g = 0; g < nseg; ++g) {
        memcpy(active[g].c, cubics + g * 8, sizeof(float) * 8);
        active[g].sid = g;
        active[g].t0 = 0.0f;
        active[g].t1 = 1.0f;
    }
    for (int depth = 0; depth <= max_depth && na > 0; ++depth) {
        int64_t nsplit = 0;
        for (int64_t i = 0; i < na; ++i) {
            if (depth >= max_depth || dc_is_flat(active[i].c, tol)) leaves[nl++] = active[i];
            else active[nsplit++] = active[i];
        }
        /* children: all left halves, then all right halves */
        for (int64_t i = 0; i < nsplit; ++i) {
            const dc_node *p = &active[i];
            dc_node *l = &next[i], *r = &next[nsplit + i];
            for (int a = 0; a < 2; ++a) {
                const float p0 = p->c[a], p1 = p->c[2 + a], p2 = p->c[4 + a], p3 = p->c[6 + a];
                const float p01 = 0.5f * (p0 + p1), p12 = 0.5f * (p1 + p2), p23 = 0.5f * (p2 + p3);
                const float p012 = 0.5f * (p01 + p12), p123 = 0.5f * (p12 + p23);
                const float p0123 = 0.5f * (p012 + p123);
                l->c[a] = p0; l->c[2 + a] = p01; l->c[4 + a] = p012; l->c[6 + a] = p0123;
                r->c[a] = p0123; r->c[2 + a] = p123; r->c[4 + a] = p23; r->c[6 + a] = p3;
            }
            const float tm = 0.5f * (p->t0 + p->t1);
            l->sid = r->sid = p->sid;
            l->t0 = p->t0; l->t1 = tm;
            r->t0 = tm; r->t1 = p->t1;
        }
        dc_node *tmp = active; active = next; next = tmp;
        na = 2 * nsplit;
    }
    dc_key_base = (int64_t)1 << max_depth;
    qsort(leaves, (size_t)nl, sizeof(dc_node), dc_cmp);
    for (int64_t g = 0; g <= nseg; ++g) seg_offs[g] = 0;
    for (int64_t i = 0; i < nl; ++i) {
        const dc_node *q = &leaves[i];
        edges[i * 4 + 0] = q->c[0]; edges[i * 4 + 1] = q->c[1];
        edges[i * 4 + 2] = q->c[6]; edges[i * 4 + 3] = q->c[7];
        t0o[i] = q->t0;
        t1o[i] = q->t1;
        seg_offs[q->sid + 1] += 1;
    }
    for (int64_t g = 0; g < nseg; ++g) seg_offs[g + 1] += seg_offs[g];
    free(active); free(next); free(leaves);
    return nl;
}

/* de Casteljau edge grads -> cubic grads over CSR edge ranges with the
   leaves' parameter intervals (cubic_splatting.py:2420-2487) */
void cso_edge_grads_csr(int64_t num_segments, const int32_t *seg_offs, const float *t_start,
                        const float *t_end, const float *v_edges, float *v_cubics) {
    for (int64_t g = 0; g < num_segments; ++g) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int64_t e = seg_offs[g]; e < seg_offs[g + 1]; ++e) {
            const float t0 = t_start[e], t1 = t_end[e];
            const float omt0 = 1.0f - t0, omt1 = 1.0f - t1;
            const float omt0_2 = omt0 * omt0, omt1_2 = omt1 * omt1;
            const float t0_2 = t0 * t0, t1_2 = t1 * t1;
            const float b00 = omt0_2 * omt0, b01 = 3.0f * omt0_2 * t0, b02 = 3.0f * omt0 * t0_2,
                        b03 = t0_2 * t0;
            const float b10 = omt1_2 * omt1, b11 = 3.0f * omt1_2 * t1, b12 = 3.0f * omt1 * t1_2,
                        b13 = t1_2 * t1;
            const float *v = v_edges + e * 4;
            const float gsx = v[0], gsy = v[1], gex = v[2], gey = v[3];
            acc[0] = acc[0] + gsx * b00 + gex * b10;
            acc[1] = acc[1] + gsy * b00 + gey * b10;
            acc[2] = acc[2] + gsx * b01 + gex * b11;
            acc[3] = acc[3] + gsy * b01 + gey * b11;
            acc[4] = acc[4] + gsx * b02 + gex * b12;
            acc[5] = acc[5] + gsy * b02 + gey * b12;
            acc[6] = acc[6] + gsx * b03 + gex * b13;
            acc[7] = acc[7] + gsy * b03 + gey * b13;
        }
        memcpy(v_cubics + g * 8, acc, sizeof(acc));
    }
}

/* ------------------------------------------------------------------------ */
/* stroke mode (manbo/ops/cubic_polyline_splatting.py:145-247, 393-658)      */

static inline float stroke_min_d2(const float *edges, int e0, int e1, float px, float py, int *best_eid,
                                  float *best_proj, float *best_cx, float *best_cy) {
    float min_d2 = 1e30f;
    *best_eid = -1; *best_proj = 0.f; *best_cx = 0.f; *best_cy = 0.f;
    for (int e = e0; e < e1; ++e) {
        const float *ed = edges + (int64_t)e * 4;
        float x0 = ed[0], y0 = ed[1], x1 = ed[2], y1 = ed[3];
        float vx = x1 - x0, vy = y1 - y0;
        float vv = vx * vx + vy * vy;
        float inv_vv = 1.0f / fmaxf_(vv, EPS_F);
        float proj, cx, cy;
        float d2 = edge_d2(x0, y0, vx, vy, inv_vv, px, py, &proj, &cx, &cy);
        if (d2 < min_d2) {
            min_d2 = d2; *best_eid = e; *best_proj = proj; *best_cx = cx; *best_cy = cy;
        }
    }
    return min_d2;
}

void cso_stroke_forward(int img_h, int img_w, int block_x, int block_y, const int32_t *prim_ids_sorted,
                        const int32_t *tile_bins, const float *edges, const int32_t *isect_edge_ranges,
                        const float *colors, const float *opac, const float *stroke_widths,
                        const float *inv_sigma2s, const float *bg, float *out, float *final_ts,
                        int32_t *final_idx) {
    const int tbx = (img_w + block_x - 1) / block_x;
    const int tby = (img_h + block_y - 1) / block_y;
    const int ntiles = tbx * tby;
#pragma omp parallel for schedule(dynamic, 1)
    for (int t = 0; t < ntiles; ++t) {
        int tx = t % tbx, ty = t / tbx;
        int rs = tile_bins[2 * t], re = tile_bins[2 * t + 1];
        for (int ly = 0; ly < block_y; ++ly)
            for (int lx = 0; lx < block_x; ++lx) {
                int i = ty * block_y + ly, j = tx * block_x + lx;
                if (i >= img_h || j >= img_w) continue;
                float px = (float)j + 0.5f, py = (float)i + 0.5f;
                float T = 1.0f, c0 = 0.f, c1 = 0.f, c2 = 0.f;
                int cur = 0;
                for (int k = rs; k < re; ++k) {
                    int pid = prim_ids_sorted[k];
                    int be; float bp, bcx, bcy;
                    float min_d2 = stroke_min_d2(edges, isect_edge_ranges[2 * k], isect_edge_ranges[2 * k + 1],
                                                 px, py, &be, &bp, &bcx, &bcy);
                    float dist = sqrtf(fmaxf_(min_d2, 0.0f));
                    float half_sw = fmaxf_(0.0f, stroke_widths[pid]) * 0.5f;
                    float inv_s2 = fmaxf_(inv_sigma2s[pid], EPS_F);
                    float edge_d = fmaxf_(0.0f, dist - half_sw);
                    float sigma = 0.5f * edge_d * edge_d * inv_s2;
                    float cov = cso_expf(-sigma);
                    float alpha = fminf_(ALPHA_CAP, opac[pid] * cov);
                    if (alpha < ALPHA_MIN) continue;
                    float next_T = T * (1.0f - alpha);
                    float vis = alpha * T;
                    c0 += colors[3 * pid] * vis;
                    c1 += colors[3 * pid + 1] * vis;
                    c2 += colors[3 * pid + 2] * vis;
                    T = next_T;
                    cur = k;
                    if (next_T <= TRANS_STOP) break;
                }
                int64_t pix = (int64_t)i * img_w + j;
                final_ts[pix] = T;
                final_idx[pix] = cur;
                out[3 * pix] = c0 + T * bg[0];
                out[3 * pix + 1] = c1 + T * bg[1];
                out[3 * pix + 2] = c2 + T * bg[2];
            }
    }
}

void cso_stroke_backward(int img_h, int img_w, int block_x, int block_y, int64_t num_edges,
                         int64_t num_prims, int64_t num_isect, const int32_t *prim_ids_sorted,
                         const int32_t *tile_bins, const float *edges, const int32_t *isect_edge_ranges,
                         const float *colors, const float *opac, const float *stroke_widths,
                         const float *inv_sigma2s, const float *bg, const float *final_ts,
                         const int32_t *final_idx, const float *v_out, float *v_edges, float *v_colors,
                         float *v_opac, float *v_stroke, float *v_inv, float *contrib_rgb,
                         float *isect_contrib) {
    const int tbx = (img_w + block_x - 1) / block_x;
    const int tby = (img_h + block_y - 1) / block_y;
    const int ntiles = tbx * tby;
    const int collect = (contrib_rgb != NULL) | (isect_contrib != NULL);
    const int nb = oracle_threads();
    grad_bufs *bufs = (grad_bufs *)calloc((size_t)nb, sizeof(grad_bufs));
    for (int b = 0; b < nb; ++b)
        grad_alloc(&bufs[b], num_edges, num_prims, num_isect, 1, contrib_rgb != NULL, isect_contrib != NULL);
#pragma omp parallel for schedule(static, 1)
    for (int t = 0; t < ntiles; ++t) {
        grad_bufs *B = &bufs[oracle_thread_id()];
        int tx = t % tbx, ty = t / tbx;
        int rs = tile_bins[2 * t], re = tile_bins[2 * t + 1];
        for (int ly = 0; ly < block_y; ++ly)
            for (int lx = 0; lx < block_x; ++lx) {
                int i = ty * block_y + ly, j = tx * block_x + lx;
                if (i >= img_h || j >= img_w) continue;
                int64_t pix = (int64_t)i * img_w + j;
                float px = (float)j + 0.5f, py = (float)i + 0.5f;
                int bin_final = final_idx[pix];
                float T = final_ts[pix];
                const float T_final = T;
                float vo0 = v_out[3 * pix], vo1 = v_out[3 * pix + 1], vo2 = v_out[3 * pix + 2];
                float bg_dot = bg[0] * vo0 + bg[1] * vo1 + bg[2] * vo2;
                float buf0 = 0.f, buf1 = 0.f, buf2 = 0.f;
                for (int k = re - 1; k >= rs; --k) {
                    if (k > bin_final) continue;
                    int pid = prim_ids_sorted[k];
                    float rgb0 = colors[3 * pid], rgb1 = colors[3 * pid + 1], rgb2 = colors[3 * pid + 2];
                    float op = opac[pid];
                    float stroke_w = stroke_widths[pid];
                    float inv_s2 = fmaxf_(inv_sigma2s[pid], EPS_F);
                    int be; float bp, bcx, bcy;
                    float min_d2 = stroke_min_d2(edges, isect_edge_ranges[2 * k], isect_edge_ranges[2 * k + 1],
                                                 px, py, &be, &bp, &bcx, &bcy);
                    float dist = sqrtf(fmaxf_(min_d2, 0.0f));
                    float half_sw = fmaxf_(0.0f, stroke_w) * 0.5f;
                    float edge_d = fmaxf_(0.0f, dist - half_sw);
                    float sigma = 0.5f * edge_d * edge_d * inv_s2;
                    float cov = cso_expf(-sigma);
                    float alpha = fminf_(ALPHA_CAP, op * cov);
                    if (!(alpha >= ALPHA_MIN)) continue;
                    float ra = 1.0f / (1.0f - alpha);
                    T = T * ra;
                    float fac = alpha * T;
                    B->v_colors[3 * pid] += fac * vo0;
                    B->v_colors[3 * pid + 1] += fac * vo1;
                    B->v_colors[3 * pid + 2] += fac * vo2;
                    if (collect) {
                        float cr0 = fac * rgb0, cr1 = fac * rgb1, cr2 = fac * rgb2;
                        if (B->contrib) {
                            B->contrib[3 * pid] += cr0; B->contrib[3 * pid + 1] += cr1; B->contrib[3 * pid + 2] += cr2;
                        }
                        if (B->isect_contrib) B->isect_contrib[k] += cr0 + cr1 + cr2;
                    }
                    float v_alpha = 0.0f;
                    v_alpha = v_alpha + (rgb0 * T - buf0 * ra) * vo0;
                    v_alpha = v_alpha + (rgb1 * T - buf1 * ra) * vo1;
                    v_alpha = v_alpha + (rgb2 * T - buf2 * ra) * vo2;
                    v_alpha = v_alpha + T_final * ra * (0.0f - bg_dot);
                    buf0 = buf0 + rgb0 * fac;
                    buf1 = buf1 + rgb1 * fac;
                    buf2 = buf2 + rgb2 * fac;
                    if (alpha < ALPHA_CAP) {
                        B->v_opac[pid] += cov * v_alpha;
                        float v_sigma = -op * cov * v_alpha;
                        B->v_inv[pid] += 0.5f * edge_d * edge_d * v_sigma;
                        if (edge_d > 0.0f) {
                            float v_edge = v_sigma * edge_d * inv_s2;
                            B->v_extra[pid] += -0.5f * v_edge;
                            if ((dist > EPS_F) & (be >= 0)) {
                                float gx = v_edge * (bcx - px) / dist;
                                float gy = v_edge * (bcy - py) / dist;
                                float *ve = B->v_edges + (int64_t)be * 4;
                                ve[0] += (1.0f - bp) * gx;
                                ve[1] += (1.0f - bp) * gy;
                                ve[2] += bp * gx;
                                ve[3] += bp * gy;
                            }
                        }
                    }
                }
            }
    }
    grad_reduce(bufs, nb, num_edges, num_prims, num_isect, v_edges, v_colors, v_opac, v_inv, v_stroke,
                contrib_rgb, isect_contrib);
    for (int b = 0; b < nb; ++b) grad_free(&bufs[b]);
    free(bufs);
}

/* ------------------------------------------------------------------------ */
/* metrics (manbo/ops/metric.py:49-91, 249-339)                              */

double cso_sse(int64_t n, const float *x, const float *y) {
    double acc = 0.0;
#pragma omp parallel for reduction(+ : acc)
    for (int64_t i = 0; i < n; ++i) {
        float d = x[i] - y[i];
        acc += (double)(d * d);
    }
    return acc;
}

/* direct (non-separable) valid-window SSIM map with win2d = outer(g, g) */
void cso_ssim_map(int64_t planes, int h, int w, int win, const float *x, const float *y,
                  const float *win2d, float c1, float c2, float *out) {
    const int oh = h - win + 1, ow = w - win + 1;
#pragma omp parallel for schedule(static)
    for (int64_t pl = 0; pl < planes; ++pl)
        for (int oy = 0; oy < oh; ++oy)
            for (int ox = 0; ox < ow; ++ox) {
                float mu1 = 0.f, mu2 = 0.f, ex2 = 0.f, ey2 = 0.f, exy = 0.f;
                for (int ky = 0; ky < win; ++ky)
                    for (int kx = 0; kx < win; ++kx) {
                        float wv = win2d[ky * win + kx];
                        float xv = x[(pl * h + oy + ky) * w + ox + kx];
                        float yv = y[(pl * h + oy + ky) * w + ox + kx];
                        mu1 += wv * xv;
                        mu2 += wv * yv;
                        ex2 += wv * xv * xv;
                        ey2 += wv * yv * yv;
                        exy += wv * xv * yv;
                    }
                float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2, mu1_mu2 = mu1 * mu2;
                float s1 = ex2 - mu1_sq, s2 = ey2 - mu2_sq, s12 = exy - mu1_mu2;
                float lum = (2.0f * mu1_mu2 + c1) / (mu1_sq + mu2_sq + c1);
                float cs = (2.0f * s12 + c2) / (s1 + s2 + c2);
                out[(pl * oh + oy) * ow + ox] = lum * cs;
            }
}

/* ------------------------------------------------------------------------ */
/* closed ring segments (manbo/ops/cubic_splatting.py:190-266, 321-395)     */

void cso_ring_segments_forward(int64_t num_curves, int k, int subdiv, const float *cp, const float *basis,
                               const float *deriv_basis, const float *dt, float *out) {
    const int kb = (k + 2) / 2, spc = 2 * subdiv;
    const float degree = (float)(kb - 1), one_third = (float)(1.0 / 3.0);
    for (int64_t sid = 0; sid < num_curves * spc; ++sid) {
        int64_t curve = sid / spc;
        int local = (int)(sid - curve * spc);
        int branch = local / subdiv, s = local - branch * subdiv, sn = s + 1;
        int base = branch * (kb - 1);
        const float *c = cp + curve * k * 2;
        float p0x = 0, p0y = 0, p3x = 0, p3y = 0, d0x = 0, d0y = 0, d1x = 0, d1y = 0;
        for (int i = 0; i < kb; ++i) {
            int idx = base + i; if (idx >= k) idx -= k;
            float w0 = basis[s * kb + i], w1 = basis[sn * kb + i];
            p0x = p0x + w0 * c[2 * idx]; p0y = p0y + w0 * c[2 * idx + 1];
            p3x = p3x + w1 * c[2 * idx]; p3y = p3y + w1 * c[2 * idx + 1];
        }
        for (int i = 0; i < kb - 1; ++i) {
            int ic = base + i, in_ = ic + 1;
            if (ic >= k) ic -= k;
            if (in_ >= k) in_ -= k;
            float dx = c[2 * in_] - c[2 * ic], dy = c[2 * in_ + 1] - c[2 * ic + 1];
            float db0 = deriv_basis[s * (kb - 1) + i], db1 = deriv_basis[sn * (kb - 1) + i];
            d0x = d0x + db0 * dx; d0y = d0y + db0 * dy;
            d1x = d1x + db1 * dx; d1y = d1y + db1 * dy;
        }
        d0x = d0x * degree; d0y = d0y * degree; d1x = d1x * degree; d1y = d1y * degree;
        float dts = dt[s] * one_third;
        float *o = out + sid * 8;
        o[0] = p0x; o[1] = p0y; o[6] = p3x; o[7] = p3y;
        o[2] = p0x + d0x * dts; o[3] = p0y + d0y * dts;
        o[4] = p3x - d1x * dts; o[5] = p3y - d1y * dts;
    }
}

void cso_ring_segments_backward(int64_t num_curves, int k, int subdiv, const float *grad_segments,
                                const float *basis, const float *deriv_basis, const float *dt,
                                float *grad_cp) {
    const int kb = (k + 2) / 2, spc = 2 * subdiv;
    const float degree = (float)(kb - 1), one_third = (float)(1.0 / 3.0);
    for (int64_t sid = 0; sid < num_curves * spc; ++sid) {
        int64_t curve = sid / spc;
        int local = (int)(sid - curve * spc);
        int branch = local / subdiv, s = local - branch * subdiv, sn = s + 1;
        int base = branch * (kb - 1);
        float dts = dt[s] * one_third;
        const float *gsg = grad_segments + sid * 8;
        float g0x = gsg[0] + gsg[2], g0y = gsg[1] + gsg[3];
        float g3x = gsg[6] + gsg[4], g3y = gsg[7] + gsg[5];
        float gd0x = gsg[2] * dts, gd0y = gsg[3] * dts;
        float gd1x = -gsg[4] * dts, gd1y = -gsg[5] * dts;
        float *gc = grad_cp + curve * k * 2;
        for (int i = 0; i < kb; ++i) {
            int idx = base + i; if (idx >= k) idx -= k;
            float w0 = basis[s * kb + i], w1 = basis[sn * kb + i];
            gc[2 * idx] += g0x * w0 + g3x * w1;
            gc[2 * idx + 1] += g0y * w0 + g3y * w1;
        }
        for (int i = 0; i < kb - 1; ++i) {
            int ic = base + i, in_ = ic + 1;
            if (ic >= k) ic -= k;
            if (in_ >= k) in_ -= k;
            float db0 = deriv_basis[s * (kb - 1) + i], db1 = deriv_basis[sn * (kb - 1) + i];
            float dcx = degree * (gd0x * db0 + gd1x * db1);
            float dcy = degree * (gd0y * db0 + gd1y * db1);
            gc[2 * ic] += -dcx; gc[2 * ic + 1] += -dcy;
            gc[2 * in_] += dcx; gc[2 * in_ + 1] += dcy;
        }
    }
}

int cso_num_threads(void) { return oracle_threads(); }

/* ------------------------------------------------------------------------ */
/* Adan step (manbo/ops/optim.py:60-104), element by element in float32.     */

void cso_adan_step(float *param, const float *grad, float *exp_avg, float *exp_avg_sq,
                   float *exp_avg_diff, float *neg_pre_grad, int64_t numel, int step,
                   float beta1, float beta2, float beta3, float bc1, float bc2, float bc3_sqrt,
                   float lr, float weight_decay, float eps, float clip, int no_prox) {
    for (int64_t i = 0; i < numel; ++i) {
        float g = grad[i] * clip;
        float ngod = (step == 1) ? 0.0f : neg_pre_grad[i] + g;
        float m_t = exp_avg[i] * beta1 + g * (1.0f - beta1);
        float d_t = exp_avg_diff[i] * beta2 + ngod * (1.0f - beta2);
        float ngod2 = ngod * beta2 + g;
        float n_t = exp_avg_sq[i] * beta3 + ngod2 * ngod2 * (1.0f - beta3);
        float denom = sqrtf(n_t) / bc3_sqrt + eps;
        float step_size = lr / bc1;
        float step_size_diff = lr * beta2 / bc2;
        float p = param[i];
        if (no_prox) {
            p = p * (1.0f - lr * weight_decay);
            p = p - step_size * m_t / denom;
            p = p - step_size_diff * d_t / denom;
        } else {
            p = p - step_size * m_t / denom;
            p = p - step_size_diff * d_t / denom;
            p = p / (1.0f + lr * weight_decay);
        }
        param[i] = p;
        exp_avg[i] = m_t;
        exp_avg_diff[i] = d_t;
        exp_avg_sq[i] = n_t;
        neg_pre_grad[i] = -g;
    }
}
