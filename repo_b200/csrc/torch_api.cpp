/*
 * torch_api.cpp -- torch binding of the C ABI for the renderer's autograd path.
 *
 * The drop-in entry points (manbo.ops.render_cubic_fill_splat_tilelang, the
 * stroke entry, mse_loss_tilelang, ssim) reach the kernels through this module
 * once per stage instead of once per kernel: one forward call clamps the
 * anti-aliasing widths, bins, stages and rasterises a frame; one backward call
 * rasterises the gradients and maps them to the control points.  Device memory
 * comes from torch's caching allocator; the kernels are the ones declared in
 * include/cubicsplat_b200.h, launched on the current torch stream.  There is
 * no CPU path.
 *
 * Intersect buffers are sized from the previous frame of the same shape (a
 * capacity cache).  The binning reports an overflow in its status word and then
 * leaves every tile empty, so a forward enqueues all of its launches before it
 * reads the counts back once; only a frame that outgrew the cached capacity is
 * binned again, with the exact sizes.  The first frame of a shape reads the
 * counts back before sizing its buffers.  Under CUDA graph capture nothing is
 * read back: the cached capacity is used (an eager frame of the same shape must
 * come first) and an overflow leaves the status word set and the image NaN.
 *
 * The reference orchestration this replaces is _CubicFillSplatFunction
 * (manbo/ops/cubic_splatting.py:2750-3125) and _CubicPolylineSplatFunction
 * (manbo/ops/cubic_polyline_splatting.py:962-1338).
 */
#include <torch/extension.h>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "cubicsplat_b200.h"

namespace py = pybind11;
using at::Tensor;
using OptT = std::optional<at::Tensor>;

namespace {

constexpr int64_t kI64Max = INT64_MAX;
constexpr int kTile = 16;

const char* err_name(int s) {
  switch (s) {
    case CS_ERR_ARG: return "invalid argument";
    case CS_ERR_CAPACITY: return "intersect capacity exceeded";
    case CS_ERR_CUDA: return "CUDA launch failed";
    case CS_ERR_UNSUPPORTED: return "unsupported configuration";
    case CS_ERR_TIMEOUT: return "device-side wait timed out";
    default: return "error";
  }
}

void check(int status, const char* what) {
  if (status != CS_OK)
    throw std::runtime_error(std::string(what) + " failed: " + err_name(status) + " (status " +
                             std::to_string(status) + ")");
}

template <class T>
T* P(const Tensor& t) {
  return static_cast<T*>(t.data_ptr());
}
template <class T>
T* P(const OptT& t) {
  return t ? static_cast<T*>(t->data_ptr()) : nullptr;
}

void* stream_of(const Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

at::TensorOptions f32(const Tensor& like) { return like.options().dtype(at::kFloat); }
at::TensorOptions i32(const Tensor& like) { return like.options().dtype(at::kInt); }

Tensor as_f32(const Tensor& t) {
  if (t.scalar_type() == at::kFloat) return t.is_contiguous() ? t : t.contiguous();
  return t.contiguous().to(at::kFloat);
}

// Smallest allocation class >= max(n, 1): multiples of 1/16 of the power of
// two below n (at most 6.25% over), at least 4096 -- frames of similar size
// reuse the caching allocator's blocks.
int64_t size_class(int64_t n) {
  n = std::max<int64_t>(n, 1);
  if (n <= 4096) return 4096;
  const int bl = 64 - __builtin_clzll(static_cast<unsigned long long>(n));
  const int64_t step = int64_t(1) << (bl - 5);
  return (n + step - 1) / step * step;
}

std::mutex g_mu;

// Zeroed workspaces, one per device and exact size: every launch that uses
// one leaves it zeroed, so launches in stream order share it.  Keyed by size
// because the binning workspace's layout depends on the tile count.
std::map<std::tuple<int, int, int64_t>, Tensor> g_ws;

Tensor workspace(const Tensor& like, int kind, int64_t nbytes, bool exact) {
  const int dev = like.device().index();
  std::lock_guard<std::mutex> lk(g_mu);
  if (!exact) {  // grown on demand
    auto key = std::make_tuple(dev, kind, int64_t(-1));
    auto it = g_ws.find(key);
    if (it != g_ws.end() && it->second.numel() >= nbytes) return it->second;
    Tensor t = at::zeros({std::max<int64_t>(nbytes, 256)}, like.options().dtype(at::kByte));
    g_ws[key] = t;
    return t;
  }
  auto key = std::make_tuple(dev, kind, nbytes);
  auto it = g_ws.find(key);
  if (it != g_ws.end()) return it->second;
  Tensor t = at::zeros({std::max<int64_t>(nbytes, 256)}, like.options().dtype(at::kByte));
  g_ws[key] = t;
  return t;
}

enum WsKind { kWsBin = 1, kWsRaster = 2, kWsMse = 3, kWsSsim = 4 };

// Intersect and staged-record capacities of the last frame of each shape.
struct Caps {
  int64_t isect = 0, dlist = 0;
};
using CapKey = std::tuple<int, int64_t, int64_t, int64_t, int64_t, int64_t, int, int64_t, int64_t>;
std::map<CapKey, Caps> g_caps;

bool capturing(const Tensor& like) {
  return cs_stream_is_capturing(stream_of(like)) != 0;
}

}  // namespace

// A binned and staged frame: the reference-format intersect list (tile_bins,
// prim_ids_sorted, isect_ids_sorted) plus the raster kernels' staged records.
struct Frame {
  OptT cubics_px, edges_px, prim_edge_offsets, prim_tile_ranges, num_tiles_hit;
  Tensor tile_bins, prim_ids_sorted;
  OptT isect_ids_sorted;
  int64_t num_intersects = 0;  // -1: unknown (enqueued under graph capture)
  int64_t isect_capacity = 0;  // rows of the per-intersect buffers
  int64_t num_records = -1;    // staged near-edge records (bound), when read back
  int64_t tbx = 0, tby = 0, samples = 0, r0 = 0, r1 = 0;
  Tensor tile_dlist, imeta;
  OptT rowoff;
  Tensor dlist, counters;
  bool stroke = false;
  Tensor isect_strips;
  OptT unit_order, unit_order_bwd, visit_lists, visit_winners;
  std::string flatten_method = "bernstein";
  OptT segment_edge_offsets, edge_t_starts, edge_t_ends;

  int64_t rows() const { return num_intersects >= 0 ? num_intersects : isect_capacity; }
  int32_t* status() const { return P<int32_t>(counters) + 1; }
};
using FrameP = std::shared_ptr<Frame>;

namespace {

struct BinInputs {
  Tensor cubics_norm, offs, depths, widths, inv_s2, colors, opac, basis;
  OptT rules, stroke_widths;
  int64_t h, w, samples, r0, r1;
  double aabb_pad;
  bool aniso, dc;
};

CapKey cap_key(const BinInputs& in, int64_t p, int64_t g) {
  const int flags = (in.stroke_widths ? 1 : 0) | (in.dc ? 2 : 0) | (in.aniso ? 4 : 0);
  return CapKey(in.cubics_norm.device().index(), p, g, in.h, in.w, in.samples, flags, in.r0,
                in.r1);
}

[[noreturn]] void offsets_error(const Tensor& offs, int64_t num_segments) {
  Tensor o = offs.to(at::kCPU);
  const int64_t a = o.numel() ? o[0].item<int64_t>() : 0;
  const int64_t b = o.numel() ? o[o.numel() - 1].item<int64_t>() : 0;
  throw py::value_error("primitive_seg_offsets must start at 0 and end at num_segments (got start=" +
                        std::to_string(a) + ", end=" + std::to_string(b) +
                        ", num_segments=" + std::to_string(num_segments) + ")");
}

// Per-intersect and staged-record buffers with `ci` rows and `cd` records.
void alloc_lists(Frame& f, const Tensor& like, int64_t ci, int64_t cd, int64_t band_tiles) {
  Tensor prim = at::empty({ci}, i32(like));
  Tensor keys = at::empty({ci}, like.options().dtype(at::kLong));
  f.prim_ids_sorted = prim;
  f.isect_ids_sorted = keys;
  f.imeta = at::empty({ci, 12}, i32(like));
  f.rowoff = f.stroke ? OptT() : OptT(at::empty({ci, 16}, i32(like)));
  f.dlist = at::empty({cd, 8}, f32(like));
  f.isect_strips = at::empty({ci, 4, 2}, i32(like));
  f.unit_order = at::empty({int64_t(cs_unit_lists_size(band_tiles) / 4)}, i32(like));
  f.isect_capacity = ci;
}

// Projection, flattening, counts and scans (cs_bin_count); then the scatter,
// per-tile sort and staging (cs_bin_sort) into buffers of the given capacity.
// With exact (no cached capacity) the counts are read back between the two and
// the buffers sized from them.  Returns the frame; num_intersects is known
// only in the exact case (else -1 until finish_frame).
FrameP bin_attempt(const BinInputs& in, int64_t icap, int64_t dcap, bool exact) {
  const Tensor& cn = in.cubics_norm;
  void* st = stream_of(cn);
  auto f = std::make_shared<Frame>();
  const int64_t s = std::max<int64_t>(2, in.samples);
  const int64_t g = cn.size(0);
  const int64_t p = in.offs.numel() - 1;
  f->tbx = (in.w + kTile - 1) / kTile;
  f->tby = (in.h + kTile - 1) / kTile;
  const int64_t nt = f->tbx * f->tby;
  f->r0 = in.r0;
  f->r1 = in.r1;
  f->samples = s;
  f->stroke = in.stroke_widths.has_value();
  f->flatten_method = in.dc ? "de_casteljau" : "bernstein";
  Tensor cubics_px = at::empty({g, 4, 2}, f32(cn));
  Tensor prim_ranges = at::empty({p, 4}, i32(cn));
  Tensor num_hit = at::empty({p}, i32(cn));
  f->tile_bins = at::empty({nt, 2}, i32(cn));
  f->tile_dlist = at::empty({nt, 2}, i32(cn));
  f->counters = at::zeros({4}, i32(cn));
  Tensor ws = workspace(cn, kWsBin, int64_t(cs_bin_workspace_size(nt)), true);
  Tensor edges, edge_offs;
  OptT peo;
  if (in.dc) {
    check(cs_project_cubics(P<float>(cn), nullptr, nullptr, P<float>(cubics_px), nullptr, nullptr,
                            g, (int32_t)in.h, (int32_t)in.w, 16, 16, 0.0f, 0, st),
          "cs_project_cubics");
    const int64_t cap = std::max<int64_t>(cs_de_casteljau_edge_capacity(g, (int32_t)s), 1);
    edges = at::empty({cap, 2, 2}, f32(cn));
    Tensor t0 = at::empty({cap}, f32(cn)), t1 = at::empty({cap}, f32(cn));
    Tensor seg = at::empty({g + 1}, i32(cn));
    edge_offs = at::empty({p + 1}, i32(cn));
    check(cs_flatten_de_casteljau(P<float>(cubics_px), P<int32_t>(in.offs), g, p, (int32_t)s, 0.5f,
                                  P<float>(edges), P<int32_t>(edge_offs), P<int32_t>(seg),
                                  P<float>(t0), P<float>(t1), cap, f->status(), st),
          "cs_flatten_de_casteljau");
    peo = edge_offs;
    f->segment_edge_offsets = seg;
    f->edge_t_starts = t0;
    f->edge_t_ends = t1;
  } else {
    edges = at::empty({g * (s - 1), 2, 2}, f32(cn));
    edge_offs = at::empty({p + 1}, i32(cn));
  }
  const Tensor sw = in.stroke_widths ? as_f32(*in.stroke_widths) : Tensor();
  const float* swp = in.stroke_widths ? P<float>(sw) : nullptr;
  check(cs_bin_count(P<float>(cn), P<int32_t>(in.offs), P<float>(in.widths), swp,
                     P<float>(in.basis), P<float>(cubics_px), P<float>(edges), P<int32_t>(peo),
                     in.dc ? nullptr : P<int32_t>(edge_offs), P<int32_t>(prim_ranges),
                     P<int32_t>(num_hit), P<int32_t>(f->tile_bins), P<int32_t>(f->tile_dlist),
                     P<int32_t>(f->counters), ws.data_ptr(), p, g, exact ? kI64Max : icap,
                     exact ? kI64Max : dcap, (int32_t)s, (int32_t)in.h, (int32_t)in.w,
                     (int32_t)in.r0, (int32_t)in.r1, (float)in.aabb_pad, in.aniso ? 1 : 0,
                     nullptr, 0, st),
        "cs_bin_count");
  f->cubics_px = cubics_px;
  f->edges_px = edges;
  f->prim_edge_offsets = edge_offs;
  f->prim_tile_ranges = prim_ranges;
  f->num_tiles_hit = num_hit;
  const int64_t band_tiles = std::max<int64_t>(1, in.r1 - in.r0) * f->tbx;
  int64_t n_sort = icap, d_sort = dcap;
  if (exact) {
    Tensor c = f->counters.to(at::kCPU);  // the one read-back of a first frame
    const int32_t* cv = c.data_ptr<int32_t>();
    const int64_t n = cv[0], status = cv[1], nd = cv[2];
    if (status == CS_ERR_ARG) offsets_error(in.offs, g);
    check((int)status, "cs_bin_count");
    f->num_intersects = n;
    f->num_records = nd;
    icap = size_class(n);
    dcap = size_class(nd);
    n_sort = n;
    d_sort = std::max<int64_t>(nd, 1);
  } else {
    f->num_intersects = -1;
  }
  alloc_lists(*f, cn, icap, dcap, band_tiles);
  if (!exact || n_sort > 0) {
    check(cs_bin_sort(P<int32_t>(prim_ranges), P<float>(in.depths), P<int32_t>(f->tile_bins),
                      P<int32_t>(f->prim_ids_sorted), P<int64_t>(f->isect_ids_sorted),
                      P<int32_t>(f->counters), ws.data_ptr(), p, n_sort, (int32_t)in.h,
                      (int32_t)in.w, (int32_t)in.r0, (int32_t)in.r1, P<float>(edges),
                      P<int32_t>(edge_offs), P<float>(in.colors), P<float>(in.opac),
                      P<float>(in.inv_s2), P<int32_t>(in.rules), swp, P<int32_t>(f->tile_dlist),
                      P<void>(f->imeta), P<int32_t>(f->rowoff), P<int32_t>(f->isect_strips),
                      P<void>(f->dlist), d_sort, P<int32_t>(f->unit_order), st),
          "cs_bin_sort");
  } else {
    f->unit_order = OptT();
  }
  if (exact) {
    const int64_t n = f->num_intersects;
    f->prim_ids_sorted = f->prim_ids_sorted.narrow(0, 0, n);
    f->isect_ids_sorted = f->isect_ids_sorted->narrow(0, 0, n);
  }
  return f;
}

// Reads the counts of an optimistic attempt back (eager only).  Returns false
// if the frame outgrew its capacity; then n and nd hold the exact sizes.
bool finish_frame(Frame& f, const BinInputs& in, int64_t& n, int64_t& nd) {
  Tensor c = f.counters.to(at::kCPU);
  const int32_t* cv = c.data_ptr<int32_t>();
  n = cv[0];
  nd = cv[2];
  const int status = cv[1];
  if (status == CS_ERR_ARG) offsets_error(in.offs, in.cubics_norm.size(0));
  if (status == CS_ERR_CAPACITY) return false;
  check(status, "cs_bin_count");
  f.num_intersects = n;
  f.num_records = nd;
  f.prim_ids_sorted = f.prim_ids_sorted.narrow(0, 0, n);
  f.isect_ids_sorted = f.isect_ids_sorted->narrow(0, 0, n);
  if (n == 0) f.unit_order = OptT();
  return true;
}

void remember(const BinInputs& in, int64_t n, int64_t nd) {
  const int64_t p = in.offs.numel() - 1, g = in.cubics_norm.size(0);
  const int64_t ci = size_class(n + n / 4 + 1024), cd = size_class(nd + nd / 4 + 16384);
  std::lock_guard<std::mutex> lk(g_mu);
  Caps& c = g_caps[cap_key(in, p, g)];
  if (c.isect < ci || c.isect > 8 * ci) c.isect = ci;
  if (c.dlist < cd || c.dlist > 8 * cd) c.dlist = cd;
}

bool cached(const BinInputs& in, Caps& out) {
  const int64_t p = in.offs.numel() - 1, g = in.cubics_norm.size(0);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_caps.find(cap_key(in, p, g));
  if (it == g_caps.end()) return false;
  out = it->second;
  return true;
}

BinInputs make_inputs(const Tensor& cubics_norm, const Tensor& offs, const Tensor& depths,
                      const Tensor& widths, const Tensor& inv_s2, const Tensor& colors,
                      const Tensor& opac, const OptT& rules, const OptT& stroke_widths,
                      const Tensor& basis, int64_t h, int64_t w, int64_t samples, double aabb_pad,
                      bool aniso, int64_t r0, int64_t r1, bool dc) {
  if (!cubics_norm.is_cuda())
    throw py::value_error("cubics_norm must be a CUDA tensor (the B200 renderer has no CPU path)");
  BinInputs in;
  in.cubics_norm = as_f32(cubics_norm);
  in.offs = offs;
  in.depths = as_f32(depths);
  in.widths = widths;
  in.inv_s2 = inv_s2;
  in.colors = colors;
  in.opac = opac;
  in.rules = rules;
  in.stroke_widths = stroke_widths;
  in.basis = basis;
  in.h = h;
  in.w = w;
  in.samples = samples;
  const int64_t tby = (h + kTile - 1) / kTile;
  in.r0 = std::max<int64_t>(0, r0);
  in.r1 = r1 < 0 ? tby : std::min<int64_t>(tby, r1);
  in.aabb_pad = aabb_pad;
  in.aniso = aniso;
  in.dc = dc;
  return in;
}

void fill_background(const Tensor& bg, const Tensor& out, const Tensor& fts, const Tensor& fidx) {
  out.copy_(bg.view({1, 1, 3}).expand_as(out));
  fts.fill_(1.0);
  fidx.fill_(0);
}

// Forward raster of a staged frame into (out, fts, fidx).
void raster_forward_into(Frame& f, const Tensor& bg, int64_t h, int64_t w, const OptT& out_chw,
                         const Tensor& out, const Tensor& fts, const Tensor& fidx) {
  if (f.num_intersects == 0) {
    fill_background(bg, out, fts, fidx);
    return;
  }
  void* st = stream_of(out);
  const int64_t nt = f.tbx * f.tby;
  Tensor ws = workspace(out, kWsRaster, int64_t(cs_raster_workspace_size(nt)), false);
  if (f.unit_order && !f.unit_order_bwd) f.unit_order_bwd = at::empty_like(*f.unit_order);
  if (!f.visit_lists) {
    const int64_t nbytes = int64_t(cs_visit_lists_size(f.rows(), nt));
    f.visit_lists = at::empty({nbytes / 4}, i32(out));
    if (!f.stroke) {
      const int64_t wbytes = int64_t(cs_visit_winners_size(f.rows(), nt));
      f.visit_winners = at::empty({wbytes / 2}, out.options().dtype(at::kShort));
    }
  }
  const Tensor bgc = as_f32(bg);
  if (!f.stroke) {
    check(cs_fill_forward(P<int32_t>(f.prim_ids_sorted), P<int32_t>(f.tile_bins),
                          P<int32_t>(f.tile_dlist), P<void>(f.imeta), P<int32_t>(f.isect_strips),
                          P<int32_t>(f.rowoff), P<void>(f.dlist), P<int32_t>(f.unit_order),
                          P<int32_t>(f.unit_order_bwd), P<int32_t>(f.visit_lists),
                          P<uint16_t>(f.visit_winners), P<float>(bgc), P<float>(out),
                          P<float>(fts), P<int32_t>(fidx), P<float>(out_chw), nullptr, nullptr,
                          f.status(), ws.data_ptr(), (int32_t)h, (int32_t)w, (int32_t)f.r0,
                          (int32_t)f.r1, st),
          "cs_fill_forward");
  } else {
    check(cs_stroke_forward(P<int32_t>(f.prim_ids_sorted), P<int32_t>(f.tile_bins),
                            P<int32_t>(f.tile_dlist), P<void>(f.imeta), P<int32_t>(f.isect_strips),
                            P<void>(f.dlist), P<int32_t>(f.unit_order),
                            P<int32_t>(f.unit_order_bwd), P<int32_t>(f.visit_lists),
                            P<uint16_t>(f.visit_winners), P<float>(bgc), P<float>(out),
                            P<float>(fts), P<int32_t>(fidx), P<float>(out_chw), nullptr, nullptr,
                            f.status(), ws.data_ptr(), (int32_t)h, (int32_t)w, (int32_t)f.r0,
                            (int32_t)f.r1, st),
          "cs_stroke_forward");
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// bound functions

// Bin and stage a frame (bin_primitives in repo_b200.render).
FrameP bin_frame(const Tensor& cubics_norm, const Tensor& offs, const Tensor& depths,
                 const Tensor& widths, const Tensor& inv_s2, const Tensor& colors,
                 const Tensor& opac, const OptT& rules, const OptT& stroke_widths,
                 const Tensor& basis, int64_t h, int64_t w, int64_t samples, double aabb_pad,
                 bool aniso, int64_t r0, int64_t r1, bool dc) {
  c10::cuda::CUDAGuard guard(cubics_norm.device());
  BinInputs in = make_inputs(cubics_norm, offs, depths, widths, inv_s2, colors, opac, rules,
                             stroke_widths, basis, h, w, samples, aabb_pad, aniso, r0, r1, dc);
  Caps c;
  const bool have = cached(in, c);
  if (capturing(in.cubics_norm)) {
    if (!have)
      throw std::runtime_error(
          "the renderer needs one call of this scene size outside CUDA graph capture before "
          "it is captured (intersect buffers are sized from it)");
    return bin_attempt(in, c.isect, c.dlist, false);
  }
  if (!have) {
    FrameP f = bin_attempt(in, 0, 0, true);
    remember(in, f->num_intersects, f->num_records);
    return f;
  }
  FrameP f = bin_attempt(in, c.isect, c.dlist, false);
  int64_t n = 0, nd = 0;
  if (!finish_frame(*f, in, n, nd)) {
    f = bin_attempt(in, size_class(n), size_class(nd), false);
    if (!finish_frame(*f, in, n, nd)) check(CS_ERR_CAPACITY, "cs_bin_count");
  }
  remember(in, n, nd);
  return f;
}

// Forward raster of a staged frame: (out [H, W, 3], final_Ts, final_idx).
std::tuple<Tensor, Tensor, Tensor> raster_forward(const FrameP& f, const Tensor& bg, int64_t h,
                                                  int64_t w, const OptT& out_chw,
                                                  const OptT& out_in, const OptT& fts_in,
                                                  const OptT& fidx_in) {
  c10::cuda::CUDAGuard guard(f->tile_bins.device());
  const Tensor& like = f->tile_bins;
  Tensor out = out_in ? *out_in : at::empty({h, w, 3}, f32(like));
  Tensor fts = fts_in ? *fts_in : at::empty({h, w}, f32(like));
  Tensor fidx = fidx_in ? *fidx_in : at::empty({h, w}, i32(like));
  raster_forward_into(*f, bg, h, w, out_chw, out, fts, fidx);
  return {out, fts, fidx};
}

// One forward of the drop-in renderer: clamped widths and 1/sigma^2, binning,
// staging and the forward raster, with one read-back of the counts between
// the binning and the raster (none under graph capture).  Returns (out, final_Ts, final_idx, frame,
// widths, inv_sigma2s).
std::tuple<Tensor, Tensor, Tensor, FrameP, Tensor, Tensor> render_forward(
    const Tensor& cubics_norm, const Tensor& offs, const Tensor& colors, const Tensor& opac,
    const Tensor& depths, const OptT& rules, const OptT& stroke_widths, const Tensor& raw_aa,
    const Tensor& bg, const Tensor& basis, int64_t h, int64_t w, int64_t samples,
    double aabb_pad, bool aniso, int64_t r0, int64_t r1, bool dc) {
  c10::cuda::CUDAGuard guard(cubics_norm.device());
  void* st = stream_of(cubics_norm);
  const int64_t p = raw_aa.numel();
  Tensor wbuf = at::empty({2, p}, f32(cubics_norm));
  Tensor widths = wbuf[0], inv_s2 = wbuf[1];
  check(cs_aa_widths_forward(P<float>(raw_aa), P<float>(widths), P<float>(inv_s2), p, st),
        "cs_aa_widths_forward");
  BinInputs in = make_inputs(cubics_norm, offs, depths, widths, inv_s2, colors, opac, rules,
                             stroke_widths, basis, h, w, samples, aabb_pad, aniso, r0, r1, dc);
  Tensor out = at::empty({h, w, 3}, f32(cubics_norm));
  Tensor fts = at::empty({h, w}, f32(cubics_norm));
  Tensor fidx = at::empty({h, w}, i32(cubics_norm));
  Caps c;
  const bool have = cached(in, c);
  if (capturing(in.cubics_norm)) {
    if (!have)
      throw std::runtime_error(
          "the renderer needs one call of this scene size outside CUDA graph capture before "
          "it is captured (intersect buffers are sized from it)");
    FrameP f = bin_attempt(in, c.isect, c.dlist, false);
    raster_forward_into(*f, bg, h, w, OptT(), out, fts, fidx);
    check(cs_poison_on_status(f->status(), P<float>(out), out.numel(), st), "cs_poison_on_status");
    return {out, fts, fidx, f, widths, inv_s2};
  }
  if (!have) {
    FrameP f = bin_attempt(in, 0, 0, true);
    remember(in, f->num_intersects, f->num_records);
    raster_forward_into(*f, bg, h, w, OptT(), out, fts, fidx);
    return {out, fts, fidx, f, widths, inv_s2};
  }
  // The counts are read back as soon as the binning is done, before the
  // raster launch: the host waits for the binning only, and the raster then
  // runs while the caller's next operations are enqueued.
  FrameP f = bin_attempt(in, c.isect, c.dlist, false);
  int64_t n = 0, nd = 0;
  if (!finish_frame(*f, in, n, nd)) {  // outgrew the cached capacity: bin again
    f = bin_attempt(in, size_class(n), size_class(nd), false);
    if (!finish_frame(*f, in, n, nd)) check(CS_ERR_CAPACITY, "cs_bin_count");
  }
  raster_forward_into(*f, bg, h, w, OptT(), out, fts, fidx);  // (background only if n == 0)
  remember(in, n, nd);
  return {out, fts, fidx, f, widths, inv_s2};
}

// Backward raster: (v_edges, v_colors, v_opacities, v_inv_sigma2s,
// v_stroke_widths, curve_contrib_rgb, curve_isect_contrib); the optional ones
// are None when not requested.  With v_output None the image gradient is the
// MSE gradient formed from out_img, target_chw and mse_scale.
std::vector<OptT> raster_backward(const FrameP& fp, int64_t num_primitives, const Tensor& bg,
                                  const Tensor& fts, const Tensor& fidx, const OptT& v_output,
                                  int64_t h, int64_t w, bool collect_contrib,
                                  bool collect_isect_contrib, const OptT& out_img,
                                  const OptT& target_chw, const OptT& mse_scale) {
  Frame& f = *fp;
  c10::cuda::CUDAGuard guard(f.tile_bins.device());
  const Tensor& like = f.tile_bins;
  const int64_t p = num_primitives;
  const int64_t ne = f.edges_px ? f.edges_px->size(0) : 0;
  const int64_t ni = f.rows();
  const int64_t total = ne * 4 + p * 3 + p + p + (f.stroke ? p : 0) +
                        (collect_contrib ? p * 3 : 0) + (collect_isect_contrib ? ni : 0);
  Tensor buf = at::zeros({std::max<int64_t>(total, 1)}, f32(like));
  int64_t o = 0;
  auto take = [&](std::initializer_list<int64_t> shape) {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    Tensor v = buf.narrow(0, o, n).view(shape);
    o += n;
    return v;
  };
  Tensor v_edges = take({ne, 2, 2}), v_colors = take({p, 3}), v_opac = take({p}),
         v_inv = take({p});
  OptT v_sw, contrib, icontrib;
  if (f.stroke) v_sw = take({p});
  if (collect_contrib) contrib = take({p, 3});
  if (collect_isect_contrib) icontrib = take({ni});
  if (ni != 0 && ne > 0) {
    void* st = stream_of(like);
    const Tensor vo = v_output ? as_f32(*v_output) : Tensor();
    const float* vop = v_output ? P<float>(vo) : nullptr;
    const int64_t nt = f.tbx * f.tby;
    Tensor ws = workspace(like, kWsRaster, int64_t(cs_raster_workspace_size(nt)), false);
    const OptT& lists = f.unit_order_bwd ? f.unit_order_bwd : f.unit_order;
    const Tensor bgc = as_f32(bg);
    if (!f.stroke) {
      check(cs_fill_backward(P<int32_t>(f.prim_ids_sorted), P<int32_t>(f.tile_bins),
                             P<int32_t>(f.tile_dlist), P<void>(f.imeta),
                             P<int32_t>(f.isect_strips), P<int32_t>(f.rowoff), P<void>(f.dlist),
                             P<int32_t>(lists), P<int32_t>(f.visit_lists),
                             P<uint16_t>(f.visit_winners), P<float>(bgc), P<float>(fts),
                             P<int32_t>(fidx), vop, P<float>(out_img), P<float>(target_chw),
                             P<float>(mse_scale), P<float>(v_edges), P<float>(v_colors),
                             P<float>(v_opac), P<float>(v_inv), P<float>(contrib),
                             P<float>(icontrib), f.status(), ws.data_ptr(), (int32_t)h,
                             (int32_t)w, (int32_t)f.r0, (int32_t)f.r1, st),
            "cs_fill_backward");
    } else {
      check(cs_stroke_backward(P<int32_t>(f.prim_ids_sorted), P<int32_t>(f.tile_bins),
                               P<int32_t>(f.tile_dlist), P<void>(f.imeta),
                               P<int32_t>(f.isect_strips), P<void>(f.dlist), P<int32_t>(lists),
                               P<int32_t>(f.visit_lists), P<uint16_t>(f.visit_winners),
                               P<float>(bgc), P<float>(fts), P<int32_t>(fidx), vop,
                               P<float>(out_img), P<float>(target_chw), P<float>(mse_scale),
                               P<float>(v_edges), P<float>(v_colors), P<float>(v_opac),
                               P<float>(v_sw), P<float>(v_inv), P<float>(contrib),
                               P<float>(icontrib), f.status(), ws.data_ptr(), (int32_t)h,
                               (int32_t)w, (int32_t)f.r0, (int32_t)f.r1, st),
            "cs_stroke_backward");
    }
  }
  return {v_edges, v_colors, v_opac, v_inv, v_sw, contrib, icontrib};
}

// Edge gradients -> cubic gradients with the frame's flatten method, scaled
// by (sx, sy) (W/2, H/2 gives the normalised-space gradient).
Tensor edge_grads(const FrameP& fp, const Tensor& v_edges, int64_t num_segments, double sx,
                  double sy) {
  const Frame& f = *fp;
  c10::cuda::CUDAGuard guard(v_edges.device());
  Tensor out = at::empty({num_segments, 4, 2}, f32(v_edges));
  if (num_segments <= 0) return out;
  void* st = stream_of(v_edges);
  if (f.flatten_method == "de_casteljau") {
    check(cs_edge_grads_to_cubics_csr(P<float>(v_edges), P<float>(f.edge_t_starts),
                                      P<float>(f.edge_t_ends), P<int32_t>(f.segment_edge_offsets),
                                      P<float>(out), num_segments, (float)sx, (float)sy, st),
          "cs_edge_grads_to_cubics_csr");
  } else {
    check(cs_edge_grads_to_cubics(P<float>(v_edges), P<float>(out), num_segments,
                                  (int32_t)(std::max<int64_t>(2, f.samples) - 1), (float)sx,
                                  (float)sy, st),
          "cs_edge_grads_to_cubics");
  }
  return out;
}

// Clamped widths and 1/sigma^2: clamp(aa, 1e-4), 1 / clamp(w^2, 1e-6).
std::tuple<Tensor, Tensor> aa_widths_forward(const Tensor& raw) {
  c10::cuda::CUDAGuard guard(raw.device());
  const int64_t n = raw.numel();
  Tensor buf = at::empty({2, n}, f32(raw));
  check(cs_aa_widths_forward(P<float>(raw), P<float>(buf[0]), P<float>(buf[1]), n,
                             stream_of(raw)),
        "cs_aa_widths_forward");
  return {buf[0], buf[1]};
}

// Gradient of the raw widths through the clamp of the entry.
Tensor aa_widths_backward(const Tensor& raw, const Tensor& widths, const Tensor& v_inv) {
  c10::cuda::CUDAGuard guard(raw.device());
  const int64_t n = widths.numel();
  Tensor out = at::empty({n}, f32(widths));
  check(cs_aa_widths_backward(P<float>(raw), P<float>(widths), P<float>(v_inv), P<float>(out), n,
                              stream_of(widths)),
        "cs_aa_widths_backward");
  return out;
}

// One backward of the drop-in renderer (no process_fn): (v_cubics scaled by
// (sx, sy), v_colors, v_opacities, v_aa_widths, v_stroke_widths).
std::tuple<Tensor, Tensor, Tensor, Tensor, OptT> render_backward(
    const FrameP& f, int64_t num_primitives, int64_t num_segments, const Tensor& bg,
    const Tensor& fts, const Tensor& fidx, const Tensor& grad_out, const Tensor& raw_aa,
    const Tensor& widths, int64_t h, int64_t w, double sx, double sy) {
  std::vector<OptT> g = raster_backward(f, num_primitives, bg, fts, fidx, grad_out, h, w, false,
                                        false, OptT(), OptT(), OptT());
  Tensor v_cubics = edge_grads(f, *g[0], num_segments, sx, sy);
  Tensor v_aa = aa_widths_backward(raw_aa, widths, *g[3]);
  return {v_cubics, *g[1], *g[2], v_aa, g[4]};
}

// MSE of two float32 CUDA tensors of the same size: a 0-d tensor (and the
// sum of squares into out_sse when given).
Tensor mse_forward(const Tensor& x, const Tensor& y, const OptT& out_sse) {
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t n = x.numel();
  Tensor out = at::empty({}, f32(x));
  Tensor ws = workspace(x, kWsMse, int64_t(cs_mse_workspace_size(n)), false);
  check(cs_mse_forward(P<float>(x), P<float>(y), n, P<float>(out_sse), P<float>(out),
                       ws.data_ptr(), stream_of(x)),
        "cs_mse_forward");
  return out;
}

// grad = scale * factor * (lhs - rhs), scale a device scalar.
Tensor mse_backward(const Tensor& lhs, const Tensor& rhs, const Tensor& scale, double factor) {
  c10::cuda::CUDAGuard guard(lhs.device());
  Tensor grad = at::empty_like(lhs, f32(lhs));
  check(cs_mse_backward(P<float>(lhs), P<float>(rhs), P<float>(scale), (float)factor,
                        P<float>(grad), lhs.numel(), stream_of(lhs)),
        "cs_mse_backward");
  return grad;
}

// Mean SSIM of each [H, W] plane of float32 inputs (optionally the map).
Tensor ssim_planes(const Tensor& x, const Tensor& y, const Tensor& gauss, int64_t planes,
                   int64_t h, int64_t w, int64_t win, double c1, double c2, const OptT& ssim_map) {
  c10::cuda::CUDAGuard guard(x.device());
  Tensor out = at::empty({planes}, f32(x));
  Tensor ws = workspace(x, kWsSsim,
                        int64_t(cs_ssim_workspace_size(planes, (int32_t)h, (int32_t)w, (int32_t)win)),
                        false);
  check(cs_ssim(P<float>(x), P<float>(y), P<float>(gauss), planes, (int32_t)h, (int32_t)w,
                (int32_t)win, (float)c1, (float)c2, P<float>(out), P<float>(ssim_map),
                ws.data_ptr(), stream_of(x)),
        "cs_ssim");
  return out;
}

void forget_capacities() {
  std::lock_guard<std::mutex> lk(g_mu);
  g_caps.clear();
}

PYBIND11_MODULE(_cs_torch, m) {
  m.doc() = "torch binding of the B200 CubicSplat C ABI (one call per autograd stage)";
  py::class_<Frame, FrameP>(m, "Frame")
      .def(py::init<>())
      .def("copy", [](const Frame& f) { return std::make_shared<Frame>(f); })
      .def_readwrite("cubics_px", &Frame::cubics_px)
      .def_readwrite("edges_px", &Frame::edges_px)
      .def_readwrite("prim_edge_offsets", &Frame::prim_edge_offsets)
      .def_readwrite("prim_tile_ranges", &Frame::prim_tile_ranges)
      .def_readwrite("num_tiles_hit", &Frame::num_tiles_hit)
      .def_readwrite("tile_bins", &Frame::tile_bins)
      .def_readwrite("prim_ids_sorted", &Frame::prim_ids_sorted)
      .def_readwrite("isect_ids_sorted", &Frame::isect_ids_sorted)
      .def_readwrite("num_intersects", &Frame::num_intersects)
      .def_readwrite("isect_capacity", &Frame::isect_capacity)
      .def_readwrite("num_records", &Frame::num_records)
      .def_readwrite("samples", &Frame::samples)
      .def_readwrite("tile_dlist", &Frame::tile_dlist)
      .def_readwrite("imeta", &Frame::imeta)
      .def_readwrite("rowoff", &Frame::rowoff)
      .def_readwrite("dlist", &Frame::dlist)
      .def_readwrite("counters", &Frame::counters)
      .def_readwrite("stroke", &Frame::stroke)
      .def_readwrite("isect_strips", &Frame::isect_strips)
      .def_readwrite("unit_order", &Frame::unit_order)
      .def_readwrite("unit_order_bwd", &Frame::unit_order_bwd)
      .def_readwrite("visit_lists", &Frame::visit_lists)
      .def_readwrite("visit_winners", &Frame::visit_winners)
      .def_readwrite("flatten_method", &Frame::flatten_method)
      .def_readwrite("segment_edge_offsets", &Frame::segment_edge_offsets)
      .def_readwrite("edge_t_starts", &Frame::edge_t_starts)
      .def_readwrite("edge_t_ends", &Frame::edge_t_ends)
      .def_property(
          "tile_bounds", [](const Frame& f) { return py::make_tuple(f.tbx, f.tby, 1); },
          [](Frame& f, py::tuple t) {
            f.tbx = t[0].cast<int64_t>();
            f.tby = t[1].cast<int64_t>();
          })
      .def_property(
          "tile_rows", [](const Frame& f) { return py::make_tuple(f.r0, f.r1); },
          [](Frame& f, py::tuple t) {
            f.r0 = t[0].cast<int64_t>();
            f.r1 = t[1].cast<int64_t>();
          });
  m.def("bin_frame", &bin_frame);
  m.def("raster_forward", &raster_forward);
  m.def("render_forward", &render_forward);
  m.def("raster_backward", &raster_backward);
  m.def("render_backward", &render_backward);
  m.def("edge_grads", &edge_grads);
  m.def("aa_widths_forward", &aa_widths_forward);
  m.def("aa_widths_backward", &aa_widths_backward);
  m.def("mse_forward", &mse_forward);
  m.def("mse_backward", &mse_backward);
  m.def("ssim_planes", &ssim_planes);
  m.def("forget_capacities", &forget_capacities);
}
