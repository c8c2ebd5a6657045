"""Device-resident training step for closed cubic fills (the B200-native path).

One step = parameters -> normalised cubics -> fused binning -> forward raster
(which also writes the clamped CHW image) -> MSE and SSIM -> backward raster
with the MSE gradient computed in the kernel -> cubic / ring gradients ->
Adam.  Nothing synchronises with the host, so the whole step can be captured
into one CUDA graph and replayed.  This is the same computation as the
reference's training step (manbo/gaussian_trace/train_ops.py:36-68 with the
cubic_fill renderer, an MSE data loss and SSIM as a forward metric), with the
intersect list sized by a fixed capacity: an overflow is reported through a
device status word (check_status) and never reads or writes out of bounds.

For multi-GPU runs ``tile_rows`` restricts the rank to a band of tile rows and
``grad_hook`` (e.g. an NCCL all-reduce) is applied to the flat gradient buffer
before the optimiser step.
"""
from __future__ import annotations

import math
from typing import Callable, Optional

import torch

from . import _native as nat
from . import metric as _metric
from . import render as _render
from .scenes import FillScene, ring_gather_index

INT64_MAX = (1 << 63) - 1


class FillTrainer:
    """Adam fitting of closed cubic fill paths to a target image on one GPU."""

    def __init__(self, scene: FillScene, device: torch.device, *, lr_points: float = 0.5,
                 lr_colors: float = 0.01, with_ssim: bool = True, capacity: Optional[int] = None,
                 tile_rows: Optional[tuple] = None,
                 grad_hook: Optional[Callable[[torch.Tensor], None]] = None):
        dev = torch.device(device)
        self.device = dev
        self.h, self.w, self.s = int(scene.height), int(scene.width), int(scene.samples)
        self.g_per_path = int(scene.segs_per_path)
        self.num_paths = p = scene.num_paths
        self.num_segments = g = p * self.g_per_path
        tbx, tby, _ = _render.tile_bounds_for(self.h, self.w)
        self.tbx, self.tby = tbx, tby
        self.num_tiles = tbx * tby
        self.tile_rows = (0, tby) if tile_rows is None else (int(tile_rows[0]), int(tile_rows[1]))
        self.with_ssim = bool(with_ssim)
        self.grad_hook = grad_hook

        f32, i32 = torch.float32, torch.int32
        self.ring = scene.ring.to(dev, f32).clone().contiguous()
        self.colors = scene.colors.to(dev, f32).clone().contiguous()
        self.opac = scene.opacities.to(dev, f32).contiguous()
        self.depths = scene.depths.to(dev, f32).contiguous()
        self.rules = scene.fill_rules.to(dev, i32).contiguous()
        self.widths = torch.clamp(scene.aa_widths.to(dev, f32), min=1e-4).contiguous()
        self.inv_s2 = (1.0 / torch.clamp(self.widths * self.widths, min=1e-6)).contiguous()
        self.bg = scene.background.to(dev, f32).contiguous()
        self.offs = scene.seg_offsets().to(dev, i32).contiguous()
        self.edge_offs = (self.offs.to(torch.int64) * (self.s - 1)).to(i32).contiguous()
        self.gidx = ring_gather_index(self.g_per_path).to(dev)
        self.half = torch.tensor([0.5 * self.w, 0.5 * self.h], device=dev, dtype=f32)
        self.target = scene.target.to(dev, f32)[0].contiguous()        # [3, H, W]
        self.basis = _render.bernstein_basis(self.s, dev)

        e = g * (self.s - 1)
        self.cub = torch.empty((p, 4 * self.g_per_path, 2), device=dev, dtype=f32)
        self.cn = torch.empty((g, 4, 2), device=dev, dtype=f32)
        self.cubics_px = torch.empty((g, 4, 2), device=dev, dtype=f32)
        self.edges = torch.empty((e, 2, 2), device=dev, dtype=f32)
        self.prim_ranges = torch.empty((p, 4), device=dev, dtype=i32)
        self.num_hit = torch.empty((p,), device=dev, dtype=i32)
        self.tile_bins = torch.empty((self.num_tiles, 2), device=dev, dtype=i32)
        self.tile_dlist = torch.empty((self.num_tiles, 2), device=dev, dtype=i32)
        # intersects, status, staged-record bound, unused
        self.counters = torch.zeros((4,), device=dev, dtype=i32)
        self.bin_ws = torch.empty((int(nat.call("cs_bin_workspace_size", self.num_tiles)),),
                                  device=dev, dtype=torch.uint8)
        self.out = torch.empty((self.h, self.w, 3), device=dev, dtype=f32)
        self.img_chw = torch.zeros((3, self.h, self.w), device=dev, dtype=f32)
        self.fts = torch.empty((self.h, self.w), device=dev, dtype=f32)
        self.fidx = torch.empty((self.h, self.w), device=dev, dtype=i32)
        self.sse = torch.zeros((3,), device=dev, dtype=f32)
        self.mse = torch.zeros((), device=dev, dtype=f32)
        n_total = 3 * self.h * self.w
        # d loss / d image = 2/N (image - target), in float32 like the reference
        self.mse_scale = (torch.ones((1,), device=dev, dtype=f32) * (2.0 / float(n_total)))
        self.mse_ws = torch.empty((int(nat.call("cs_mse_workspace_size", n_total)),), device=dev,
                                  dtype=torch.uint8)
        self.ssim_planes = torch.zeros((3,), device=dev, dtype=f32)
        self.gauss = _metric.gaussian_1d(11, 1.5, dev)
        self.ssim_ws = torch.empty(
            (int(nat.call("cs_ssim_workspace_size", 3, self.h, self.w, 11)),), device=dev,
            dtype=torch.uint8)

        # raster scratch gradients: v_edges | v_opacity | v_inv_sigma2 (zeroed every step)
        self.scratch = torch.zeros((e * 4 + 2 * p,), device=dev, dtype=f32)
        self.v_edges = self.scratch[:e * 4].view(e, 2, 2)
        self.v_opac = self.scratch[e * 4:e * 4 + p]
        self.v_inv = self.scratch[e * 4 + p:]
        self.v_cn = torch.empty((g, 4, 2), device=dev, dtype=f32)
        self.v_cub = torch.empty((p, 4 * self.g_per_path, 2), device=dev, dtype=f32)
        # parameter gradients live in one flat buffer: ring | colors | band SSE
        n_ring = self.ring.numel()
        self.flat_grad = torch.zeros((n_ring + 3 * p + 1,), device=dev, dtype=f32)
        self.ring.grad = self.flat_grad[:n_ring].view_as(self.ring)
        self.colors.grad = self.flat_grad[n_ring:n_ring + 3 * p].view(p, 3)
        self.sse_slot = self.flat_grad[n_ring + 3 * p:]
        self.ring.requires_grad_(True)
        self.colors.requires_grad_(True)
        self.opt = torch.optim.Adam([{"params": [self.ring], "lr": float(lr_points)},
                                     {"params": [self.colors], "lr": float(lr_colors)}],
                                    fused=True, capturable=True)
        if capacity is None:
            capacity = self.probe_capacity()
        self.capacity, self.dcapacity = (int(c) for c in capacity)
        self.prim_sorted = torch.empty((self.capacity,), device=dev, dtype=i32)
        self.isect_sorted = torch.empty((self.capacity,), device=dev, dtype=torch.int64)
        self.imeta = torch.empty((self.capacity, 12), device=dev, dtype=i32)
        self.rowoff = torch.empty((self.capacity, 16), device=dev, dtype=i32)
        self.dlist = torch.empty((self.dcapacity, 8), device=dev, dtype=f32)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.launches_per_step = 0

    # ------------------------------------------------------------------
    def _params_to_cubics(self):
        with torch.no_grad():
            torch.index_select(self.ring, 1, self.gidx, out=self.cub)
            torch.div(self.cub.view(-1, 4, 2), self.half, out=self.cn)
            self.cn.sub_(1.0)

    def _bin(self, capacity: int, dcapacity: int):
        st = nat.stream(self.device)
        r0, r1 = self.tile_rows
        self.counters.zero_()
        nat.check(nat.call("cs_bin_count", self.cn.data_ptr(), self.offs.data_ptr(),
                           self.widths.data_ptr(), None, self.basis.data_ptr(),
                           self.cubics_px.data_ptr(), self.edges.data_ptr(),
                           self.prim_ranges.data_ptr(), self.num_hit.data_ptr(),
                           self.tile_bins.data_ptr(), self.tile_dlist.data_ptr(),
                           self.counters.data_ptr(), self.bin_ws.data_ptr(), self.num_paths,
                           self.num_segments, capacity, dcapacity, self.s, self.h, self.w, r0, r1,
                           float(_render.DEFAULT_AABB_PAD), 0, st), "cs_bin_count")

    def probe_capacity(self, slack: float = 1.5, extra: int = 4096) -> tuple[int, int]:
        """Intersect and staged-record capacities from one counting pass (one
        host sync, at set-up), with slack for the parameters to move."""
        self._params_to_cubics()
        self._bin(INT64_MAX, INT64_MAX)
        n, _, nd, _ = (int(v) for v in self.counters.tolist())
        return int(math.ceil(n * slack)) + extra, int(math.ceil(nd * slack)) + 16 * extra

    def forward_backward(self):
        """Enqueue one forward + loss + backward; no host synchronisation."""
        st = nat.stream(self.device)
        r0, r1 = self.tile_rows
        self._params_to_cubics()
        self._bin(self.capacity, self.dcapacity)
        status = self.counters.data_ptr() + 4
        nat.check(nat.call("cs_bin_sort", self.prim_ranges.data_ptr(), self.depths.data_ptr(),
                           self.tile_bins.data_ptr(), self.prim_sorted.data_ptr(),
                           self.isect_sorted.data_ptr(), self.counters.data_ptr(),
                           self.bin_ws.data_ptr(), self.num_paths, self.capacity, self.h, self.w,
                           r0, r1, self.edges.data_ptr(), self.edge_offs.data_ptr(),
                           self.colors.data_ptr(), self.opac.data_ptr(), self.inv_s2.data_ptr(),
                           self.rules.data_ptr(), None, self.tile_dlist.data_ptr(),
                           self.imeta.data_ptr(), self.rowoff.data_ptr(), self.dlist.data_ptr(),
                           self.dcapacity, st), "cs_bin_sort")
        nat.check(nat.call("cs_fill_forward", self.prim_sorted.data_ptr(),
                           self.tile_bins.data_ptr(), self.tile_dlist.data_ptr(),
                           self.imeta.data_ptr(), self.rowoff.data_ptr(), self.dlist.data_ptr(),
                           self.bg.data_ptr(), self.out.data_ptr(), self.fts.data_ptr(),
                           self.fidx.data_ptr(), self.img_chw.data_ptr(), status, self.h, self.w,
                           r0, r1, st), "cs_fill_forward")
        self._loss(st)
        self.scratch.zero_()
        self.flat_grad.zero_()
        nat.check(nat.call("cs_fill_backward", self.prim_sorted.data_ptr(),
                           self.tile_bins.data_ptr(), self.tile_dlist.data_ptr(),
                           self.imeta.data_ptr(), self.rowoff.data_ptr(), self.dlist.data_ptr(),
                           self.bg.data_ptr(), self.fts.data_ptr(), self.fidx.data_ptr(), None,
                           self.out.data_ptr(), self.target.data_ptr(),
                           self.mse_scale.data_ptr(), self.v_edges.data_ptr(),
                           self.colors.grad.data_ptr(), self.v_opac.data_ptr(),
                           self.v_inv.data_ptr(), None, None, status, self.h, self.w, r0, r1, st),
                  "cs_fill_backward")
        nat.check(nat.call("cs_edge_grads_to_cubics", self.v_edges.data_ptr(),
                           self.v_cn.data_ptr(), self.num_segments, self.s - 1,
                           0.5 * float(self.w), 0.5 * float(self.h), st),
                  "cs_edge_grads_to_cubics")
        with torch.no_grad():
            # d/d ring of (gather(ring) / half - 1): scatter-add of grad / half
            torch.div(self.v_cn.view(self.num_paths, -1, 2), self.half, out=self.v_cub)
            self.ring.grad.index_add_(1, self.gidx, self.v_cub)
            self.sse_slot.copy_(self.sse.sum().view(1))
        self.launches_per_step = 9 + (2 if self.with_ssim else 0) + (
            2 if self.tile_rows != (0, self.tby) else 0)

    def _loss(self, st):
        r0, r1 = self.tile_rows
        hw = self.h * self.w
        if self.tile_rows == (0, self.tby):
            nat.check(nat.call("cs_mse_forward", self.img_chw.data_ptr(), self.target.data_ptr(),
                               3 * hw, self.sse.data_ptr(), self.mse.data_ptr(),
                               self.mse_ws.data_ptr(), st), "cs_mse_forward")
            if self.with_ssim:
                nat.check(nat.call("cs_ssim", self.img_chw.data_ptr(), self.target.data_ptr(),
                                   self.gauss.data_ptr(), 3, self.h, self.w, 11, 0.01 ** 2,
                                   0.03 ** 2, self.ssim_planes.data_ptr(), None,
                                   self.ssim_ws.data_ptr(), st), "cs_ssim")
        else:
            # band: SSE of this rank's rows, one contiguous span per channel
            y0, y1 = r0 * 16, min(self.h, r1 * 16)
            n = (y1 - y0) * self.w
            self.sse.zero_()
            for c in range(3):
                off = 4 * (c * hw + y0 * self.w)
                nat.check(nat.call("cs_mse_forward", self.img_chw.data_ptr() + off,
                                   self.target.data_ptr() + off, n, self.sse.data_ptr() + 4 * c,
                                   None, self.mse_ws.data_ptr(), st), "cs_mse_forward")

    def optimizer_step(self):
        if self.grad_hook is not None:
            self.grad_hook(self.flat_grad)
        self.opt.step()

    def step_eager(self):
        self.forward_backward()
        self.optimizer_step()

    def capture(self, warmup: int = 3):
        """Capture one full training step into a CUDA graph."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step_eager()
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step_eager()
        return self.graph

    def step(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self.step_eager()

    # ------------------------------------------------------------------
    def check_status(self) -> tuple[int, int]:
        """(intersect count of the last step, device status); syncs."""
        n, status, _, _ = (int(v) for v in self.counters.tolist())
        return n, status

    def loss_value(self) -> float:
        return float(self.mse)

    def ssim_value(self) -> float:
        return float(self.ssim_planes.mean())
