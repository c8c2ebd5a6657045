"""Device-resident training step for closed cubic fills (the B200-native path).

One step, all on the device and capturable as one CUDA graph:

  ring params -> projection, AABB, flatten,
  tile counts, scans                             cs_bin_count (reads the ring)
  scatter, per-tile sort, edge staging           cs_bin_sort
  forward raster + clamped CHW image + MSE loss  cs_fill_forward (target given)
  SSIM (forward metric)                          cs_ssim
  backward raster with the MSE gradient inside   cs_fill_backward (v_output NULL)
  edge -> ring gradients (clears edge grads)     cs_edge_grads_to_ring
  Adam on [ring | colours] (clears grads)        cs_adam_step

This is the reference's training step (manbo/gaussian_trace/train_ops.py:36-68
with the cubic_fill renderer, an MSE data loss and SSIM as a forward metric)
with Adam (lr 0.5 on points, 0.01 on colours).  Gradient buffers are cleared
by the kernels that consume them, so no memset is needed between steps.  The
intersect list and staged edge records use fixed capacities: an overflow is
recorded in a sticky device status word (check_status) and never reads or
writes out of bounds.

For multi-GPU runs ``tile_rows`` restricts the rank to a band of tile rows and
``grad_hook`` (e.g. an NCCL all-reduce) is applied to the flat buffer
[ring grads | colour grads | sse, mse | SSIM sums of the three planes] before
the optimiser step.  SSIM on a band needs the next band's first win - 1 rows
(``halo_gather``, e.g. repo_b200.bands.allgather_halo): the band's SSIM runs on
its own rows plus that halo on the side stream, and its per-plane sums join
the gradients in the same all-reduce.
"""
from __future__ import annotations

import math
from typing import Callable, Optional

import torch

from . import _native as nat
from . import metric as _metric
from . import render as _render
from .scenes import FillScene

INT64_MAX = (1 << 63) - 1


class FillTrainer:
    """Adam fitting of closed cubic fill paths to a target image on one GPU."""

    def __init__(self, scene: FillScene, device: torch.device, *, lr_points: float = 0.5,
                 lr_colors: float = 0.01, with_ssim: bool = True, capacity=None,
                 tile_rows: Optional[tuple] = None,
                 grad_hook: Optional[Callable[[torch.Tensor], None]] = None,
                 halo_gather: Optional[Callable[[torch.Tensor], Optional[torch.Tensor]]] = None,
                 peer_group=None, betas=(0.9, 0.999), eps: float = 1e-8):
        dev = torch.device(device)
        self.device = dev
        self.h, self.w, self.s = int(scene.height), int(scene.width), int(scene.samples)
        self.g_per_path = G = int(scene.segs_per_path)
        self.num_paths = p = scene.num_paths
        self.num_segments = g = p * G
        tbx, tby, _ = _render.tile_bounds_for(self.h, self.w)
        self.tbx, self.tby = tbx, tby
        self.num_tiles = nt = tbx * tby
        self.tile_rows = (0, tby) if tile_rows is None else (int(tile_rows[0]), int(tile_rows[1]))
        self.with_ssim = bool(with_ssim)
        self.band_ssim = self.with_ssim and self.tile_rows != (0, tby)
        if peer_group is not None and (grad_hook is not None or halo_gather is not None):
            raise ValueError("peer_group replaces grad_hook and halo_gather: pass one or the other")
        if self.band_ssim and halo_gather is None and peer_group is None:
            # a band renders only its own rows; the SSIM window also reads the
            # next band's first rows
            raise ValueError("with_ssim=True on a band of tile rows needs halo_gather (the next "
                             "band's first rows, e.g. repo_b200.bands.allgather_halo); or pass "
                             "with_ssim=False")
        self.halo_gather = halo_gather
        self.grad_hook = grad_hook
        self.lr = (float(lr_points), float(lr_colors))
        self.betas, self.eps = (float(betas[0]), float(betas[1])), float(eps)

        f32, i32 = torch.float32, torch.int32
        n_ring = p * 3 * G * 2
        self.n_ring = n_ring
        self.n_params = n_ring + 3 * p
        # parameters [ring | colours], Adam moments, gradients [.. | sse, mse]
        self.params = torch.cat([scene.ring.reshape(-1), scene.colors.reshape(-1)]).to(dev, f32)
        self.ring = self.params[:n_ring].view(p, 3 * G, 2)
        self.colors = self.params[n_ring:].view(p, 3)
        self.exp_avg = torch.zeros_like(self.params)
        self.exp_avg_sq = torch.zeros_like(self.params)
        # [primitive gradients | sse, mse of this rank's tiles | per-plane SSIM
        # sums of its band]; with a peer group, two buffers in its symmetric
        # memory (step t writes buffer t % 2) and the reduced tail in self.tail
        self.peer = None
        if peer_group is not None:
            from .peer import PeerGroup
            self.peer = PeerGroup(peer_group, dev, self.n_params + 5, (3, 10, self.w))
            self._grad_bufs = self.peer.grads
        else:
            self._grad_bufs = [torch.zeros((self.n_params + 5,), device=dev, dtype=f32)]
        self.tail = torch.zeros((5,), device=dev, dtype=f32)
        self._t = 0  # steps enqueued (host count; selects the gradient buffer)
        self._set_parity(0)
        self.step_count = torch.zeros((1,), device=dev, dtype=i32)
        self.adam_ws = torch.zeros((int(nat.call("cs_adam_workspace_size")),), device=dev,
                                   dtype=torch.uint8)

        self.opac = scene.opacities.to(dev, f32).contiguous()
        self.depths = scene.depths.to(dev, f32).contiguous()
        self.rules = scene.fill_rules.to(dev, i32).contiguous()
        self.widths = torch.clamp(scene.aa_widths.to(dev, f32), min=1e-4).contiguous()
        self.inv_s2 = (1.0 / torch.clamp(self.widths * self.widths, min=1e-6)).contiguous()
        self.bg = scene.background.to(dev, f32).contiguous()
        self.offs = scene.seg_offsets().to(dev, i32).contiguous()
        self.edge_offs = (self.offs.to(torch.int64) * (self.s - 1)).to(i32).contiguous()
        self.target = scene.target.to(dev, f32)[0].contiguous()        # [3, H, W]
        self.basis = _render.bernstein_basis(self.s, dev)

        e = g * (self.s - 1)
        self.cubics_px = torch.empty((g, 4, 2), device=dev, dtype=f32)
        self.edges = torch.empty((e, 2, 2), device=dev, dtype=f32)
        self.v_edges = torch.zeros((e, 2, 2), device=dev, dtype=f32)
        self.prim_ranges = torch.empty((p, 4), device=dev, dtype=i32)
        self.num_hit = torch.empty((p,), device=dev, dtype=i32)
        self.tile_bins = torch.empty((nt, 2), device=dev, dtype=i32)
        self.tile_dlist = torch.empty((nt, 2), device=dev, dtype=i32)
        # dispatch lists of the band's strips (4 per tile), heaviest bucket first
        band_tiles = max(1, (self.tile_rows[1] - self.tile_rows[0]) * tbx)
        self.unit_order = torch.empty((int(nat.call("cs_unit_lists_size", band_tiles)) // 4,),
                                      device=dev, dtype=i32)
        self.unit_order_bwd = torch.empty_like(self.unit_order)  # filled by the forward
        # intersects, sticky status, staged-record bound, unused
        self.counters = torch.zeros((4,), device=dev, dtype=i32)
        # zeroed once: every cs_bin_count leaves its counters zeroed again
        self.bin_ws = torch.zeros((int(nat.call("cs_bin_workspace_size", nt)),), device=dev,
                                  dtype=torch.uint8)
        self.raster_ws = torch.zeros((int(nat.call("cs_raster_workspace_size", nt)),), device=dev,
                                   dtype=torch.uint8)
        self.out = torch.empty((self.h, self.w, 3), device=dev, dtype=f32)
        self.img_chw = torch.zeros((3, self.h, self.w), device=dev, dtype=f32)
        self.fts = torch.empty((self.h, self.w), device=dev, dtype=f32)
        self.fidx = torch.empty((self.h, self.w), device=dev, dtype=i32)
        n_total = 3 * self.h * self.w
        # d loss / d image = 2/N (image - target), in float32 like the reference
        self.mse_scale = torch.ones((1,), device=dev, dtype=f32) * (2.0 / float(n_total))
        self.ssim_planes = torch.zeros((3,), device=dev, dtype=f32)
        self.gauss = _metric.gaussian_1d(11, 1.5, dev)
        win = 11
        self.ssim_total = float((self.h - win + 1) * (self.w - win + 1))
        ssim_h = self.h
        if self.band_ssim:
            # the band's pixel rows [y0, y1), plus the next band's first rows
            y0 = self.tile_rows[0] * _render.BLOCK_Y
            y1 = min(self.tile_rows[1] * _render.BLOCK_Y, self.h)
            self.band_px = (y0, y1)
            self.halo = max(0, min(win - 1, self.h - y1))
            ssim_h = (y1 - y0) + self.halo
            self.ssim_count = float(max(0, ssim_h - win + 1) * (self.w - win + 1))
            self.ssim_in = torch.zeros((3, ssim_h, self.w), device=dev, dtype=f32)
            self.ssim_tgt = self.target[:, y0:y0 + ssim_h, :].contiguous()
            self.halo_send = torch.zeros((3, win - 1, self.w), device=dev, dtype=f32)
        self.ssim_h = ssim_h
        self.ssim_ws = torch.zeros(
            (int(nat.call("cs_ssim_workspace_size", 3, ssim_h, self.w, win)),), device=dev,
            dtype=torch.uint8)
        if capacity is None:
            capacity = self.probe_capacity()
        self.capacity, self.dcapacity = (int(c) for c in capacity)
        self.prim_sorted = torch.empty((self.capacity,), device=dev, dtype=i32)
        self.isect_sorted = torch.empty((self.capacity,), device=dev, dtype=torch.int64)
        self.imeta = torch.empty((self.capacity, 12), device=dev, dtype=i32)
        self.rowoff = torch.empty((self.capacity, 16), device=dev, dtype=i32)
        self.istrips = torch.empty((self.capacity, 4, 2), device=dev, dtype=i32)
        self.dlist = torch.empty((self.dcapacity, 8), device=dev, dtype=f32)
        self.visits = torch.empty(
            (int(nat.call("cs_visit_lists_size", self.capacity, self.tile_bins.shape[0])) // 4,),
            device=dev, dtype=i32)
        self.winners = torch.empty(
            (int(nat.call("cs_visit_winners_size", self.capacity, self.tile_bins.shape[0])) // 2,),
            device=dev, dtype=torch.int16)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        # SSIM runs beside the backward at low priority, so that it takes only
        # the SMs the backward leaves free; the step itself is captured on a
        # high-priority stream
        lo, hi = torch.cuda.Stream.priority_range()
        self._side = torch.cuda.Stream(dev, priority=lo)
        self._main = torch.cuda.Stream(dev, priority=hi)
        self._fork = torch.cuda.Event()
        self._join = torch.cuda.Event()
        self.launches_per_step = 7 + (1 if self.with_ssim else 0)
        if self.peer is not None:  # grads signal; halo signal and wait-copy of band SSIM
            rank, world = self.peer.rank, self.peer.world
            self.launches_per_step += 1
            if self.band_ssim:
                self.launches_per_step += (1 if rank > 0 else 0) + (1 if self.halo > 0 else 0)
        self.graphs = None
        self._timing = None  # CUDA events around the raster launches (enable_kernel_timing)

    def enable_kernel_timing(self):
        """Record timing events around the forward and backward raster
        launches, also inside a captured graph (external events, so that each
        replay re-records them): kernel_times() reads the last step's."""
        self._timing = tuple(torch.cuda.Event(enable_timing=True, external=True)
                             for _ in range(4))

    def kernel_times(self) -> tuple[float, float]:
        """(forward, backward) raster launch times of the last step in ms
        (after enable_kernel_timing; synchronises)."""
        ev = self._timing
        ev[3].synchronize()
        return ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3])

    # ------------------------------------------------------------------
    def _bin(self, capacity: int, dcapacity: int, st):
        """Projection, flattening, tile counts and scans, reading the control
        points straight from the ring parameters."""
        r0, r1 = self.tile_rows
        nat.check(nat.call("cs_bin_count", None, self.offs.data_ptr(),
                           self.widths.data_ptr(), None, self.basis.data_ptr(),
                           self.cubics_px.data_ptr(), self.edges.data_ptr(), None, None,
                           self.prim_ranges.data_ptr(), self.num_hit.data_ptr(),
                           self.tile_bins.data_ptr(), self.tile_dlist.data_ptr(),
                           self.counters.data_ptr(), self.bin_ws.data_ptr(), self.num_paths,
                           self.num_segments, capacity, dcapacity, self.s, self.h, self.w, r0, r1,
                           float(_render.DEFAULT_AABB_PAD), 0, self.ring.data_ptr(),
                           self.g_per_path, st), "cs_bin_count")

    def probe_capacity(self, slack: float = 1.5, extra: int = 4096) -> tuple[int, int]:
        """Intersect and staged-record capacities from one counting pass (one
        host sync, at set-up), with slack for the parameters to move."""
        st = nat.stream(self.device)
        self._bin(INT64_MAX, INT64_MAX, st)
        n, _, nd, _ = (int(v) for v in self.counters.tolist())
        return int(math.ceil(n * slack)) + extra, int(math.ceil(nd * slack)) + 64 * extra

    def forward_backward(self, join: bool = True):
        """Enqueue one forward + loss + backward; no host synchronisation.  The
        SSIM side stream is joined back unless join is False (the caller then
        calls _join_side once the rest of its step is enqueued)."""
        st = nat.stream(self.device)
        r0, r1 = self.tile_rows
        status = self.counters.data_ptr() + 4
        self._bin(self.capacity, self.dcapacity, st)
        nat.check(nat.call("cs_bin_sort", self.prim_ranges.data_ptr(), self.depths.data_ptr(),
                           self.tile_bins.data_ptr(), self.prim_sorted.data_ptr(),
                           self.isect_sorted.data_ptr(), self.counters.data_ptr(),
                           self.bin_ws.data_ptr(), self.num_paths, self.capacity, self.h, self.w,
                           r0, r1, self.edges.data_ptr(), self.edge_offs.data_ptr(),
                           self.colors.data_ptr(), self.opac.data_ptr(), self.inv_s2.data_ptr(),
                           self.rules.data_ptr(), None, self.tile_dlist.data_ptr(),
                           self.imeta.data_ptr(), self.rowoff.data_ptr(), self.istrips.data_ptr(),
                           self.dlist.data_ptr(), self.dcapacity, self.unit_order.data_ptr(), st),
                  "cs_bin_sort")
        ev = self._timing
        if ev is not None:
            ev[0].record()
        nat.check(nat.call("cs_fill_forward", self.prim_sorted.data_ptr(),
                           self.tile_bins.data_ptr(), self.tile_dlist.data_ptr(),
                           self.imeta.data_ptr(), self.istrips.data_ptr(), self.rowoff.data_ptr(),
                           self.dlist.data_ptr(), self.unit_order.data_ptr(),
                           self.unit_order_bwd.data_ptr(), self.visits.data_ptr(),
                           self.winners.data_ptr(), self.bg.data_ptr(), self.out.data_ptr(),
                           self.fts.data_ptr(),
                           self.fidx.data_ptr(),
                           self.img_chw.data_ptr(), self.target.data_ptr(), self.loss.data_ptr(),
                           status, self.raster_ws.data_ptr(), self.h, self.w, r0, r1, st),
                  "cs_fill_forward")
        if ev is not None:
            ev[1].record()
        if self.with_ssim:
            # SSIM needs only the forward's image: it runs on a side stream
            # beside the backward and fills the SMs the backward leaves idle
            main = torch.cuda.current_stream(self.device)
            self._fork.record(main)
            self._side.wait_event(self._fork)
            if self.band_ssim:
                with torch.cuda.stream(self._side):
                    self._band_ssim()
            else:
                nat.check(nat.call("cs_ssim", self.img_chw.data_ptr(), self.target.data_ptr(),
                                   self.gauss.data_ptr(), 3, self.h, self.w, 11, 0.01 ** 2,
                                   0.03 ** 2, self.ssim_planes.data_ptr(), None,
                                   self.ssim_ws.data_ptr(), self._side.cuda_stream), "cs_ssim")
            self._join.record(self._side)
        if ev is not None:
            ev[2].record()
        nat.check(nat.call("cs_fill_backward", self.prim_sorted.data_ptr(),
                           self.tile_bins.data_ptr(), self.tile_dlist.data_ptr(),
                           self.imeta.data_ptr(), self.istrips.data_ptr(), self.rowoff.data_ptr(),
                           self.dlist.data_ptr(), self.unit_order_bwd.data_ptr(),
                           self.visits.data_ptr(), self.winners.data_ptr(), self.bg.data_ptr(),
                           self.fts.data_ptr(),
                           self.fidx.data_ptr(), None,
                           self.out.data_ptr(),
                           self.target.data_ptr(), self.mse_scale.data_ptr(),
                           self.v_edges.data_ptr(), self.v_colors.data_ptr(), None, None, None,
                           None, status, self.raster_ws.data_ptr(), self.h, self.w, r0, r1, st),
                  "cs_fill_backward")
        if ev is not None:
            ev[3].record()
        nat.check(nat.call("cs_edge_grads_to_ring", self.v_edges.data_ptr(),
                           self.v_ring.data_ptr(), self.num_paths, self.g_per_path, self.s - 1,
                           self.h, self.w, 1, self.prim_ranges.data_ptr(), r0, r1, st),
                  "cs_edge_grads_to_ring")
        if join:
            self._join_side()

    def _set_parity(self, parity: int):
        """Point the gradient views at buffer `parity` (one buffer without a
        peer group)."""
        self._parity = parity if len(self._grad_bufs) > 1 else 0
        fg = self._grad_bufs[self._parity]
        n_ring, n = self.n_ring, self.n_params
        self.flat_grad = fg
        self.v_ring = fg[:n_ring]
        self.v_colors = fg[n_ring:n]
        self.loss = fg[n:n + 2]
        self.ssim_sums = fg[n + 2:]

    def _band_ssim(self):
        """SSIM of this band (on the current stream): its first rows go to
        the other bands, the next band's first rows extend its own, and the
        SSIM of the extended rows gives the band's per-plane output sums."""
        y0, y1 = self.band_px
        rows = y1 - y0
        send = min(rows, self.halo_send.shape[1])
        if self.peer is not None:
            # my first rows into my halo region, a flag to the previous band,
            # then the next band's rows read through its peer pointer
            pg = self.peer
            pg.halo[:, :send].copy_(self.img_chw[:, y0:y0 + send])
            if pg.rank > 0:
                pg.signal(1, self.step_count, only_peer=pg.rank - 1)
            self.ssim_in[:, :rows].copy_(self.img_chw[:, y0:y1])
            if self.halo > 0:
                pg.wait_copy(1, pg.rank + 1, self.step_count, self.counters[1:2],
                             pg.halo_ptrs[pg.rank + 1], pg.halo_shape[1] * self.w, self.ssim_in,
                             rows * self.w, self.ssim_h * self.w, self.halo * self.w, 3)
        else:
            self.halo_send[:, :send].copy_(self.img_chw[:, y0:y0 + send])
            recv = self.halo_gather(self.halo_send)  # every band takes part
            self.ssim_in[:, :rows].copy_(self.img_chw[:, y0:y1])
            if self.halo > 0:
                self.ssim_in[:, rows:].copy_(recv[:, :self.halo])
        if self.ssim_count > 0:
            nat.check(nat.call("cs_ssim", self.ssim_in.data_ptr(), self.ssim_tgt.data_ptr(),
                               self.gauss.data_ptr(), 3, self.ssim_h, self.w, 11, 0.01 ** 2,
                               0.03 ** 2, self.ssim_planes.data_ptr(), None,
                               self.ssim_ws.data_ptr(), nat.stream(self.device)), "cs_ssim")
            torch.mul(self.ssim_planes, self.ssim_count, out=self.ssim_sums)
        else:
            self.ssim_sums.zero_()

    def _join_side(self):
        if self.with_ssim:
            torch.cuda.current_stream(self.device).wait_event(self._join)

    def optimizer_step(self):
        if self.band_ssim:
            self._join_side()  # the band's SSIM sums travel with the gradients
        if self.grad_hook is not None:
            self.grad_hook(self.flat_grad)
        if self.peer is not None:
            # every rank's gradients (and loss / SSIM sums) through peer
            # memory, summed in rank order, then Adam: one kernel
            self.peer.signal(0, self.step_count)
            self.peer.allreduce_adam(self._parity, self.params, self.exp_avg, self.exp_avg_sq,
                                     self.n_params, self.n_ring, 5, self.tail, self.lr, self.betas,
                                     self.eps, self.step_count, self.counters[1:2])
            return
        nat.check(nat.call("cs_adam_step", self.params.data_ptr(), self.flat_grad.data_ptr(),
                           self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(), self.n_params,
                           self.n_ring, self.lr[0], self.lr[1], self.betas[0], self.betas[1],
                           self.eps, self.step_count.data_ptr(), self.adam_ws.data_ptr(), 1,
                           nat.stream(self.device)), "cs_adam_step")

    def _enqueue(self, parity: int):
        # SSIM overlaps the backward, the edge-to-ring pass and the optimiser
        # step (with a peer group it joins before the gradient exchange,
        # which carries its sums); the step ends when it is done
        self._set_parity(parity)
        self.forward_backward(join=False)
        self.optimizer_step()
        self._join_side()

    def _next_parity(self) -> int:
        return (self._t + 1) % 2

    def step_eager(self):
        self._enqueue(self._next_parity())
        self._t += 1

    def capture(self, warmup: int = 3):
        """Capture one full training step into a CUDA graph (with a peer
        group, one graph per gradient buffer, replayed alternately)."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step_eager()
        torch.cuda.current_stream(self.device).wait_stream(side)
        parities = (0, 1) if self.peer is not None else (0,)
        graphs = []
        for parity in parities:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self._main):
                self._enqueue(parity)
            graphs.append(g)
        self.graphs = graphs
        self.graph = graphs[0]
        return self.graph

    def step(self):
        if self.graphs is not None:
            self.graphs[self._next_parity() if len(self.graphs) > 1 else 0].replay()
            self._t += 1
        else:
            self.step_eager()

    def release_graphs(self):
        """Drop the captured graphs (before the process group they may hold
        collectives of goes away)."""
        self.graphs = None
        self.graph = None

    # ------------------------------------------------------------------
    def check_status(self) -> tuple[int, int]:
        """(intersect count of the last step, sticky device status); syncs."""
        n, status, _, _ = (int(v) for v in self.counters.tolist())
        return n, status

    def loss_value(self) -> float:
        """MSE of the last step (with a peer group, summed over the bands)."""
        if self.peer is not None:
            return float(self.tail[1])
        return float(self.loss[1])

    def ssim_value(self) -> float:
        """SSIM of the last step: the mean over planes of each plane's mean
        (in band mode, of the all-reduced per-plane sums)."""
        if self.band_ssim:
            sums = self.tail[2:5] if self.peer is not None else self.ssim_sums
            return float((sums / self.ssim_total).mean())
        return float(self.ssim_planes.mean())
