"""Tile-row bands: one large image rendered and optimised across several GPUs.

Every rank holds all primitive parameters, projects and flattens every
primitive (cheap), but bins, rasterises and back-propagates only the tiles of
its band of tile rows.  The partial gradients of all primitives (plus the
band's sum of squared differences) sit in one flat float32 buffer per rank;
one all-reduce (SUM) per step makes them the full-image gradient on every
rank, and the replicated Adam step keeps the parameters identical.  The MSE is
normalised by the whole image's element count on every rank, so the sum of
the band gradients is exactly the full-image gradient up to summation order.

Bands are balanced by a per-tile-row work estimate (edge slots + 8 per
intersect, from one binning pass of the starting scene).

In the fused training step (repo_b200.train.FillTrainer) the band's first
win - 1 rows reach the previous band by one all-gather (allgather_halo) and
the band's per-plane SSIM sums ride in the gradient all-reduce.

SSIM over bands (band_ssim_sums): the valid-window SSIM output of row y reads
input rows [y, y + win - 1], so a band owning pixel rows [y0, y1) produces the
outputs of rows [y0, min(y1, H - win + 1)) from its own rows plus the first
win - 1 rows of the next band (the halo, one point-to-point transfer per
band boundary); the per-plane sums of the bands' outputs then add up
(all-reduce) to the whole image's (manbo/metric.py:215-273 takes the mean of
each plane's map, then over planes).
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch

from . import render as _render
from .scenes import FillScene


def balanced_bands(row_work: Sequence[float], parts: int) -> List[Tuple[int, int]]:
    """Split rows [0, len(row_work)) into `parts` contiguous bands [r0, r1)
    minimising the largest band's work (exact, by dynamic programming over
    prefix sums).  Every band is non-empty when there are at least `parts`
    rows; otherwise the trailing bands are empty."""
    n = len(row_work)
    parts = int(parts)
    if parts <= 0:
        raise ValueError("parts must be >= 1")
    if n == 0:
        return [(0, 0)] * parts
    k = min(parts, n)
    pre = [0.0]
    for v in row_work:
        pre.append(pre[-1] + max(0.0, float(v)) + 1e-9)  # tiny per-row cost: no free rows
    inf = float("inf")
    # best[j][i]: minimal max-load splitting rows [0, i) into j non-empty bands
    best = [[inf] * (n + 1) for _ in range(k + 1)]
    cut = [[0] * (n + 1) for _ in range(k + 1)]
    best[0][0] = 0.0
    for j in range(1, k + 1):
        for i in range(j, n + 1):
            for m in range(j - 1, i):
                c = max(best[j - 1][m], pre[i] - pre[m])
                if c < best[j][i]:
                    best[j][i], cut[j][i] = c, m
    bounds = []
    i = n
    for j in range(k, 0, -1):
        m = cut[j][i]
        bounds.append((m, i))
        i = m
    bounds.reverse()
    return bounds + [(n, n)] * (parts - k)


def tile_row_work(scene: FillScene, device: torch.device) -> List[float]:
    """Work estimate of every tile row of a fill scene: the edge slots (every
    edge of every primitive on a tile) plus 8 per intersect, summed over the
    row's tiles, from one binning pass (one host synchronisation)."""
    dev = torch.device(device)
    h, w = int(scene.height), int(scene.width)
    widths = torch.clamp(scene.aa_widths.to(dev, torch.float32), min=1e-4)
    b = _render.bin_primitives(
        scene.cubics_norm().to(dev), scene.seg_offsets().to(dev), scene.depths.to(dev), widths,
        h, w, scene.samples, colors=scene.colors.to(dev), opacities=scene.opacities.to(dev),
        inv_sigma2s=_render._inv_sigma2(widths), fill_rules=scene.fill_rules.to(dev))
    tbx, tby, _ = b.tile_bounds
    bins = b.tile_bins.view(tby, tbx, 2).to(torch.int64)
    slots = b.tile_dlist.view(tby, tbx, 2)[..., 1].to(torch.int64)
    work = (bins[..., 1] - bins[..., 0]) * 8 + slots
    return [float(v) for v in work.sum(dim=1).cpu().tolist()]


def band_for_rank(scene: FillScene, device: torch.device, rank: int, world: int,
                  row_work: Optional[Sequence[float]] = None) -> Tuple[int, int]:
    """This rank's band of tile rows (the same split on every rank)."""
    if row_work is None:
        row_work = tile_row_work(scene, device)
    return balanced_bands(row_work, world)[rank]


def allreduce_hook(group=None) -> Callable[[torch.Tensor], None]:
    """Gradient hook for FillTrainer: all-reduce (SUM) of the flat buffer
    [primitive gradients | band SSE, band MSE] over the process group."""
    import torch.distributed as dist

    def hook(flat: torch.Tensor) -> None:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)

    return hook


def allgather_halo(rank: int, world: int, group=None
                   ) -> Callable[[torch.Tensor], Optional[torch.Tensor]]:
    """halo_gather for FillTrainer's band SSIM: every rank contributes the
    first rows of its band ([C, win - 1, W], one all-gather over the process
    group, capturable in a CUDA graph) and gets back the next rank's, or None
    on the last rank.  Rank i owns band i."""
    import torch.distributed as dist
    bufs = {}

    def gather(send: torch.Tensor) -> Optional[torch.Tensor]:
        key = (send.device, tuple(send.shape))
        out = bufs.get(key)
        if out is None:  # allocated on the first (eager) call, reused afterwards
            # the ranks' tensors concatenated along dim 0 (both NCCL and gloo)
            shape = (world * send.shape[0],) + tuple(send.shape[1:])
            out = torch.empty(shape, dtype=send.dtype, device=send.device)
            bufs[key] = out
        dist.all_gather_into_tensor(out, send, group=group)
        c = send.shape[0]
        return out[(rank + 1) * c:(rank + 2) * c] if rank + 1 < world else None

    return gather


def ssim_halo_rows(bands_px: Sequence[Tuple[int, int]], index: int, height: int,
                   win_size: int) -> int:
    """Rows the band `index` of pixel-row bands `bands_px` (contiguous,
    covering [0, height) in order) needs from the next band: win_size - 1,
    fewer at the bottom of the image, none for an empty band."""
    y0, y1 = bands_px[index]
    if y1 <= y0:
        return 0
    need = min(win_size - 1, height - y1)
    if need > 0:
        nxt = bands_px[index + 1] if index + 1 < len(bands_px) else (y1, y1)
        if nxt[0] != y1 or nxt[1] - nxt[0] < need:
            raise ValueError(f"band {index} needs {need} halo rows from the next band, "
                             f"which has {max(0, nxt[1] - nxt[0])}")
    return max(0, need)


def exchange_ssim_halo(img_chw: torch.Tensor, bands_px: Sequence[Tuple[int, int]], rank: int,
                       win_size: int, group=None) -> torch.Tensor:
    """This rank's rows of img_chw [C, H, W] (full-size buffer; only the band's
    rows are read) extended by the next band's first rows: [C, rows + halo, W].
    Every rank sends its first rows to the previous rank and receives the
    next rank's (torch.distributed point-to-point; rank i owns band i).  A
    rank with neither (an empty band) makes no call, so with NCCL some
    collective must have run on the group before (NCCL's batched
    point-to-point needs every rank in its first call)."""
    import torch.distributed as dist

    c, h, w = img_chw.shape
    y0, y1 = bands_px[rank]
    ops = []
    recv = None
    halo = ssim_halo_rows(bands_px, rank, h, win_size)
    if halo > 0:
        recv = torch.empty((c, halo, w), dtype=img_chw.dtype, device=img_chw.device)
        ops.append(dist.P2POp(dist.irecv, recv, rank + 1, group))
    send = None
    if rank > 0:
        prev_halo = ssim_halo_rows(bands_px, rank - 1, h, win_size)
        if prev_halo > 0:
            send = img_chw[:, y0:y0 + prev_halo, :].contiguous()
            ops.append(dist.P2POp(dist.isend, send, rank - 1, group))
    if ops:
        for work in dist.batch_isend_irecv(ops):
            work.wait()
    own = img_chw[:, y0:y1, :]
    return torch.cat([own, recv], dim=1) if recv is not None else own.contiguous()


def band_ssim_sums(img_ext: torch.Tensor, target_chw: torch.Tensor, y0: int, win_size: int,
                   plane_means: Callable[[torch.Tensor, torch.Tensor], torch.Tensor]
                   ) -> torch.Tensor:
    """Per-plane sums of the SSIM outputs a band owns, from its rows extended
    by the halo (exchange_ssim_halo) and the matching target rows.
    plane_means(x, y) returns the mean of each plane's valid SSIM map of
    [C, rows, W] inputs (metric.ssim_per_plane on the GPU)."""
    c, rows, w = img_ext.shape
    out_rows, out_cols = rows - win_size + 1, w - win_size + 1
    if out_rows <= 0 or out_cols <= 0:
        return torch.zeros((c,), dtype=torch.float64, device=img_ext.device)
    tgt = target_chw[:, y0:y0 + rows, :].contiguous()
    means = plane_means(img_ext.contiguous(), tgt).to(torch.float64)
    return means * float(out_rows * out_cols)


def band_ssim(img_chw: torch.Tensor, target_chw: torch.Tensor,
              bands_px: Sequence[Tuple[int, int]], rank: int, *, win_size: int = 11,
              win_sigma: float = 1.5, k1: float = 0.01, k2: float = 0.03,
              data_range: float = 1.0, plane_means=None, group=None) -> torch.Tensor:
    """Whole-image SSIM (mean over planes of each plane's mean) of an image
    rendered in bands, each rank holding its own rows of img_chw [C, H, W]:
    one halo exchange, the band's per-plane sums, one all-reduce (SUM) of C
    values.  Returns the same scalar on every rank."""
    import torch.distributed as dist

    from . import metric as _metric

    c, h, w = img_chw.shape
    if plane_means is None:
        c1, c2 = (k1 * data_range) ** 2, (k2 * data_range) ** 2

        def plane_means(x, y):
            return _metric.ssim_per_plane(x.unsqueeze(0), y.unsqueeze(0), win_size, win_sigma,
                                          c1, c2)
    ext = exchange_ssim_halo(img_chw, bands_px, rank, win_size, group)
    sums = band_ssim_sums(ext, target_chw, bands_px[rank][0], win_size, plane_means)
    dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
    count = float((h - win_size + 1) * (w - win_size + 1))
    return (sums / count).mean()


__all__ = ["balanced_bands", "tile_row_work", "band_for_rank", "allreduce_hook", "allgather_halo",
           "ssim_halo_rows", "exchange_ssim_halo", "band_ssim_sums", "band_ssim"]
