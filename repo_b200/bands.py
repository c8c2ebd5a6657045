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


__all__ = ["balanced_bands", "tile_row_work", "band_for_rank", "allreduce_hook"]
