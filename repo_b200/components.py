"""4-connected component labelling over the C ABI (``cs_ccl_*``), with the
arguments, checks and return layout of the reference's
``connected_components_labels_4_tilelang``,
``connected_components_with_stats_4_tilelang`` and
``select_largest_component_center`` (manbo/ops/connected_components.py:98-283).
"""
from __future__ import annotations

from typing import Tuple

import torch

from . import _native as nat

DEFAULT_THREADS = 256
DEFAULT_MAX_ITERS = 4096


def _check(mask: torch.Tensor, max_iters: int) -> torch.Tensor:
    if mask.ndim != 2:
        raise ValueError(f"mask must be [H, W], got {tuple(mask.shape)}")
    if max_iters <= 0:
        raise ValueError("max_iters must be > 0")
    nat.require_cuda(mask, "mask")
    return mask.to(dtype=torch.uint8).contiguous()


def _workspace(dev: torch.device, n: int) -> torch.Tensor:
    return torch.empty((int(nat.call("cs_ccl_workspace_size", n)),), dtype=torch.uint8,
                       device=dev)


def _status_check(status: torch.Tensor, name: str) -> None:
    if int(status.item()) != 0:
        raise RuntimeError(f"{name}: device status {int(status.item())}")


def connected_components_labels_4(mask: torch.Tensor, *, max_iters: int = DEFAULT_MAX_ITERS,
                                  threads: int = DEFAULT_THREADS,
                                  workspace: torch.Tensor = None) -> torch.Tensor:
    """[H, W] int32: each component labelled with its smallest linear index
    + 1, background 0.  The union-find always converges, so max_iters is only
    validated."""
    m = _check(mask, max_iters)
    h, w = (int(v) for v in m.shape)
    dev = m.device
    labels = torch.zeros((h, w), dtype=torch.int32, device=dev)
    if h * w == 0:
        return labels
    ws = workspace if workspace is not None else _workspace(dev, h * w)
    status = torch.zeros((1,), dtype=torch.int32, device=dev)
    nat.check(nat.call("cs_ccl_labels_4", m.data_ptr(), h, w, labels.data_ptr(),
                       status.data_ptr(), ws.data_ptr(), nat.stream(dev)), "cs_ccl_labels_4")
    _status_check(status, "cs_ccl_labels_4")
    return labels


def connected_components_with_stats_4(mask: torch.Tensor, *, max_iters: int = DEFAULT_MAX_ITERS,
                                      threads: int = DEFAULT_THREADS
                                      ) -> Tuple[int, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(num_labels including the background, labels [H, W] int32 numbered 1..
    in raster order of each component's first pixel, stats [n, 5] int32
    (x, y, width, height, area), centres [n, 2] float32)."""
    m = _check(mask, max_iters)
    h, w = (int(v) for v in m.shape)
    dev = m.device
    empty = (1, torch.zeros((h, w), dtype=torch.int32, device=dev),
             torch.empty((0, 5), dtype=torch.int32, device=dev),
             torch.empty((0, 2), dtype=torch.float32, device=dev))
    if h * w == 0:
        return empty
    ws = _workspace(dev, h * w)
    raw = connected_components_labels_4(m, max_iters=max_iters, workspace=ws)
    compact = torch.empty_like(raw)
    count = torch.zeros((1,), dtype=torch.int32, device=dev)
    status = torch.zeros((1,), dtype=torch.int32, device=dev)
    st = nat.stream(dev)
    nat.check(nat.call("cs_ccl_compact_4", raw.data_ptr(), h, w, compact.data_ptr(),
                       count.data_ptr(), status.data_ptr(), ws.data_ptr(), st), "cs_ccl_compact_4")
    n = int(count.item())
    _status_check(status, "cs_ccl_compact_4")
    if n == 0:
        return empty
    stats = torch.empty((n, 5), dtype=torch.int32, device=dev)
    centres = torch.empty((n, 2), dtype=torch.float32, device=dev)
    nat.check(nat.call("cs_ccl_stats_4", h, w, n, stats.data_ptr(), centres.data_ptr(),
                       ws.data_ptr(), st), "cs_ccl_stats_4")
    return n + 1, compact, stats, centres


def select_largest_component_center(labels: torch.Tensor, stats: torch.Tensor,
                                    centers: torch.Tensor):
    """(row, col, label, area, mask) of the pixel of the largest component
    closest to its centre, first in raster order on ties
    (manbo/ops/connected_components.py:239-272)."""
    if labels.ndim != 2:
        raise ValueError(f"labels must be [H, W], got {tuple(labels.shape)}")
    if stats.ndim != 2 or stats.shape[-1] != 5:
        raise ValueError(f"stats must be [N, 5], got {tuple(stats.shape)}")
    if centers.ndim != 2 or centers.shape[-1] != 2:
        raise ValueError(f"centers must be [N, 2], got {tuple(centers.shape)}")
    if stats.shape[0] <= 0:
        raise ValueError("stats must contain at least one foreground component")
    k = int(torch.argmax(stats[:, 4]).item())
    label, area = k + 1, int(stats[k, 4].item())
    comp = labels == label
    rc = torch.nonzero(comp, as_tuple=False)  # raster order
    if rc.numel() <= 0:
        raise RuntimeError("selected connected component has zero pixels")
    centre = torch.stack([centers[k, 1], centers[k, 0]]).to(torch.float32)
    d = torch.norm(rc.to(torch.float32) - centre.unsqueeze(0), dim=1)
    best = int(torch.argmin(d).item())
    return int(rc[best, 0].item()), int(rc[best, 1].item()), label, area, comp


__all__ = ["connected_components_labels_4", "connected_components_with_stats_4",
           "select_largest_component_center", "DEFAULT_THREADS", "DEFAULT_MAX_ITERS"]
