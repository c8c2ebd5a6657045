"""Per-tile intersect ranges (manbo/ops/tile_bins.py), backed by the B200 kernel."""
from __future__ import annotations

import torch

from repo_b200 import _native as nat

BLOCK_X = 16
BLOCK_Y = 16
DEFAULT_THREADS = 256


def get_tile_bin_edges_kernel(threads: int = DEFAULT_THREADS):
    def kernel(isect_ids_sorted, tile_bins):
        nat.check(nat.call("cs_tile_bin_edges", nat.ptr(isect_ids_sorted),
                           int(isect_ids_sorted.numel()), nat.ptr(tile_bins),
                           int(tile_bins.shape[0]), nat.stream(tile_bins.device)),
                  "cs_tile_bin_edges")
    return kernel


def get_tile_bin_edges_tilelang(num_intersects: int, isect_ids_sorted: torch.Tensor, *,
                                num_tiles: int, compact: bool = False,
                                threads: int = DEFAULT_THREADS):
    rows = num_tiles if compact else max(int(num_tiles), int(num_intersects))
    tile_bins = torch.zeros((rows, 2), dtype=torch.int32, device=isect_ids_sorted.device)
    get_tile_bin_edges_kernel(threads)(isect_ids_sorted.contiguous(), tile_bins)
    return tile_bins
