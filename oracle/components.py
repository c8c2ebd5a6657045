"""CPU oracle for the reference's 4-connected component labelling -- TEST
INFRASTRUCTURE ONLY.

``connected_components_labels_4_tilelang`` (manbo/ops/connected_components.py:
98-131) starts every foreground pixel at its linear index + 1 and relaxes each
label to the minimum over its 4-neighbours until nothing changes, so a
component ends labelled with its smallest linear index + 1 (background 0).
``connected_components_with_stats_4_tilelang`` (:134-236) renumbers the
components 1.. in the order of those labels (raster order of their first
pixel) and returns OpenCV-style stats [x, y, width, height, area] and float32
centres [mean x, mean y].  Here scipy's raster-order labelling gives the
components; ``relax_labels_4`` restates the reference's iteration itself for
small masks.  Only ``tests/`` may use this module.
"""
from __future__ import annotations

import numpy as np


def _components(mask: np.ndarray):
    from scipy import ndimage
    m = np.asarray(mask) != 0
    lab, n = ndimage.label(m, structure=[[0, 1, 0], [1, 1, 1], [0, 1, 0]])
    return m, lab.astype(np.int64), int(n)


def labels_4(mask: np.ndarray) -> np.ndarray:
    """Raw labels: smallest linear index + 1 of each component, 0 outside."""
    m, lab, n = _components(mask)
    out = np.zeros(lab.shape, np.int32)
    if n == 0:
        return out
    flat = lab.reshape(-1)
    idx = np.arange(flat.size)
    first = np.full(n + 1, flat.size, np.int64)
    np.minimum.at(first, flat[flat > 0], idx[flat > 0])
    out.reshape(-1)[flat > 0] = (first[flat[flat > 0]] + 1).astype(np.int32)
    return out


def relax_labels_4(mask: np.ndarray, max_iters: int = 4096) -> np.ndarray:
    """The reference's own iteration (cc_init_labels_kernel, cc_relax_4_kernel):
    slow, for small masks."""
    m = np.asarray(mask) != 0
    h, w = m.shape
    lab = np.where(m, np.arange(h * w).reshape(h, w) + 1, 0).astype(np.int64)
    for _ in range(max_iters):
        best = lab.copy()
        for dy, dx in ((-1, 0), (1, 0), (0, -1), (0, 1)):
            nb = np.zeros_like(lab)
            ys = slice(max(0, dy), h + min(0, dy))
            yd = slice(max(0, -dy), h + min(0, -dy))
            xs = slice(max(0, dx), w + min(0, dx))
            xd = slice(max(0, -dx), w + min(0, -dx))
            nb[yd, xd] = lab[ys, xs]
            cand = np.where(nb > 0, nb, np.iinfo(np.int64).max)
            best = np.where(m, np.minimum(best, cand), 0)
        if np.array_equal(best, lab):
            return lab.astype(np.int32)
        lab = best
    raise RuntimeError(f"CCL did not converge within max_iters={max_iters}")


def with_stats_4(mask: np.ndarray):
    """(num_labels incl. background, compact labels [H, W] int32,
    stats [n, 5] int32 (x, y, width, height, area), centres [n, 2] float32)."""
    m, lab, n = _components(mask)
    h, w = lab.shape
    if n == 0:
        return 1, np.zeros((h, w), np.int32), np.zeros((0, 5), np.int32), \
            np.zeros((0, 2), np.float32)
    ys, xs = np.nonzero(lab)
    ids = lab[ys, xs]
    stats = np.zeros((n, 5), np.int32)
    centres = np.zeros((n, 2), np.float32)
    for k in range(1, n + 1):
        sel = ids == k
        x, y = xs[sel], ys[sel]
        stats[k - 1] = (x.min(), y.min(), x.max() - x.min() + 1, y.max() - y.min() + 1, sel.sum())
        # float32 sums of integer coordinates are exact below 2^24, as in the
        # reference's scatter_add; then one float32 division
        centres[k - 1, 0] = np.float32(x.sum()) / np.float32(sel.sum())
        centres[k - 1, 1] = np.float32(y.sum()) / np.float32(sel.sum())
    return n + 1, lab.astype(np.int32), stats, centres


__all__ = ["labels_4", "relax_labels_4", "with_stats_4"]
