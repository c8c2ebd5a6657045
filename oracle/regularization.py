"""CPU oracle for the reference's regularisation loss -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of ``regularization_loss_tilelang`` (manbo/regularization.py:
65-250) and its per-term kernels (manbo/ops/regularization.py):

  L = L_shape + L_opacity + [closed] (L_curvature + L_boundary)

* L_shape = lambda_proj / N * sum phi(alpha), phi(a) = relu(a - 1)^2 +
  relu(-a)^2, alpha = ((m - p0) . v) / (|v|^2 + 1e-8), v = pend - p0, over the
  middle control points m of each curve (:32-54, :119-206); open curves
  project onto the chord p0 -> p[K-1] (:209-295), closed ones onto
  p0 -> p[split] and skip the split point (split = shape degree + 1,
  manbo/regularization.py:52-62).
* L_opacity = opacity_weight * mean |sigmoid(op) - 1| (:298-354).
* L_boundary = mean over the joints p[0], p[d], p[2d], ... and both
  coordinates of relu(x - bound) + relu(-bound - x) (:357-420, :592-628).
* L_curvature = sum over samples f = 0, s, 2s, ... of the closed sample path
  [xyz[:, 0], reversed xyz[:, 1]] (length L) of |prev - 2 curr + next|^2,
  prev/next 5 samples back/ahead (cyclic), kept where the cosine of the angle
  at curr exceeds cos(thresh), divided by N * ceil(L / s) (:423-515, :646-699).

Gradients follow the reference's backward kernels (:702-1081): the same
scales, every term's exact derivative (the curvature mask is held fixed).
Only ``tests/`` may use this module.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

CURVATURE_ROLL_OFFSET = 5
EPS = 1e-8


def shape_degree(mode: str, num_beziers: int, bezier_degree: int) -> int:
    """manbo/regularization.py:52-62."""
    if mode == "unclosed" or int(num_beziers) <= 2:
        return int(bezier_degree)
    return int(bezier_degree) * int(num_beziers // 2) + 1


def _shape_terms(cp: np.ndarray, split_idx: Optional[int]):
    n, k, _ = cp.shape
    if split_idx is None:
        pend, mids = k - 1, np.arange(1, k - 1)
    else:
        pend = int(split_idx)
        mids = np.array([i for i in range(1, k) if i != pend], dtype=np.int64)
    p0 = cp[:, 0, :]
    v = cp[:, pend, :] - p0                                   # [N, 2]
    u = cp[:, mids, :] - p0[:, None, :]                       # [N, M, 2]
    denom = v[:, 0] * v[:, 0] + v[:, 1] * v[:, 1] + cp.dtype.type(EPS)
    alpha = (u[..., 0] * v[:, None, 0] + u[..., 1] * v[:, None, 1]) / denom[:, None]
    return pend, mids, v, u, denom, alpha


def shape_sum(cp: np.ndarray, split_idx: Optional[int] = None) -> float:
    """Sum of phi(alpha) over curves and middle points (open when split_idx
    is None)."""
    cp = np.asarray(cp)
    if cp.shape[0] == 0 or cp.shape[1] <= 2:
        return 0.0
    _, _, _, _, _, alpha = _shape_terms(cp, split_idx)
    pos = np.maximum(alpha - 1, 0)
    neg = np.maximum(-alpha, 0)
    return float((pos * pos + neg * neg).sum(dtype=np.float64))


def shape_grad(cp: np.ndarray, split_idx: Optional[int], scale: float) -> np.ndarray:
    cp = np.asarray(cp)
    g = np.zeros_like(cp)
    if cp.shape[0] == 0 or cp.shape[1] <= 2:
        return g
    pend, mids, v, u, denom, alpha = _shape_terms(cp, split_idx)
    inv = 1 / denom[:, None]
    d_alpha = np.where(alpha > 1, 2 * (alpha - 1), np.where(alpha < 0, 2 * alpha, 0))
    ds = d_alpha * cp.dtype.type(scale)
    g_mid = ds[..., None] * v[:, None, :] * inv[..., None]                     # [N, M, 2]
    g_end = ds[..., None] * (u * inv[..., None] - 2 * alpha[..., None] * v[:, None, :]
                             * inv[..., None])
    np.add.at(g, (slice(None), mids), g_mid)
    g[:, pend, :] += g_end.sum(axis=1)
    g[:, 0, :] -= (g_mid + g_end).sum(axis=1)
    return g


def _sigmoid(x):
    return 1 / (1 + np.exp(-x))


def opacity_sum(op: np.ndarray) -> float:
    op = np.asarray(op).reshape(-1)
    return float(np.abs(_sigmoid(op) - 1).sum(dtype=np.float64))


def opacity_grad(op: np.ndarray, scale: float) -> np.ndarray:
    op = np.asarray(op)
    sig = _sigmoid(op)
    return (op.dtype.type(scale) * np.sign(sig - 1) * sig * (1 - sig)).astype(op.dtype)


def boundary_sum(cp: np.ndarray, degree: int, bound: float) -> float:
    joints = np.asarray(cp)[:, ::int(degree), :]
    b = joints.dtype.type(bound)
    return float((np.maximum(joints - b, 0) + np.maximum(-b - joints, 0)).sum(dtype=np.float64))


def boundary_grad(cp: np.ndarray, degree: int, bound: float, scale: float) -> np.ndarray:
    cp = np.asarray(cp)
    g = np.zeros_like(cp)
    j = cp[:, ::int(degree), :]
    s = cp.dtype.type(scale)
    g[:, ::int(degree), :] = np.where(j > bound, s, np.where(j < -bound, -s, 0))
    return g


def _curvature_samples(xyz: np.ndarray, stride: int):
    n, _, m, _ = xyz.shape
    full = np.concatenate([xyz[:, 0], xyz[:, 1, ::-1]], axis=1)          # [N, L, 2]
    length = 2 * m
    f = np.arange(0, length, int(stride))
    fp = (f - CURVATURE_ROLL_OFFSET) % length
    fn = (f + CURVATURE_ROLL_OFFSET) % length
    return full, f, fp, fn, length


def _curvature_mask(prev, curr, nxt, angle_thresh_deg):
    v1, v2 = prev - curr, nxt - curr
    e = prev.dtype.type(EPS)
    n1 = np.sqrt(v1[..., 0] ** 2 + v1[..., 1] ** 2 + e)
    n2 = np.sqrt(v2[..., 0] ** 2 + v2[..., 1] ** 2 + e)
    dot = (v1[..., 0] / n1) * (v2[..., 0] / n2) + (v1[..., 1] / n1) * (v2[..., 1] / n2)
    dot = np.minimum(1, np.maximum(-1, dot))
    return dot > math.cos(math.radians(float(angle_thresh_deg)))


def curvature_sum(xyz: np.ndarray, stride: int, angle_thresh_deg: float = 60.0
                  ) -> Tuple[float, int]:
    """(sum of the masked second-difference energy, samples per curve)."""
    xyz = np.asarray(xyz)
    full, f, fp, fn, _ = _curvature_samples(xyz, stride)
    if f.size == 0:
        return 0.0, 0
    prev, curr, nxt = full[:, fp], full[:, f], full[:, fn]
    sec = prev - 2 * curr + nxt
    energy = sec[..., 0] ** 2 + sec[..., 1] ** 2
    mask = _curvature_mask(prev, curr, nxt, angle_thresh_deg)
    return float(np.where(mask, energy, 0).sum(dtype=np.float64)), int(f.size)


def curvature_grad(xyz: np.ndarray, stride: int, angle_thresh_deg: float, scale: float
                   ) -> np.ndarray:
    xyz = np.asarray(xyz)
    g_full = np.zeros((xyz.shape[0], 2 * xyz.shape[2], 2), xyz.dtype)
    full, f, fp, fn, length = _curvature_samples(xyz, stride)
    if f.size:
        prev, curr, nxt = full[:, fp], full[:, f], full[:, fn]
        sec = prev - 2 * curr + nxt
        mask = _curvature_mask(prev, curr, nxt, angle_thresh_deg)
        d = xyz.dtype.type(scale) * mask[..., None] * sec
        for idx, w in ((fp, 1), (f, -2), (fn, 1)):
            np.add.at(g_full, (slice(None), idx), w * d)
    m = xyz.shape[2]
    g = np.zeros_like(xyz)
    g[:, 0] = g_full[:, :m]
    g[:, 1] = g_full[:, m:][:, ::-1]
    return g


def regularization_loss(cp, op, xyz=None, *, mode: str, num_beziers: int, bezier_degree: int,
                        num_samples: int, lambda_proj: float = 1e-2,
                        opacity_weight: float = 1e-2, boundary_degree: Optional[int] = None,
                        boundary_bound: float = 1.0,
                        curvature_angle_thresh_deg: float = 60.0) -> float:
    """manbo/regularization.py:65-164 (float64 accumulation)."""
    mode = str(mode).lower()
    cp = np.asarray(cp)
    n = cp.shape[0]
    bdeg = int(bezier_degree) + 1 if boundary_degree is None else int(boundary_degree)
    if mode == "unclosed":
        loss = float(lambda_proj) * shape_sum(cp) / max(1, n)
    else:
        sd = shape_degree(mode, num_beziers, bezier_degree)
        if cp.shape[1] != 2 * sd + 2:
            raise ValueError(f"expected K={2 * sd + 2}, got {cp.shape[1]}")
        loss = float(lambda_proj) * shape_sum(cp, sd + 1) / n
    opf = np.asarray(op).reshape(-1)
    loss += float(opacity_weight) * opacity_sum(opf) / max(1, opf.size)
    if mode == "closed":
        csum, per = curvature_sum(xyz, num_samples, curvature_angle_thresh_deg)
        loss += csum / max(1, n * per)
        joints = (cp.shape[1] + bdeg - 1) // bdeg
        loss += boundary_sum(cp, bdeg, boundary_bound) / max(1, n * joints * 2)
    return loss


def regularization_grads(cp, op, xyz=None, *, mode: str, num_beziers: int, bezier_degree: int,
                         num_samples: int, lambda_proj: float = 1e-2,
                         opacity_weight: float = 1e-2, boundary_degree: Optional[int] = None,
                         boundary_bound: float = 1.0, curvature_angle_thresh_deg: float = 60.0):
    """(d L / d cp, d L / d op, d L / d xyz or None): manbo/regularization.py:
    167-249 with the scales of manbo/ops/regularization.py:1084-1237."""
    mode = str(mode).lower()
    cp = np.asarray(cp)
    n = cp.shape[0]
    bdeg = int(bezier_degree) + 1 if boundary_degree is None else int(boundary_degree)
    scale = float(lambda_proj) / max(1, n)
    if mode == "unclosed":
        g_cp = shape_grad(cp, None, scale)
    else:
        sd = shape_degree(mode, num_beziers, bezier_degree)
        g_cp = shape_grad(cp, sd + 1, scale)
        joints = (cp.shape[1] + bdeg - 1) // bdeg
        g_cp = g_cp + boundary_grad(cp, bdeg, boundary_bound, 1.0 / max(1, n * joints * 2))
    op = np.asarray(op)
    g_op = opacity_grad(op, float(opacity_weight) / max(1, op.size))
    g_xyz = None
    if mode == "closed":
        xyz = np.asarray(xyz)
        per = -(-2 * xyz.shape[2] // int(num_samples))
        g_xyz = curvature_grad(xyz, num_samples, curvature_angle_thresh_deg,
                               2.0 / max(1, n * per))
    return g_cp, g_op, g_xyz


__all__ = ["regularization_loss", "regularization_grads", "shape_sum", "shape_grad",
           "opacity_sum", "opacity_grad", "boundary_sum", "boundary_grad", "curvature_sum",
           "curvature_grad", "shape_degree"]
