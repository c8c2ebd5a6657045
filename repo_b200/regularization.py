"""Regularisation loss of the curve model over the C ABI
(``cs_regularization_forward`` / ``cs_regularization_backward``), with the
argument checks and defaults of the reference's ``regularization_loss_tilelang``
(manbo/regularization.py:359-430): one launch for the loss, one for all
gradients.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _native as nat


def shape_bezier_degree(mode: str, num_beziers: int, bezier_degree: int) -> int:
    """Degree of the chord the closed shape term projects onto
    (manbo/regularization.py:52-62)."""
    if mode == "unclosed" or int(num_beziers) <= 2:
        return int(bezier_degree)
    return int(bezier_degree) * int(num_beziers // 2) + 1


_WS = {}


def _workspace(dev: torch.device) -> torch.Tensor:
    key = str(dev)
    ws = _WS.get(key)
    if ws is None:
        ws = torch.zeros((int(nat.call("cs_regularization_workspace_size")),), dtype=torch.uint8,
                         device=dev)
        _WS[key] = ws
    return ws


def _f32(x: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(x, torch.Tensor) or x.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    return x.detach().to(torch.float32).contiguous()


def _args(cp, op, xyz, mode, num_beziers, bezier_degree, num_samples, lambda_proj,
          opacity_weight, boundary_degree, boundary_bound, angle_deg):
    n, k = int(cp.shape[0]), int(cp.shape[1])
    closed = mode == "closed"
    split = 0
    m = 0
    if closed:
        sd = shape_bezier_degree(mode, num_beziers, bezier_degree)
        if k != 2 * sd + 2:
            raise ValueError(f"control_points shape mismatch for closed regularizer: "
                             f"expected K={2 * sd + 2}, got {k}")
        split = sd + 1
        if xyz.dim() != 4 or xyz.shape[0] != n or xyz.shape[1] != 2 or xyz.shape[-1] != 2:
            raise ValueError(f"paths must have shape [N, 2, M, 2], got {tuple(xyz.shape)}")
        if int(num_samples) <= 0:
            raise ValueError("stride must be > 0")
        if int(boundary_degree) <= 0:
            raise ValueError("degree must be > 0")
        m = int(xyz.shape[2])
    cos_t = float(math.cos(math.radians(float(angle_deg))))
    return (n, k, int(op.numel()), m, int(closed), int(split), int(boundary_degree),
            float(boundary_bound), int(num_samples), cos_t, float(lambda_proj),
            float(opacity_weight))


class _RegularizationFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, control_points, opacity, xyz, args):
        cp = _f32(control_points, "control_points")
        op = _f32(opacity, "opacity").view(-1)
        xz = _f32(xyz, "xyz") if xyz is not None else None
        loss = torch.empty((), dtype=torch.float32, device=cp.device)
        nat.check(nat.call("cs_regularization_forward", cp.data_ptr(), op.data_ptr(),
                           xz.data_ptr() if xz is not None else None, *args, loss.data_ptr(),
                           _workspace(cp.device).data_ptr(), nat.stream(cp.device)),
                  "cs_regularization_forward")
        ctx.save_for_backward(cp, op, xz if xz is not None else cp.new_empty((0,)))
        ctx.args = args
        ctx.has_xyz = xz is not None
        ctx.op_shape = opacity.shape
        return loss

    @staticmethod
    def backward(ctx, grad_output):
        cp, op, xz = ctx.saved_tensors
        need_cp, need_op, need_xyz = ctx.needs_input_grad[:3]
        g_cp = torch.empty_like(cp) if need_cp else None
        g_op = torch.empty_like(op) if need_op else None
        g_xyz = torch.empty_like(xz) if (need_xyz and ctx.has_xyz) else None
        go = grad_output.detach().to(torch.float32).contiguous()
        nat.check(nat.call("cs_regularization_backward", cp.data_ptr(), op.data_ptr(),
                           xz.data_ptr() if ctx.has_xyz else None, *ctx.args, go.data_ptr(),
                           g_cp.data_ptr() if g_cp is not None else None,
                           g_op.data_ptr() if g_op is not None else None,
                           g_xyz.data_ptr() if g_xyz is not None else None,
                           nat.stream(cp.device)), "cs_regularization_backward")
        return (g_cp, g_op.view(ctx.op_shape) if g_op is not None else None, g_xyz, None)


def regularization_loss(control_points: torch.Tensor, opacity: torch.Tensor,
                        xyz: Optional[torch.Tensor] = None, *, mode: str, num_beziers: int,
                        bezier_degree: int, num_samples: int, lambda_proj: float = 1e-2,
                        opacity_weight: float = 1e-2, boundary_degree: Optional[int] = None,
                        boundary_bound: float = 1.0, curvature_angle_thresh_deg: float = 60.0,
                        use_autograd: bool = True) -> torch.Tensor:
    """L = L_shape + L_opacity + [closed] (L_curvature + L_boundary), a 0-dim
    float32 tensor (manbo/regularization.py:359-430)."""
    mode = str(mode).lower()
    if mode not in {"closed", "unclosed"}:
        raise ValueError(f"Unsupported mode={mode!r}; expected 'closed' or 'unclosed'")
    if mode == "closed" and xyz is None:
        raise ValueError("xyz must be provided when mode='closed'")
    if control_points.dim() != 3 or control_points.shape[-1] != 2:
        raise ValueError(f"control_points must have shape [N, K, 2], "
                         f"got {tuple(control_points.shape)}")
    if int(control_points.shape[0]) <= 0:
        raise ValueError("control_points must include at least one curve")
    bdeg = int(bezier_degree) + 1 if boundary_degree is None else int(boundary_degree)
    args = _args(control_points, opacity, xyz, mode, num_beziers, bezier_degree, num_samples,
                 lambda_proj, opacity_weight, bdeg, boundary_bound, curvature_angle_thresh_deg)
    x = xyz if mode == "closed" else None
    if not use_autograd:
        with torch.no_grad():
            return _RegularizationFn.apply(control_points, opacity, x, args)
    return _RegularizationFn.apply(control_points, opacity, x, args)


__all__ = ["regularization_loss", "shape_bezier_degree"]
