"""Regularisation loss of the curve model (manbo/regularization.py:359-430),
one launch for the loss and one for all of its gradients on the B200 kernels
(repo_b200.regularization)."""
from typing import Optional

import torch

from repo_b200.regularization import regularization_loss as _regularization_loss

DEFAULT_REG_THREADS = 256
DEFAULT_REG_ITEMS_PER_THREAD = 8


def regularization_loss_tilelang(control_points: torch.Tensor, opacity: torch.Tensor,
                                 xyz: Optional[torch.Tensor] = None, *, mode: str,
                                 num_beziers: int, bezier_degree: int, num_samples: int,
                                 lambda_proj: float = 1e-2, opacity_weight: float = 1e-2,
                                 boundary_degree: Optional[int] = None,
                                 boundary_bound: float = 1.0,
                                 curvature_angle_thresh_deg: float = 60.0,
                                 threads: int = DEFAULT_REG_THREADS,
                                 items_per_thread: int = DEFAULT_REG_ITEMS_PER_THREAD,
                                 use_autograd: bool = True) -> torch.Tensor:
    """L = L_shape + L_opacity + [closed] (L_curvature + L_boundary), a 0-dim
    float32 tensor; ``threads`` and ``items_per_thread`` (TileLang launch
    shape in the reference) are accepted and unused."""
    return _regularization_loss(
        control_points, opacity, xyz, mode=mode, num_beziers=num_beziers,
        bezier_degree=bezier_degree, num_samples=num_samples, lambda_proj=lambda_proj,
        opacity_weight=opacity_weight, boundary_degree=boundary_degree,
        boundary_bound=boundary_bound, curvature_angle_thresh_deg=curvature_angle_thresh_deg,
        use_autograd=use_autograd)


__all__ = ["regularization_loss_tilelang"]
