"""``manbo.ops`` with the reference's exported names (manbo/ops/__init__.py:45-176).

Hot-path operators (cubic fill / stroke renderer stages, tile bins, ring
segments, metric kernels) run on the B200 sm_100a kernels, and so do the Adan
step (train.py's default optimiser) and the 4-connected component labelling.
The Gaussian renderer's operators are outside the B200 hot path, and the
reference's per-term regularisation kernels have no counterpart (one launch
computes every term of ``manbo.regularization_loss_tilelang``): their names
exist so imports succeed, and calling them raises NotImplementedError.
"""
from .._unavailable import unavailable
from .connected_components import (
    connected_components_labels_4_tilelang,
    connected_components_with_stats_4_tilelang,
    select_largest_component_center,
)
from .cubic_polyline_splatting import render_cubic_polyline_splat_tilelang
from .cubic_splatting import (
    closed_cubic_fill_segments_backward_kernel,
    closed_cubic_fill_segments_forward_kernel,
    closed_cubic_fill_segments_tilelang,
    map_cubic_to_intersects_kernel,
    map_cubic_to_intersects_tilelang,
    project_cubics_2d_forward_kernel,
    project_cubics_2d_forward_tilelang,
    rasterize_cubic_fill_backward_kernel,
    rasterize_cubic_fill_backward_tilelang,
    rasterize_cubic_fill_forward_kernel,
    rasterize_cubic_fill_forward_tilelang,
    render_cubic_fill_splat_tilelang,
)
from .metric import (
    mse_backward_diff_kernel,
    mse_backward_diff_tilelang,
    mse_partial_sum_kernel,
    reduce_sum_1d_tilelang,
    reduce_sum_partial_kernel,
    ssim_map_kernel,
)
from .optim import adan_step_from_grad_tilelang
from .tile_bins import get_tile_bin_edges_tilelang

_OUT_OF_SCOPE = [
    "project_gaussians_2d_scale_rot_forward_tilelang",
    "project_gaussians_2d_scale_rot_backward_tilelang",
    "map_gaussian_to_intersects_tilelang",
    "map_gaussian_meta_to_intersects",
    "rasterize_forward_tilelang",
    "rasterize_backward_tilelang",
    "bezier_shape_backward_kernel",
    "bezier_open_backward_kernel",
    "opacity_backward_kernel",
    "boundary_backward_kernel",
    "curvature_backward_kernel",
    "bezier_shape_partial_sum_kernel",
    "bezier_open_partial_sum_kernel",
    "opacity_partial_sum_kernel",
    "boundary_partial_sum_kernel",
    "curvature_partial_sum_kernel",
    "bezier_shape_proj_outside_grad_tilelang",
    "bezier_shape_proj_outside_sum_tilelang",
    "bezier_open_proj_outside_grad_tilelang",
    "bezier_open_proj_outside_sum_tilelang",
    "opacity_abs_sigmoid_delta_grad_tilelang",
    "opacity_abs_sigmoid_delta_sum_tilelang",
    "boundary_joints_penalty_grad_tilelang",
    "boundary_joints_penalty_sum_tilelang",
    "curvature_masked_second_diff_grad_tilelang",
    "curvature_masked_second_diff_sum_tilelang",
]
for _name in _OUT_OF_SCOPE:
    globals()[_name] = unavailable(_name)
DEFAULT_REG_THREADS = 256
DEFAULT_REG_ITEMS_PER_THREAD = 8

__all__ = [
    "project_cubics_2d_forward_kernel",
    "project_cubics_2d_forward_tilelang",
    "closed_cubic_fill_segments_forward_kernel",
    "closed_cubic_fill_segments_backward_kernel",
    "closed_cubic_fill_segments_tilelang",
    "map_cubic_to_intersects_kernel",
    "map_cubic_to_intersects_tilelang",
    "rasterize_cubic_fill_backward_kernel",
    "rasterize_cubic_fill_backward_tilelang",
    "rasterize_cubic_fill_forward_kernel",
    "rasterize_cubic_fill_forward_tilelang",
    "render_cubic_fill_splat_tilelang",
    "render_cubic_polyline_splat_tilelang",
    "get_tile_bin_edges_tilelang",
    "mse_backward_diff_kernel",
    "mse_backward_diff_tilelang",
    "mse_partial_sum_kernel",
    "reduce_sum_partial_kernel",
    "ssim_map_kernel",
    "reduce_sum_1d_tilelang",
    "adan_step_from_grad_tilelang",
    "connected_components_labels_4_tilelang",
    "connected_components_with_stats_4_tilelang",
    "select_largest_component_center",
    "DEFAULT_REG_THREADS",
    "DEFAULT_REG_ITEMS_PER_THREAD",
] + _OUT_OF_SCOPE
