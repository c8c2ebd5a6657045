"""Drop-in ``manbo`` package backed by the B200 (sm_100a) CubicSplat kernels.

Same module paths and names as the reference's ``manbo`` (manbo/__init__.py:1-29)
for the render/optimise hot path: the cubic fill and stroke renderers, their
per-stage operators, the ring-segment conversion, the MSE / PSNR / SSIM
metrics and the Adan optimiser that train.py uses by default.  Subsystems
outside that path (Gaussian renderer, regularisation, connected components)
keep their names so that imports succeed, and raise NotImplementedError when
called.
"""
from . import ops
from .metric import mse_loss_tilelang, psnr, ssim
from .optim import Adan
from .regularization import regularization_loss_tilelang
from .tilelang_renderer import GsRenderFunction, GsRenderModule, gs_render, set_gs_profile_ctx_factory

__all__ = [
    "ops",
    "mse_loss_tilelang",
    "regularization_loss_tilelang",
    "psnr",
    "ssim",
    "Adan",
    "GsRenderFunction",
    "GsRenderModule",
    "set_gs_profile_ctx_factory",
    "gs_render",
]
