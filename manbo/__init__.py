"""Drop-in ``manbo`` package backed by the B200 (sm_100a) CubicSplat kernels.

Same module paths and names as the reference's ``manbo`` (manbo/__init__.py:1-29)
for the render/optimise hot path: the cubic fill and stroke renderers, their
per-stage operators, the ring-segment conversion, the MSE / PSNR / SSIM
metrics, the Adan optimiser that train.py uses by default, the regularisation
loss and the connected-component labelling.  The Gaussian renderer, outside
that path, keeps its names so that imports succeed, and raises
NotImplementedError when called.
"""
import importlib.util as _ilu
import pkgutil as _pkgutil
import sys as _sys

# Subpackages this package does not provide (the reference's model glue
# `gaussian_trace`, its `profile` tooling, `sparse_init`) are found in any
# other `manbo` directory on sys.path, such as an installed copy of the
# reference: its Python glue then runs on these kernels, because it imports
# the renderer, metrics and optimiser from `manbo`, which is this package.
__path__ = _pkgutil.extend_path(__path__, __name__)
def _importable(name: str) -> bool:
    if name in _sys.modules:
        return True
    try:
        return _ilu.find_spec(name) is not None
    except (ImportError, ValueError):
        return False


if not _importable("visual_debug"):
    from . import _visual_debug
    _sys.modules["visual_debug"] = _visual_debug

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
