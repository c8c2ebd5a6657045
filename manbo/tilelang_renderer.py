"""Gaussian splat renderer names (manbo/tilelang_renderer.py); outside the B200 hot path."""
from ._unavailable import unavailable, unavailable_class

_PROFILE_CTX_FACTORY = None


def set_gs_profile_ctx_factory(factory):
    """Accepted for compatibility; the B200 kernels do not use it."""
    global _PROFILE_CTX_FACTORY
    _PROFILE_CTX_FACTORY = factory


gs_render = unavailable("gs_render")
GsRenderFunction = unavailable_class("GsRenderFunction")
GsRenderModule = unavailable_class("GsRenderModule")

__all__ = ["GsRenderFunction", "GsRenderModule", "gs_render", "set_gs_profile_ctx_factory"]
