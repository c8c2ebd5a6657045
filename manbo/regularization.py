"""Regularisation losses (manbo/regularization.py); outside the B200 hot path."""
from ._unavailable import unavailable

regularization_loss_tilelang = unavailable("regularization_loss_tilelang")

__all__ = ["regularization_loss_tilelang"]
