"""Adan optimiser name (manbo/optim.py:10); not part of the B200 hot path."""
from ._unavailable import unavailable_class

Adan = unavailable_class("Adan")

__all__ = ["Adan"]
