"""Model-level seam: the DeepMD facade and its fused-operator bindings."""

from .dpa4 import DPA4Model

__all__ = ["DPA4Model"]
