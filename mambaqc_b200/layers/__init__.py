"""Layers of the block (drop-in for ``mambaqc.layers``, mambaqc/layers/__init__.py:5-13)."""

from .quaternion_linear import QuaternionLinear
from .quaternion_norm import QuaternionLayerNorm
from .causal_conv1d import CausalConv1d

__all__ = ["QuaternionLinear", "QuaternionLayerNorm", "CausalConv1d"]
