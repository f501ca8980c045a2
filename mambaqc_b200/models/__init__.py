"""Models: drop-ins for the block and the LM wrapper of ``mambaqc.models``."""

from .quaternion_mamba2_block import QuaternionMamba2Block
from .quaternion_mamba2 import (
    QuaternionMamba2,
    quaternion_mamba2_base,
    quaternion_mamba2_large,
    quaternion_mamba2_small,
)

__all__ = [
    "QuaternionMamba2Block",
    "QuaternionMamba2",
    "quaternion_mamba2_small",
    "quaternion_mamba2_base",
    "quaternion_mamba2_large",
]
