"""Models (drop-in for the block of ``mambaqc.models``)."""

from .quaternion_mamba2_block import QuaternionMamba2Block

__all__ = ["QuaternionMamba2Block"]
