"""Re-export of the GPU QuaternionLayerNorm (mirrors mambaqc/layers/quaternion_norm.py:7-17)."""

from mambaqc_b200.kernels.quaternion_norm import QuaternionLayerNorm, quaternion_layer_norm_fused

__all__ = ["QuaternionLayerNorm", "quaternion_layer_norm_fused"]
