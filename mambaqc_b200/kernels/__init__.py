"""GPU kernels of the quaternion SSM hot path (drop-in for ``mambaqc.kernels``).

Same exported names as the reference package (mambaqc/kernels/__init__.py:10-33),
plus the fused ``ssm_scan_cayley``.
"""

from .quaternion_ops import (
    quaternion_multiply,
    quaternion_multiply_batched,
    quaternion_conjugate,
    quaternion_inverse,
    quaternion_norm,
)
from .cayley_transform import cayley_discretization_fused
from .parallel_scan import parallel_scan_quaternion
from .quaternion_norm import quaternion_layer_norm_fused
from .ssm_fused import ssm_step_fused, ssm_forward_fused, ssm_scan_cayley

__all__ = [
    "quaternion_multiply",
    "quaternion_multiply_batched",
    "quaternion_conjugate",
    "quaternion_inverse",
    "quaternion_norm",
    "cayley_discretization_fused",
    "parallel_scan_quaternion",
    "quaternion_layer_norm_fused",
    "ssm_step_fused",
    "ssm_forward_fused",
    "ssm_scan_cayley",
]
