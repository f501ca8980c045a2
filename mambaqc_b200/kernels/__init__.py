"""GPU kernels of the quaternion SSM hot path (drop-in for ``mambaqc.kernels``).

Same exported names as the reference package (mambaqc/kernels/__init__.py:10-33),
plus the fused ``ssm_scan_cayley`` and the block's fused glue ops
(``causal_conv1d_silu``, ``ssm_scan_inputs``, ``gate_residual``).
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
from .ssm_fused import (ssm_step_fused, ssm_forward_fused, ssm_scan_cayley,
                        ssm_scan_cayley_from_host, ssm_step_cayley, ssm_scan_summary,
                        ssm_scan_carry, ssm_scan_cayley_resume)
from .block_fused import causal_conv1d_silu, gate_residual, ssm_scan_inputs

# Importing the submodule ``quaternion_norm`` (the LayerNorm file) rebinds the
# package attribute of that name to the module; bind the function again so that
# ``kernels.quaternion_norm`` is the quaternion norm, as its export list says.
from .quaternion_ops import quaternion_norm  # noqa: E402,F811

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
    "ssm_scan_cayley_from_host",
    "ssm_step_cayley",
    "ssm_scan_summary",
    "ssm_scan_carry",
    "ssm_scan_cayley_resume",
    "causal_conv1d_silu",
    "ssm_scan_inputs",
    "gate_residual",
]
