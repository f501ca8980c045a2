"""mambaqc_b200: B200-native (sm_100a) quaternion SSM hot path of polux06/mambaqc.

Drop-in for the reference's Python API on that path:

* ``mambaqc_b200.kernels.quaternion_ops`` -- quaternion_multiply & co.
* ``mambaqc_b200.kernels.cayley_transform.cayley_discretization_fused``
* ``mambaqc_b200.kernels.parallel_scan.parallel_scan_quaternion``
* ``mambaqc_b200.kernels.ssm_fused`` -- ssm_step_fused, ssm_forward_fused and
  the fused ``ssm_scan_cayley``
* ``mambaqc_b200.layers.QuaternionLayerNorm``
* ``mambaqc_b200.models.QuaternionMamba2Block``

All compute runs in hand-written CUDA kernels in ``libmambaqc_b200.so`` (C ABI,
``include/mambaqc_b200.h``); there is no CPU path. ``install_as_mambaqc()``
registers these modules under the reference's import names.
"""

from __future__ import annotations

import importlib
import sys

__version__ = "0.1.0"

_ALIASES = {
    "mambaqc": "mambaqc_b200",
    "mambaqc.kernels": "mambaqc_b200.kernels",
    "mambaqc.kernels.quaternion_ops": "mambaqc_b200.kernels.quaternion_ops",
    "mambaqc.kernels.cayley_transform": "mambaqc_b200.kernels.cayley_transform",
    "mambaqc.kernels.parallel_scan": "mambaqc_b200.kernels.parallel_scan",
    "mambaqc.kernels.ssm_fused": "mambaqc_b200.kernels.ssm_fused",
    "mambaqc.kernels.quaternion_norm": "mambaqc_b200.kernels.quaternion_norm",
    "mambaqc.layers": "mambaqc_b200.layers",
    "mambaqc.layers.quaternion_norm": "mambaqc_b200.layers.quaternion_norm",
    "mambaqc.layers.quaternion_linear": "mambaqc_b200.layers.quaternion_linear",
    "mambaqc.layers.causal_conv1d": "mambaqc_b200.layers.causal_conv1d",
    "mambaqc.models": "mambaqc_b200.models",
    "mambaqc.models.quaternion_mamba2_block": "mambaqc_b200.models.quaternion_mamba2_block",
    "mambaqc.models.quaternion_mamba2": "mambaqc_b200.models.quaternion_mamba2",
}


def install_as_mambaqc() -> None:
    """Make ``import mambaqc.<module>`` resolve to this package's GPU modules.

    Only the modules listed above are aliased (the hot path, the block and the
    LM wrapper that the training harness uses); the rest of the reference
    package (Lite variant, trainer, utils) is not part of this library.
    """
    for alias, target in _ALIASES.items():
        sys.modules[alias] = importlib.import_module(target)


def __getattr__(name):
    if name == "QuaternionMamba2Block":
        from .models import QuaternionMamba2Block
        return QuaternionMamba2Block
    raise AttributeError(name)
