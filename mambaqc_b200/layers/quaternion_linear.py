"""Real <-> quaternion projections used by the block shell (plain dense GEMMs).

Mirrors the parameterisation of ``QuaternionLinear`` and the two convenience
constructors of the reference (mambaqc/layers/quaternion_linear.py:16-266): a
single ``weight`` [out_features, in_features] (and optional ``bias``), normal
initialisation with the reference's variance scaling, applied with
``F.linear`` (cuBLAS). Same parameter names, shapes and RNG consumption, so a
reference checkpoint or a seeded initialisation carries over unchanged. These
GEMMs are outside the quaternion hot path.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["QuaternionLinear", "real_to_quaternion_projection", "quaternion_to_real_projection"]


class QuaternionLinear(nn.Module):
    """Linear map between real and quaternion feature spaces (quaternion_linear.py:16-208)."""

    def __init__(self, in_features: int, out_features: int, input_type: str = "real",
                 output_type: str = "quaternion", bias: bool = True):
        super().__init__()
        assert input_type in ("real", "quaternion")
        assert output_type in ("real", "quaternion")
        if input_type == "quaternion":
            assert in_features % 4 == 0, f"in_features must be divisible by 4, got {in_features}"
        if output_type == "quaternion":
            assert out_features % 4 == 0, f"out_features must be divisible by 4, got {out_features}"
        self.in_features = in_features
        self.out_features = out_features
        self.input_type = input_type
        self.output_type = output_type
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        if input_type == "real" and output_type == "quaternion":
            std = math.sqrt(2.0 / (in_features + out_features // 4))
            nn.init.normal_(self.weight, mean=0.0, std=std)
        elif input_type == "quaternion" and output_type == "real":
            std = math.sqrt(2.0 / (in_features // 4 + out_features))
            nn.init.normal_(self.weight, mean=0.0, std=std)
        elif input_type == "quaternion" and output_type == "quaternion":
            std = math.sqrt(2.0 / (in_features // 4 + out_features // 4))
            nn.init.normal_(self.weight, mean=0.0, std=std)
        else:
            nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if bias:
            if output_type == "quaternion":
                self.bias = nn.Parameter(torch.zeros(out_features // 4, 4))
            else:
                self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.input_type == "quaternion":
            x = x.reshape(*x.shape[:-2], x.shape[-2] * 4)
        if self.output_type == "quaternion":
            out = F.linear(x, self.weight)
            out = out.view(*out.shape[:-1], self.out_features // 4, 4)
            return out if self.bias is None else out + self.bias
        return F.linear(x, self.weight, self.bias)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"input_type={self.input_type}, output_type={self.output_type}, "
                f"bias={self.bias is not None}")


def real_to_quaternion_projection(in_features: int, out_quat_dim: int,
                                  bias: bool = True) -> QuaternionLinear:
    """R^in -> H^out_quat_dim (quaternion_linear.py:227-245)."""
    return QuaternionLinear(in_features, out_quat_dim * 4, "real", "quaternion", bias)


def quaternion_to_real_projection(in_quat_dim: int, out_features: int,
                                  bias: bool = True) -> QuaternionLinear:
    """H^in_quat_dim -> R^out (quaternion_linear.py:248-266)."""
    return QuaternionLinear(in_quat_dim * 4, out_features, "quaternion", "real", bias)
