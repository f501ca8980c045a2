"""Depthwise causal conv used by the block shell (mirrors mambaqc/layers/causal_conv1d.py:17-91).

``CausalConv1d(d_model, kernel_size, bias)`` holds an ``nn.Conv1d`` named ``conv``
(so reference state_dict keys ``conv.weight``/``conv.bias`` match), initialised
with Xavier-uniform weights and zero bias, applied after left padding by
kernel_size - 1. It is a cuDNN op outside the quaternion hot path.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["CausalConv1d"]


class CausalConv1d(nn.Module):
    def __init__(self, d_model: int, kernel_size: int = 4, bias: bool = True):
        super().__init__()
        self.d_model = d_model
        self.kernel_size = kernel_size
        self.padding = kernel_size - 1
        self.conv = nn.Conv1d(d_model, d_model, kernel_size, padding=0, groups=d_model, bias=bias)
        nn.init.xavier_uniform_(self.conv.weight)
        if self.conv.bias is not None:
            nn.init.zeros_(self.conv.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x.transpose(1, 2)
        if self.padding > 0:
            x = F.pad(x, (self.padding, 0))
        return self.conv(x).transpose(1, 2)

    def extra_repr(self) -> str:
        return f"d_model={self.d_model}, kernel_size={self.kernel_size}"
