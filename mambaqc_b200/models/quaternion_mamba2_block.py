"""QuaternionMamba2Block with the GPU fused scan: drop-in for
``mambaqc.models.quaternion_mamba2_block.QuaternionMamba2Block``.

Constructor signature, submodule names, parameter names/shapes and the order
of random initialisation follow the reference (models/quaternion_mamba2_block.py:55-122),
so a reference state_dict loads unchanged and ``torch.manual_seed(s)`` gives the
same initial weights. The forward follows :124-230 with two differences:

* ``_ssm_forward`` calls ``ssm_scan_cayley`` (one fused kernel) instead of
  materialising z = Delta*Lambda and q = Cayley(z) and looping over time
  (:214-228);
* the output gate uses ``sigmoid(z[..., :d_model])``: the reference multiplies
  a d_inner-wide gate with the d_model-wide projection (:160-161), which fails
  for expand_factor != 1; its Lite block slices the same way
  (quaternion_mamba2_lite_block.py:163).

The in/dt/gate/B/C projections stay dense PyTorch linears (cuBLAS). Everything
between them runs in ``libmambaqc_b200.so``:
* the causal conv + SiLU, read in place from the in_proj output;
* the step sizes and gated signal (softplus, sigmoid gate);
* the scan, the quaternion LayerNorm, and the output gate + residual.
Each has a forward and a backward kernel. Two tcgen05 fusions replace pairs of
ops under bf16 autocast, both opt-in because at the config-4 block shape they
still measure slower than the unfused kernels: ``fused_norm_out_proj`` (the
LayerNorm as the operand prologue of the output projection's GEMM) and
``fused_bc_proj`` (the B/C projections computed inside the scan kernel).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from mambaqc_b200.kernels.bc_proj_scan import bc_proj_scan, bc_proj_scan_supported
from mambaqc_b200.kernels.block_fused import causal_conv1d_silu, gate_residual, ssm_scan_inputs
from mambaqc_b200.kernels.quaternion_norm import quaternion_layer_norm_linear
from mambaqc_b200.kernels.ssm_fused import ssm_scan_cayley, ssm_step_cayley
from mambaqc_b200.layers.causal_conv1d import CausalConv1d
from mambaqc_b200.layers.quaternion_linear import (
    quaternion_to_real_projection,
    real_to_quaternion_projection,
)
from mambaqc_b200.layers.quaternion_norm import QuaternionLayerNorm

__all__ = ["QuaternionMamba2Block"]


class QuaternionMamba2Block(nn.Module):
    """Single Quaternion Mamba-2 block: [batch, seq_len, d_model] -> same shape."""

    def __init__(self, d_model: int, d_state: int = 64, d_conv: int = 4,
                 expand_factor: int = 2, dt_rank: str | int = "auto", bias: bool = False):
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.d_conv = d_conv
        self.d_inner = d_model * expand_factor
        self.dt_rank = max(16, d_model // 16) if dt_rank == "auto" else dt_rank
        self.in_proj = nn.Linear(d_model, self.d_inner * 2, bias=bias)
        self.conv1d = CausalConv1d(self.d_inner, kernel_size=d_conv, bias=True)
        self.Lambda_alpha = nn.Parameter(torch.randn(self.d_inner, d_state) * 0.5 + 1.0)
        self.Lambda_imag = nn.Parameter(torch.randn(self.d_inner, d_state, 3) * 0.1)
        self.dt_proj = nn.Linear(self.d_inner, self.d_inner, bias=True)
        self.B_proj = real_to_quaternion_projection(self.d_inner, self.d_inner * d_state, bias=False)
        self.C_proj = real_to_quaternion_projection(self.d_inner, self.d_inner * d_state, bias=False)
        self.D = nn.Parameter(torch.ones(self.d_inner))
        self.gate_proj = nn.Linear(self.d_inner, self.d_inner, bias=False)
        self.norm = QuaternionLayerNorm(self.d_inner, eps=1e-5)
        self.out_proj = quaternion_to_real_projection(self.d_inner, d_model, bias=bias)
        # Optional fixed Lambda [d_inner, d_state, 4] used instead of the
        # (-softplus(alpha), tanh(imag)) parameterisation (not part of state_dict).
        self.lambda_override: torch.Tensor | None = None
        # Under bf16 autocast, compute B_proj/C_proj inside the scan kernel
        # (``bc_proj_scan``) instead of storing them; ``forward(..., fused_bc_proj=)``
        # overrides it per call. Off by default: at the config-4 block shape the
        # fused forward measures slower than cuBLAS projections + the scan.
        self.fused_bc_proj = False
        # Under bf16 autocast, apply the LayerNorm inside the output projection's
        # GEMM (``quaternion_layer_norm_linear``): True, False, or "auto" (fused
        # when no gradient is needed). Off by default: at the config-4 block
        # shape the fused forward measures 0.14-0.18 ms against 0.11-0.14 ms
        # for the LayerNorm kernel + cuBLAS on the same box.
        self.fused_norm_out_proj: bool | str = False

    def ssm_lambda(self) -> torch.Tensor:
        """Lambda [d_inner, d_state, 4] = (-softplus(alpha), tanh(imag)) (block.py:206-212)."""
        if self.lambda_override is not None:
            return self.lambda_override
        real = -F.softplus(self.Lambda_alpha.float())
        imag = torch.tanh(self.Lambda_imag.float())
        return torch.cat([real.unsqueeze(-1), imag], dim=-1)

    def forward(self, x: torch.Tensor, return_ssm_state: bool = False,
                fused_bc_proj: bool | None = None):
        xz = self.in_proj(x)
        x_inner, z = xz.chunk(2, dim=-1)
        conv = self.conv1d.conv
        x_act = causal_conv1d_silu(x_inner, conv.weight, conv.bias)
        y_quat, h_T = self._ssm_forward(x_act, return_state=True, fused_bc_proj=fused_bc_proj)
        y_real = self._norm_out_proj(y_quat)
        out = gate_residual(x, z[..., : self.d_model], y_real)
        return (out, h_T) if return_ssm_state else out

    def _norm_out_proj(self, y_quat: torch.Tensor) -> torch.Tensor:
        """``out_proj(norm(y_quat))`` (block lines 154-157). With
        ``fused_norm_out_proj`` (True, or "auto" when no gradient is needed),
        under bf16 autocast -- where the projection
        would run in bf16 on the LayerNorm's bf16 output -- the LayerNorm is
        applied inside the projection GEMM (``quaternion_layer_norm_linear``), so
        the normalised activations are never written to memory; otherwise the
        two modules run in turn."""
        w = self.out_proj.weight
        want = self.fused_norm_out_proj
        if want == "auto":
            want = not (torch.is_grad_enabled() and
                        (y_quat.requires_grad or w.requires_grad))
        fusable = (bool(want) and y_quat.is_cuda and
                   y_quat.dtype == torch.bfloat16 and
                   torch.is_autocast_enabled("cuda") and
                   torch.get_autocast_dtype("cuda") == torch.bfloat16 and
                   self.d_inner % 16 == 0 and y_quat.dim() == 4)
        if not fusable:
            return self.out_proj(self.norm(y_quat))
        bias = self.out_proj.bias
        with torch.autocast("cuda", enabled=False):
            return quaternion_layer_norm_linear(
                y_quat, self.norm.gamma, self.norm.beta, w.to(torch.bfloat16),
                None if bias is None else bias.to(torch.bfloat16), self.norm.eps)

    def _bc_fusable(self, x: torch.Tensor, fused_bc_proj: bool | None) -> bool:
        want = self.fused_bc_proj if fused_bc_proj is None else fused_bc_proj
        return (bool(want) and x.is_cuda and torch.is_autocast_enabled("cuda") and
                torch.get_autocast_dtype("cuda") == torch.bfloat16 and x.dim() == 3 and
                self.B_proj.bias is None and self.C_proj.bias is None and
                bc_proj_scan_supported(self.d_inner, self.d_state))

    def _ssm_forward(self, x: torch.Tensor, return_state: bool = False,
                     fused_bc_proj: bool | None = None):
        bsz, seqlen, d_inner = x.shape
        delta, s_real = ssm_scan_inputs(self.dt_proj(x), self.gate_proj(x), x)
        if self._bc_fusable(x, fused_bc_proj):
            # B_proj / C_proj (block lines 186-191) as the scan kernel's own
            # tensor-core prologue: the projections are never stored
            bf = torch.bfloat16
            with torch.autocast("cuda", enabled=False):
                y, h_T = bc_proj_scan(x.to(bf), self.B_proj.weight.to(bf),
                                      self.C_proj.weight.to(bf), delta.to(bf), self.ssm_lambda(),
                                      s_real.to(bf), self.D, return_final_state=True)
            return (y, h_T) if return_state else y
        Bq = self.B_proj(x).view(bsz, seqlen, d_inner, self.d_state, 4)
        Cq = self.C_proj(x).view(bsz, seqlen, d_inner, self.d_state, 4)
        dt = Bq.dtype
        y, h_T = ssm_scan_cayley(delta.to(dt), self.ssm_lambda(), Bq, Cq.to(dt), s_real.to(dt),
                                 self.D, return_final_state=True)
        return (y, h_T) if return_state else y

    @torch.no_grad()
    def prefill(self, x: torch.Tensor):
        """Forward over a prompt x [B, T, d_model] that also returns the cache a
        recurrent continuation needs: {"conv": the last d_conv-1 conv inputs
        [B, d_conv-1, d_inner] (zeros before the start), "h": the SSM state
        [B, d_inner, d_state, 4] fp32}."""
        out, h_T = self.forward(x, return_ssm_state=True)
        k1 = self.d_conv - 1
        x_inner = self.in_proj(x)[..., : self.d_inner]
        hist = x_inner.new_zeros(x.shape[0], k1, self.d_inner)
        take = min(k1, x.shape[1])
        if take > 0:
            hist[:, k1 - take:] = x_inner[:, -take:]
        return out, {"conv": hist, "h": h_T.contiguous()}

    @torch.no_grad()
    def step(self, x_t: torch.Tensor, cache: dict) -> torch.Tensor:
        """One token through the block, x_t [B, d_model] -> [B, d_model], from
        and into ``cache`` (see ``prefill``): the conv runs over the cached
        inputs plus this one, and the SSM advances its state in place
        (``ssm_step_cayley``). Same result as running the whole sequence
        through ``forward`` and taking the last position."""
        bsz = x_t.shape[0]
        xz = self.in_proj(x_t)
        x_in, z = xz.chunk(2, dim=-1)
        window = torch.cat([cache["conv"].to(x_in.dtype), x_in[:, None]], dim=1)
        conv = self.conv1d.conv
        x_act = causal_conv1d_silu(window, conv.weight, conv.bias)[:, -1].contiguous()
        cache["conv"] = window[:, 1:].contiguous()
        delta, s_real = ssm_scan_inputs(self.dt_proj(x_act), self.gate_proj(x_act), x_act)
        Bq = self.B_proj(x_act).view(bsz, self.d_inner, self.d_state, 4)
        Cq = self.C_proj(x_act).view(bsz, self.d_inner, self.d_state, 4)
        dt = Bq.dtype
        y = ssm_step_cayley(delta.to(dt).contiguous(), self.ssm_lambda(), Bq.contiguous(),
                            Cq.to(dt).contiguous(), s_real.to(dt).contiguous(), self.D,
                            cache["h"])
        y_real = self.out_proj(self.norm(y[:, None]))[:, 0]
        return gate_residual(x_t, z[..., : self.d_model], y_real)

    def extra_repr(self) -> str:
        return (f"d_model={self.d_model}, d_state={self.d_state}, d_inner={self.d_inner}, "
                f"d_conv={self.d_conv}, dt_rank={self.dt_rank}")
