"""CPU restatement of the reference quaternion SSM hot path (TEST INFRASTRUCTURE).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and
reference legs may use this module. It is the checker and the timed CPU
baseline; the product path (``mambaqc_b200``) never imports it.

Every function restates a function of polux06/mambaqc in plain PyTorch
elementwise code, running on whatever device/dtype its inputs have (the tests use
CPU float64 for ground truth and CPU float32 for the reference's own precision).
Citations are ``path:line`` inside the reference project.

Two places deliberately differ from the shipped reference code because the
shipped code cannot run there:

* ``ssm_step``: the reference multiplies ``B`` [B,D,N,4] by ``S.unsqueeze(2)``
  [B,D,1,4] through a shape-asserting product
  (``mambaqc/kernels/ssm_fused.py:418`` -> ``quaternion_ops.py:270``), which
  raises. Its own comment says "Broadcast S across d_state"; we do exactly that.
* ``block_forward``: ``mambaqc/models/quaternion_mamba2_block.py:160-161``
  multiplies ``sigmoid(z)`` (d_inner wide) with ``y_real`` (d_model wide), which
  raises for ``expand_factor != 1``. We gate with ``z[..., :d_model]``, the way
  the reference's Lite block does (``quaternion_mamba2_lite_block.py:163``).

Parity of this module against the reference itself is pinned by
``tests/golden/*.pt`` (made by ``tests/golden/make_golden.py`` from the
reference package) and checked in ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

__all__ = [
    "qmul", "qconj", "qinv", "qnorm", "cayley", "prefix_product",
    "ssm_step", "ssm_forward", "ssm_scan_cayley", "layer_norm",
    "layer_norm_padded_compat", "block_forward", "lambda_from_params",
    "block_ssm_channels",
]


# ---------------------------------------------------------------------------
# Quaternion algebra: mambaqc/kernels/quaternion_ops.py
# ---------------------------------------------------------------------------

def qmul(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """Hamilton product p (x) q on the last axis (size 4, order r,i,j,k).

    Follows the CPU branch of ``quaternion_multiply``
    (``mambaqc/kernels/quaternion_ops.py:273-282``): split into components,
    form each output component as a sum of four products, stack. Unlike the
    reference wrapper this oracle allows broadcasting between p and q.
    """
    a0, a1, a2, a3 = p.unbind(-1)
    b0, b1, b2, b3 = q.unbind(-1)
    real = a0 * b0 - a1 * b1 - a2 * b2 - a3 * b3
    ci = a0 * b1 + a1 * b0 + a2 * b3 - a3 * b2
    cj = a0 * b2 - a1 * b3 + a2 * b0 + a3 * b1
    ck = a0 * b3 + a1 * b2 - a2 * b1 + a3 * b0
    return torch.stack((real, ci, cj, ck), dim=-1)


def qconj(q: torch.Tensor) -> torch.Tensor:
    """(a, -b, -c, -d); ``quaternion_conjugate`` CPU branch, quaternion_ops.py:372-374."""
    sign = torch.tensor([1.0, -1.0, -1.0, -1.0], dtype=q.dtype, device=q.device)
    return q * sign


def qinv(q: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """conj(q) / max(|q|^2, eps); ``quaternion_inverse`` CPU branch, quaternion_ops.py:407-410."""
    n2 = (q * q).sum(dim=-1, keepdim=True).clamp_min(eps)
    return qconj(q) / n2


def qnorm(q: torch.Tensor) -> torch.Tensor:
    """Euclidean norm of each quaternion; ``quaternion_norm`` CPU branch, quaternion_ops.py:443-444."""
    return torch.linalg.vector_norm(q, dim=-1)


# ---------------------------------------------------------------------------
# Cayley discretisation: mambaqc/kernels/cayley_transform.py:199-223
# ---------------------------------------------------------------------------

def cayley(z: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """q = (1 - z/2)^-1 (x) (1 + z/2), inverse via ``qinv`` with the eps clamp.

    Same sequence of operations as ``cayley_discretization_reference``
    (cayley_transform.py:207-221): numerator and denominator around the identity,
    quaternion inverse of the denominator, then a left product.
    """
    one = torch.zeros(4, dtype=z.dtype, device=z.device)
    one[0] = 1.0
    num = one + 0.5 * z
    den = one - 0.5 * z
    return qmul(qinv(den, eps=eps), num)


# ---------------------------------------------------------------------------
# Prefix product: mambaqc/kernels/parallel_scan.py:267-295
# ---------------------------------------------------------------------------

def prefix_product(q_seq: torch.Tensor) -> torch.Tensor:
    """cum[:, t] = q[:, t] (x) cum[:, t-1], cum[:, -1] = 1, for q_seq [B,T,D,N,4].

    Restates ``parallel_scan_quaternion_reference`` (parallel_scan.py:279-295):
    an accumulator starting at the identity, left-multiplied by each step.
    """
    bsz, seqlen, dm, ds, _ = q_seq.shape
    acc = torch.zeros(bsz, dm, ds, 4, dtype=q_seq.dtype, device=q_seq.device)
    acc[..., 0] = 1.0
    out = []
    for t in range(seqlen):
        acc = qmul(q_seq[:, t], acc)
        out.append(acc)
    return torch.stack(out, dim=1)


# ---------------------------------------------------------------------------
# SSM recurrence: mambaqc/kernels/ssm_fused.py
# ---------------------------------------------------------------------------

def _expand_bc(m: torch.Tensor, d_model: int) -> torch.Tensor:
    """Shared per-step [B,N,4] B/C broadcast over channels -> [B,D,N,4]."""
    if m.dim() == 3:
        return m.unsqueeze(1).expand(m.shape[0], d_model, m.shape[1], 4)
    return m


def _as_quaternion_signal(s: torch.Tensor) -> torch.Tensor:
    """Real signal [...,] -> (s, 0, 0, 0), as the block embeds it (block.py:200-202)."""
    out = torch.zeros(*s.shape, 4, dtype=s.dtype, device=s.device)
    out[..., 0] = s
    return out


def ssm_step(q, B, S, C, D, h_prev):
    """One step: h' = q (x) h + B (x) S;  y = sum_n C (x) h' + D * S.

    Restates ``ssm_step_reference`` (ssm_fused.py:405-430) with S broadcast over
    d_state (the reference's intent at :418). Shapes: q, h_prev [B,D,N,4];
    B, C [B,D,N,4] or shared [B,N,4]; S [B,D,4]; D [B,D] or [D].
    """
    dm = q.shape[1]
    Bx = _expand_bc(B, dm)
    Cx = _expand_bc(C, dm)
    h_new = qmul(q, h_prev) + qmul(Bx, S.unsqueeze(2).expand_as(Bx))
    y = qmul(Cx, h_new).sum(dim=2) + D.unsqueeze(-1) * S
    return h_new, y


def ssm_forward(q, B, S, C, D, h0=None):
    """Sequential scan over time; returns (y [B,T,D,4], h_T [B,D,N,4]).

    Restates the CPU branch of ``ssm_forward_fused`` (ssm_fused.py:363-379):
    state starts at zero (or ``h0``), one ``ssm_step`` per timestep.
    ``D`` may be [B,T,D] (the reference's expanded skip) or [D].
    """
    bsz, seqlen, dm, ds, _ = q.shape
    if h0 is None:
        h = torch.zeros(bsz, dm, ds, 4, dtype=q.dtype, device=q.device)
    else:
        h = h0
    ys = []
    for t in range(seqlen):
        d_t = D[:, t] if D.dim() == 3 else D
        h, y_t = ssm_step(q[:, t], B[:, t], S[:, t], C[:, t], d_t, h)
        ys.append(y_t)
    return torch.stack(ys, dim=1), h


def ssm_scan_cayley(delta, Lam, B, C, S, D, h0=None, eps=1e-6, t_slab=64):
    """Fused-op semantics: z = delta * Lambda, q = cayley(z), then the scan.

    Composes ``QuaternionMamba2Block._ssm_forward``
    (models/quaternion_mamba2_block.py:214-228): ``z = Delta[...,None,None] *
    Lambda`` (:217-221), ``cayley_discretization_fused(z, eps=1e-6)`` (:225),
    ``ssm_forward_fused`` (:228). Time is processed in slabs of ``t_slab`` steps
    so that z and q never exceed B*t_slab*D*N quaternions.

    delta [B,T,D]; Lam [D,N,4]; B, C shared [B,T,N,4] or per-channel
    [B,T,D,N,4]; S real [B,T,D] or quaternion [B,T,D,4]; D [D] or [B,T,D].
    Returns (y [B,T,D,4], h_T [B,D,N,4]).
    """
    bsz, seqlen, dm = delta.shape
    ds = Lam.shape[1]
    if S.dim() == 3:
        S = _as_quaternion_signal(S)
    h = h0 if h0 is not None else torch.zeros(bsz, dm, ds, 4, dtype=delta.dtype,
                                              device=delta.device)
    ys = []
    for t0 in range(0, seqlen, t_slab):
        t1 = min(seqlen, t0 + t_slab)
        z = delta[:, t0:t1, :, None, None] * Lam[None, None]
        q = cayley(z, eps=eps)
        for t in range(t1 - t0):
            d_t = D[:, t0 + t] if D.dim() == 3 else D
            h, y_t = ssm_step(q[:, t], B[:, t0 + t], S[:, t0 + t], C[:, t0 + t], d_t, h)
            ys.append(y_t)
    return torch.stack(ys, dim=1), h


# ---------------------------------------------------------------------------
# Quaternion LayerNorm: mambaqc/kernels/quaternion_norm.py
# ---------------------------------------------------------------------------

def layer_norm(q, gamma, beta, eps=1e-5):
    """Norm-only LayerNorm over d_model, preserving each quaternion's direction.

    Restates ``quaternion_layer_norm_reference`` (quaternion_norm.py:219-245):
    n = sqrt(|q|^2 + eps); mean and biased variance of n over the row;
    out = gamma * (n - mean)/sqrt(var + eps) * q/(n + eps) + beta.
    """
    n = torch.sqrt((q * q).sum(dim=-1) + eps)
    mu = n.mean(dim=-1, keepdim=True)
    var = ((n - mu) ** 2).mean(dim=-1, keepdim=True)
    nhat = (n - mu) / torch.sqrt(var + eps)
    direction = q / (n.unsqueeze(-1) + eps)
    return gamma.view(1, 1, -1, 1) * nhat.unsqueeze(-1) * direction + beta.view(1, 1, -1, 4)


def layer_norm_padded_compat(q, gamma, beta, eps=1e-5):
    """Bug-compatible form of the reference *Triton* LayerNorm kernel.

    ``quaternion_layer_norm_kernel`` (quaternion_norm.py:65-89, launched with
    BLOCK_D = next_power_of_2(d_model) at :158) loads 0 into the padded lanes,
    which then contribute sqrt(eps) to the norm sum and (sqrt(eps) - mean)^2 to
    the variance sum, while both sums are divided by d_model. For a power-of-two
    d_model this equals ``layer_norm``.
    """
    dm = q.shape[-2]
    block = 1 << (dm - 1).bit_length()
    pad = block - dm
    n = torch.sqrt((q * q).sum(dim=-1) + eps)
    pad_norm = torch.sqrt(torch.tensor(eps, dtype=q.dtype))
    mu = (n.sum(dim=-1, keepdim=True) + pad * pad_norm) / dm
    var = (((n - mu) ** 2).sum(dim=-1, keepdim=True) + pad * (pad_norm - mu) ** 2) / dm
    nhat = (n - mu) / torch.sqrt(var + eps)
    direction = q / (n.unsqueeze(-1) + eps)
    return gamma.view(1, 1, -1, 1) * nhat.unsqueeze(-1) * direction + beta.view(1, 1, -1, 4)


# ---------------------------------------------------------------------------
# Block composition: mambaqc/models/quaternion_mamba2_block.py:124-230
# ---------------------------------------------------------------------------

def lambda_from_params(alpha, imag):
    """Lambda = (-softplus(alpha), tanh(imag)) [D,N,4] (block.py:206-212)."""
    lam = torch.zeros(*alpha.shape, 4, dtype=alpha.dtype, device=alpha.device)
    lam[..., 0] = -F.softplus(alpha)
    lam[..., 1:] = torch.tanh(imag)
    return lam


def block_forward(params: dict, x: torch.Tensor, d_state: int, d_conv: int = 4,
                  Lam: torch.Tensor | None = None, eps_ln: float = 1e-5,
                  return_state: bool = False):
    """QuaternionMamba2Block.forward (block.py:124-166) with the gate fix.

    ``params`` holds the block's state_dict tensors under the reference names
    (``in_proj.weight``, ``conv1d.conv.weight``, ``Lambda_alpha``, ...).
    ``Lam`` overrides the Lambda computed from ``Lambda_alpha``/``Lambda_imag``.
    """
    bsz, seqlen, d_model = x.shape
    p = params
    xz = F.linear(x, p["in_proj.weight"], p.get("in_proj.bias"))
    x_in, z = xz.chunk(2, dim=-1)
    d_inner = x_in.shape[-1]
    # CausalConv1d (layers/causal_conv1d.py:68-91): left pad by k-1, depthwise.
    xc = F.pad(x_in.transpose(1, 2), (d_conv - 1, 0))
    xc = F.conv1d(xc, p["conv1d.conv.weight"], p.get("conv1d.conv.bias"), groups=d_inner)
    xa = F.silu(xc.transpose(1, 2))
    # _ssm_forward (block.py:168-230)
    delta = F.softplus(F.linear(xa, p["dt_proj.weight"], p["dt_proj.bias"]))
    Bq = F.linear(xa, p["B_proj.weight"]).view(bsz, seqlen, d_inner, d_state, 4)
    Cq = F.linear(xa, p["C_proj.weight"]).view(bsz, seqlen, d_inner, d_state, 4)
    gate = torch.sigmoid(F.linear(xa, p["gate_proj.weight"]))
    s_real = gate * xa
    if Lam is None:
        Lam = lambda_from_params(p["Lambda_alpha"], p["Lambda_imag"])
    y_q, h_T = ssm_scan_cayley(delta, Lam, Bq, Cq, s_real, p["D"])
    y_n = layer_norm(y_q, p["norm.gamma"], p["norm.beta"], eps_ln)
    y_r = F.linear(y_n.reshape(bsz, seqlen, d_inner * 4), p["out_proj.weight"],
                   p.get("out_proj.bias"))
    out = x + torch.sigmoid(z[..., :d_model]) * y_r
    if return_state:
        return out, h_T
    return out


def block_ssm_channels(params: dict, x: torch.Tensor, d_state: int, chans: torch.Tensor,
                       d_conv: int = 4):
    """The block's SSM (block.py:130-144 then :168-230) on a subset of channels.

    Runs in_proj, the causal conv + SiLU and dt_proj / gate_proj over all
    channels (they are cheap and the SSM inputs of a channel need the whole conv
    output row), but projects B and C only for the channels in ``chans``
    (rows ``c*d_state*4 .. (c+1)*d_state*4`` of B_proj / C_proj), and scans those.
    Channels are independent recurrences, so the result equals the same channels
    of the full block's SSM. Returns (y_q [B,T,k,4], h_T [B,k,N,4]).
    """
    bsz, seqlen, _ = x.shape
    p = params
    xz = F.linear(x, p["in_proj.weight"], p.get("in_proj.bias"))
    x_in, _ = xz.chunk(2, dim=-1)
    d_inner = x_in.shape[-1]
    xc = F.pad(x_in.transpose(1, 2), (d_conv - 1, 0))
    xc = F.conv1d(xc, p["conv1d.conv.weight"], p.get("conv1d.conv.bias"), groups=d_inner)
    xa = F.silu(xc.transpose(1, 2))
    delta = F.softplus(F.linear(xa, p["dt_proj.weight"], p["dt_proj.bias"]))
    s_real = torch.sigmoid(F.linear(xa, p["gate_proj.weight"])) * xa
    rows = (chans[:, None] * (d_state * 4) + torch.arange(d_state * 4)).reshape(-1)
    k = chans.numel()
    Bq = F.linear(xa, p["B_proj.weight"][rows]).view(bsz, seqlen, k, d_state, 4)
    Cq = F.linear(xa, p["C_proj.weight"][rows]).view(bsz, seqlen, k, d_state, 4)
    Lam = lambda_from_params(p["Lambda_alpha"][chans], p["Lambda_imag"][chans])
    return ssm_scan_cayley(delta[..., chans], Lam, Bq, Cq, s_real[..., chans], p["D"][chans])
