"""Generate golden input/output fixtures from the reference implementation.

Run in a container where the reference package (polux06/mambaqc) is present:

    REFERENCE_ROOT=/path/to/mambaqc python tests/golden/make_golden.py

It imports the reference's own CPU functions, runs them on small seeded inputs
and writes ``tests/golden/reference_golden.pt`` (a dict of cases, each a dict
of input and output tensors). The GPU box has no reference checkout, so the
fixtures are committed; this script is the record of how they were made.

Where the reference cannot run as shipped, the script applies the smallest fix
and says so in the case's ``note``:

* ``ssm_step_reference`` multiplies B [B,D,N,4] by ``S.unsqueeze(2)`` through a
  shape-asserting product (``mambaqc/kernels/ssm_fused.py:418``). The script
  replaces it with the same three reference ``quaternion_multiply`` calls and
  ``S`` expanded over d_state, then lets the reference's own
  ``ssm_forward_fused`` CPU loop (``ssm_fused.py:363-379``) drive it.
* ``QuaternionMamba2Block.forward`` gates a d_model-wide output with a
  d_inner-wide ``sigmoid(z)`` (``quaternion_mamba2_block.py:160-161``). The
  script runs the block's own submodules in order and gates with
  ``z[..., :d_model]``.

The LayerNorm case additionally runs the reference Triton kernel under the
Triton CPU interpreter at a non-power-of-two d_model, which pins the padded-lane
behaviour of ``quaternion_layer_norm_kernel`` (``quaternion_norm.py:65-89``).
"""

from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_golden.pt"


def _ref_root() -> Path:
    root = os.environ.get("REFERENCE_ROOT")
    if not root:
        raise SystemExit("set REFERENCE_ROOT to the reference checkout")
    return Path(root)


def _source_hashes(root: Path) -> dict:
    files = [
        "mambaqc/kernels/quaternion_ops.py",
        "mambaqc/kernels/cayley_transform.py",
        "mambaqc/kernels/parallel_scan.py",
        "mambaqc/kernels/ssm_fused.py",
        "mambaqc/kernels/quaternion_norm.py",
        "mambaqc/models/quaternion_mamba2_block.py",
        "mambaqc/layers/quaternion_linear.py",
        "mambaqc/layers/causal_conv1d.py",
    ]
    return {f: hashlib.sha256((root / f).read_bytes()).hexdigest() for f in files}


def _triton_ln_case(root: Path) -> dict:
    """Run the reference Triton LayerNorm kernel under TRITON_INTERPRET=1 in a child."""
    code = r"""
import sys, torch
sys.dont_write_bytecode = True
from mambaqc.kernels.quaternion_norm import quaternion_layer_norm_fused
g = torch.Generator().manual_seed(7)
q = torch.randn(2, 3, 24, 4, generator=g)
gamma = 1.0 + 0.1 * torch.randn(24, generator=g)
beta = 0.1 * torch.randn(24, 4, generator=g)
out = quaternion_layer_norm_fused(q, gamma, beta, 1e-5)
torch.save({"q": q, "gamma": gamma, "beta": beta, "out": out}, sys.argv[1])
"""
    tmp = HERE / "_triton_ln_tmp.pt"
    env = dict(os.environ, TRITON_INTERPRET="1", PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=str(root))
    subprocess.run([sys.executable, "-c", code, str(tmp)], check=True, env=env)
    import torch
    case = torch.load(tmp)
    tmp.unlink()
    case["note"] = ("reference Triton quaternion_layer_norm_kernel run by the Triton "
                    "CPU interpreter, d_model=24 (BLOCK_D=32, 8 padded lanes)")
    return case


def main() -> None:
    root = _ref_root()
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(root))
    import torch
    import torch.nn.functional as F
    from mambaqc.kernels import quaternion_ops as qo
    from mambaqc.kernels import cayley_transform as ct
    from mambaqc.kernels import parallel_scan as ps
    from mambaqc.kernels import quaternion_norm as qn
    from mambaqc.kernels import ssm_fused as sf
    from mambaqc.models.quaternion_mamba2_block import QuaternionMamba2Block

    def fixed_step(q, B, S, C, D, h_prev):
        qh = qo.quaternion_multiply(q, h_prev)
        bs = qo.quaternion_multiply(B, S.unsqueeze(2).expand_as(B).contiguous())
        h_new = qh + bs
        y = qo.quaternion_multiply(C, h_new).sum(dim=2) + D.unsqueeze(-1) * S
        return h_new, y

    sf.ssm_step_reference = fixed_step  # the module-level name ssm_forward_fused calls

    cases: dict = {}
    g = torch.Generator().manual_seed(1234)

    def randn(*shape, dtype=torch.float64):
        return torch.randn(*shape, generator=g, dtype=dtype)

    # --- quaternion algebra (quaternion_ops.py:259-461, CPU branches) ---
    for dt, tag in ((torch.float64, "f64"), (torch.float32, "f32")):
        p, q = randn(257, 4, dtype=dt), randn(257, 4, dtype=dt)
        cases[f"qmul_{tag}"] = {"p": p, "q": q, "out": qo.quaternion_multiply(p, q)}
        cases[f"qconj_{tag}"] = {"q": q, "out": qo.quaternion_conjugate(q)}
        qi = q + 0.5
        cases[f"qinv_{tag}"] = {"q": qi, "out": qo.quaternion_inverse(qi, eps=1e-6)}
        cases[f"qnorm_{tag}"] = {"q": q, "out": qo.quaternion_norm(q)}
    pa = torch.tensor([[1.0, 1.0, 0.0, 0.0]])
    pb = torch.tensor([[1.0, 0.0, 1.0, 0.0]])
    cases["qmul_noncommuting_pair"] = {"p": pa, "q": pb, "pq": qo.quaternion_multiply(pa, pb),
                                       "qp": qo.quaternion_multiply(pb, pa)}
    tiny = torch.tensor([[1e-4, 0.0, 0.0, 0.0], [0.0, 0.0, 0.0, 0.0]], dtype=torch.float64)
    cases["qinv_eps_clamp"] = {"q": tiny, "out": qo.quaternion_inverse(tiny, eps=1e-6)}

    # --- Cayley (cayley_transform.py:199-223) ---
    for dt, tag in ((torch.float64, "f64"), (torch.float32, "f32")):
        z = randn(2, 4, 8, 16, 4, dtype=dt)
        cases[f"cayley_{tag}"] = {"z": z, "eps": 1e-6,
                                  "out": ct.cayley_discretization_reference(z, eps=1e-6)}
    zs = randn(2, 4, 8, 16, 4)
    zs[..., 0] = -zs[..., 0].abs()
    cases["cayley_stable_f64"] = {"z": zs, "eps": 1e-6,
                                  "out": ct.cayley_discretization_reference(zs, eps=1e-6)}
    # near the pole z = 2: |1 - z/2|^2 falls under eps and the clamp is active
    zp = torch.zeros(1, 1, 1, 4, 4, dtype=torch.float64)
    zp[..., 0] = torch.tensor([2.0, 2.0 + 1e-4, 1.999, 0.0], dtype=torch.float64).view(1, 1, 1, 4)
    cases["cayley_pole_f64"] = {"z": zp, "eps": 1e-6,
                                "out": ct.cayley_discretization_reference(zp, eps=1e-6)}

    # --- prefix product (parallel_scan.py:267-295) ---
    u = randn(2, 16, 8, 16, 4)
    r = 0.9 + 0.099 * torch.rand(2, 16, 8, 16, 1, generator=g, dtype=torch.float64)
    qseq = u / u.norm(dim=-1, keepdim=True) * r
    cases["prefix_f64"] = {"q": qseq, "out": ps.parallel_scan_quaternion_reference(qseq)}
    qseq32 = randn(1, 8, 4, 8, 4, dtype=torch.float32)
    cases["prefix_f32"] = {"q": qseq32, "out": ps.parallel_scan_quaternion_reference(qseq32)}

    # --- LayerNorm reference (quaternion_norm.py:219-245) ---
    for dm in (16, 24):
        qq = randn(2, 5, dm, 4)
        gamma = 1.0 + 0.1 * randn(dm)
        beta = 0.1 * randn(dm, 4)
        cases[f"layernorm_d{dm}_f64"] = {
            "q": qq, "gamma": gamma, "beta": beta, "eps": 1e-5,
            "out": qn.quaternion_layer_norm_reference(qq, gamma, beta, 1e-5)}
    cases["layernorm_triton_interp_d24"] = _triton_ln_case(root)

    # --- SSM step / forward (ssm_fused.py:340-430, S broadcast fix) ---
    bsz, seqlen, dm, ds = 2, 12, 8, 16
    q = randn(bsz, dm, ds, 4) * 0.5
    Bm, Cm, h = randn(bsz, dm, ds, 4), randn(bsz, dm, ds, 4), randn(bsz, dm, ds, 4)
    S, D = randn(bsz, dm, 4), randn(bsz, dm)
    h_new, y = sf.ssm_step_reference(q, Bm, S, Cm, D, h)
    cases["ssm_step_f64"] = {"q": q, "B": Bm, "S": S, "C": Cm, "D": D, "h_prev": h,
                             "h_new": h_new, "y": y,
                             "note": "ssm_step_reference with S expanded over d_state"}
    qs = randn(bsz, seqlen, dm, ds, 4)
    qs = qs / qs.norm(dim=-1, keepdim=True) * 0.97
    Bs, Cs = randn(bsz, seqlen, dm, ds, 4), randn(bsz, seqlen, dm, ds, 4)
    Ss = randn(bsz, seqlen, dm, 4)
    Dv = randn(dm)
    Ds = Dv.view(1, 1, dm).expand(bsz, seqlen, dm)
    y_fwd = sf.ssm_forward_fused(qs, Bs, Ss, Cs, Ds)
    cases["ssm_forward_f64"] = {"q": qs, "B": Bs, "S": Ss, "C": Cs, "D": Dv, "y": y_fwd,
                                "note": "reference ssm_forward_fused CPU loop, fixed step"}

    # --- fused Cayley + scan, composed as in block._ssm_forward (block.py:214-228) ---
    delta = F.softplus(randn(bsz, seqlen, dm) - 3.0)
    lam = torch.zeros(dm, ds, 4, dtype=torch.float64)
    lam[..., 0] = -torch.exp(torch.empty(dm, ds, dtype=torch.float64).uniform_(
        torch.log(torch.tensor(1e-3)).item(), torch.log(torch.tensor(1e-1)).item(), generator=g))
    lam[..., 1:] = 0.5 * randn(dm, ds, 3)
    Bsh = randn(bsz, seqlen, ds, 4) / 8.0
    Csh = randn(bsz, seqlen, ds, 4) / 8.0
    xr = randn(bsz, seqlen, dm)
    Sq = torch.zeros(bsz, seqlen, dm, 4, dtype=torch.float64)
    Sq[..., 0] = xr
    z = delta[..., None, None] * lam[None, None]
    qz = ct.cayley_discretization_reference(z, eps=1e-6)
    Bx = Bsh[:, :, None].expand(bsz, seqlen, dm, ds, 4).contiguous()
    Cx = Csh[:, :, None].expand(bsz, seqlen, dm, ds, 4).contiguous()
    Dk = torch.ones(dm, dtype=torch.float64) + 0.1 * randn(dm)
    y_scan = sf.ssm_forward_fused(qz, Bx, Sq, Cx, Dk.view(1, 1, dm).expand(bsz, seqlen, dm))
    hT = torch.zeros(bsz, dm, ds, 4, dtype=torch.float64)
    for t in range(seqlen):
        hT, _ = sf.ssm_step_reference(qz[:, t], Bx[:, t], Sq[:, t], Cx[:, t],
                                      Dk.view(1, dm).expand(bsz, dm), hT)
    cases["scan_cayley_shared_f64"] = {
        "delta": delta, "Lambda": lam, "B": Bsh, "C": Csh, "x": xr, "D": Dk,
        "y": y_scan, "h_T": hT,
        "note": "z=delta*Lambda, cayley_discretization_reference, ssm_forward_fused "
                "(fixed step); B/C shared over channels"}

    # --- block forward (block.py:124-230), small shape, gate fix ---
    torch.manual_seed(0)
    blk = QuaternionMamba2Block(d_model=16, d_state=4, d_conv=4, expand_factor=2).double()
    xb = torch.randn(2, 10, 16, dtype=torch.float64)
    with torch.no_grad():
        xz = blk.in_proj(xb)
        x_in, zg = xz.chunk(2, dim=-1)
        xa = F.silu(blk.conv1d(x_in))
        yq = blk._ssm_forward(xa)
        yr = blk.out_proj(blk.norm(yq))
        out = xb + torch.sigmoid(zg[..., :16]) * yr
    cases["block_f64"] = {
        "state_dict": {k: v.clone() for k, v in blk.state_dict().items()},
        "config": {"d_model": 16, "d_state": 4, "d_conv": 4, "expand_factor": 2},
        "x": xb, "y_quat": yq, "out": out,
        "note": "reference block submodules in order; gate uses z[..., :d_model]"}

    torch.save({"cases": cases, "reference_sha256": _source_hashes(root),
                "torch_version": torch.__version__}, OUT)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(cases)} cases)")


if __name__ == "__main__":
    main()
