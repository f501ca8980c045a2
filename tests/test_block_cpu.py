"""Block shell checks that need no GPU: parameter names, shapes and seeded
initialisation equal the reference block's (golden state_dict made by the
reference under torch.manual_seed(0)), and the alias installer."""

import sys

import torch

from mambaqc_b200.models import QuaternionMamba2Block


def test_block_state_dict_matches_reference(golden):
    c = golden["block_f64"]
    cfg = c["config"]
    torch.manual_seed(0)
    blk = QuaternionMamba2Block(cfg["d_model"], d_state=cfg["d_state"], d_conv=cfg["d_conv"],
                                expand_factor=cfg["expand_factor"])
    mine = blk.state_dict()
    ref = c["state_dict"]
    assert sorted(mine) == sorted(ref)
    for k in ref:
        assert mine[k].shape == ref[k].shape, k
        assert torch.equal(mine[k].double(), ref[k]), k  # same RNG consumption order


def test_block_loads_reference_checkpoint(golden):
    c = golden["block_f64"]
    blk = QuaternionMamba2Block(16, d_state=4)
    missing, unexpected = blk.load_state_dict({k: v.float() for k, v in c["state_dict"].items()})
    assert not missing and not unexpected


def test_lambda_parameterisation_is_stable():
    blk = QuaternionMamba2Block(8, d_state=4)
    lam = blk.ssm_lambda()
    assert lam.shape == (16, 4, 4)
    assert torch.all(lam[..., 0] < 0)
    assert torch.all(lam[..., 1:].abs() < 1)


def test_install_as_mambaqc_aliases_modules():
    import mambaqc_b200
    saved = {k: v for k, v in sys.modules.items() if k == "mambaqc" or k.startswith("mambaqc.")}
    try:
        mambaqc_b200.install_as_mambaqc()
        from mambaqc.kernels.quaternion_ops import quaternion_multiply
        from mambaqc.layers import QuaternionLayerNorm
        from mambaqc.models.quaternion_mamba2_block import QuaternionMamba2Block as Blk
        import mambaqc_b200.kernels.quaternion_ops as qo
        assert quaternion_multiply is qo.quaternion_multiply
        assert Blk is QuaternionMamba2Block
        assert QuaternionLayerNorm.__module__.startswith("mambaqc_b200")
    finally:
        for k in [k for k in sys.modules if k == "mambaqc" or k.startswith("mambaqc.")]:
            del sys.modules[k]
        sys.modules.update(saved)
