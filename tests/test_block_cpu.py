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


def test_lm_structure_and_init_follow_the_reference_layout():
    """Parameter names, vocabulary padding and init of the LM wrapper
    (models/quaternion_mamba2.py:29-95), built on the CPU without running it."""
    import torch
    from mambaqc_b200.models import QuaternionMamba2, QuaternionMamba2Block

    torch.manual_seed(0)
    lm = QuaternionMamba2(100, d_model=16, n_layers=2, d_state=4)
    assert lm.vocab_size_padded == 104
    keys = list(lm.state_dict())
    assert keys[0] == "embedding.weight" and keys[-3:] == ["norm_f.weight", "norm_f.bias",
                                                           "lm_head.weight"]
    blk = set(QuaternionMamba2Block(16, d_state=4).state_dict())
    for i in range(2):
        assert {k[len(f"layers.{i}."):] for k in keys if k.startswith(f"layers.{i}.")} == blk
    assert abs(lm.embedding.weight.std().item() - 0.02) < 0.005
    assert abs(lm.layers[0].in_proj.weight.std().item() - 0.02) < 0.005
    assert lm.get_num_params() == sum(p.numel() for p in lm.parameters()) - 2 * 104 * 16


def test_oracle_block_ssm_channel_subset_matches_full_block():
    """The oracle's channel-subset SSM (used by the config-4 GPU test to check
    sampled channels) equals the same channels of the full oracle block SSM."""
    from oracle import ref

    torch.manual_seed(0)
    blk = QuaternionMamba2Block(16, d_state=4)
    params = {k: v.double() for k, v in blk.state_dict().items()}
    x = torch.randn(2, 12, 16, generator=torch.Generator().manual_seed(1), dtype=torch.float64)
    _, h_full = ref.block_forward(params, x, d_state=4, return_state=True)
    chans = torch.tensor([0, 5, 31])
    _, h_sub = ref.block_ssm_channels(params, x, 4, chans)
    assert torch.allclose(h_sub, h_full[:, chans], rtol=1e-12, atol=1e-14)
