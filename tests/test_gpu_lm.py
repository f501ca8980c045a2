"""The LM wrapper (config-4 harness) on the GPU: loss and gradients against an
fp64 composition of the oracle block (embedding -> oracle blocks -> LayerNorm
-> head -> cross-entropy), activation checkpointing against the plain
backward, and a few data-parallel-harness training steps."""

import pytest
import torch
import torch.nn.functional as F

from oracle import ref
from tests.gpu_util import DEV, RTOL_F32, gen, rel_l2

pytestmark = pytest.mark.gpu

from mambaqc_b200.models import QuaternionMamba2  # noqa: E402
from mambaqc_b200.training import data_parallel, train_step  # noqa: E402

V, DM, NL, NS = 61, 32, 2, 8


def _oracle_loss(params, ids, labels):
    x = F.embedding(ids, params["embedding.weight"])
    for i in range(NL):
        pre = f"layers.{i}."
        x = ref.block_forward({k[len(pre):]: v for k, v in params.items() if k.startswith(pre)},
                              x, d_state=NS)
    x = F.layer_norm(x, (DM,), params["norm_f.weight"], params["norm_f.bias"])
    logits = F.linear(x, params["lm_head.weight"])[..., :V]
    return F.cross_entropy(logits.reshape(-1, V), labels.reshape(-1))


def test_lm_loss_and_gradients_match_oracle():
    prev = torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32
    torch.backends.cudnn.allow_tf32 = torch.backends.cuda.matmul.allow_tf32 = False
    try:
        torch.manual_seed(0)
        lm = QuaternionMamba2(V, d_model=DM, n_layers=NL, d_state=NS)
        assert lm.vocab_size_padded == 64
        g = gen(1)
        ids = torch.randint(0, V, (2, 48), generator=g)
        labels = torch.randint(0, V, (2, 48), generator=g)
        params = {k: v.detach().double().requires_grad_() for k, v in lm.state_dict().items()}
        loss_ref = _oracle_loss(params, ids, labels)
        loss_ref.backward()
        lm = lm.to(DEV)
        out = lm(ids.to(DEV), labels=labels.to(DEV))
        out["loss"].backward()
        assert out["logits"].shape == (2, 48, V)
        assert abs(out["loss"].item() - loss_ref.item()) / loss_ref.item() < RTOL_F32
        for name, p in lm.named_parameters():
            err = rel_l2(p.grad, params[name].grad)
            assert err < 1e-4, (name, err)
    finally:
        torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = prev


def test_gradient_checkpointing_matches_plain_backward():
    torch.manual_seed(0)
    lm = QuaternionMamba2(V, d_model=DM, n_layers=NL, d_state=NS).to(DEV)
    ids = torch.randint(0, V, (2, 40), generator=gen(3)).to(DEV)
    grads = []
    for ck in (False, True):
        lm.zero_grad(set_to_none=True)
        lm.gradient_checkpointing = ck
        lm.train()
        lm(ids, labels=ids)["loss"].backward()
        grads.append({n: p.grad.clone() for n, p in lm.named_parameters()})
    for n in grads[0]:
        assert rel_l2(grads[1][n], grads[0][n]) < RTOL_F32, n


def test_training_steps_reduce_the_loss():
    """Harness steps (bf16 autocast, checkpointed blocks, AdamW, clipping) on one
    repeated batch: the loss falls and stays finite."""
    torch.manual_seed(0)
    lm = data_parallel(QuaternionMamba2(V, d_model=DM, n_layers=NL, d_state=NS).to(DEV))
    assert lm.gradient_checkpointing
    opt = torch.optim.AdamW(lm.parameters(), lr=3e-3)
    seq = torch.randint(0, V, (4, 65), generator=gen(5)).to(DEV)
    losses = [train_step(lm, opt, seq[:, :-1], seq[:, 1:]).item() for _ in range(30)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < 0.8 * losses[0], losses


def test_generate_shapes_and_sampling_controls():
    torch.manual_seed(0)
    lm = QuaternionMamba2(V, d_model=DM, n_layers=NL, d_state=NS).to(DEV)
    prompt = torch.randint(0, V, (2, 5), generator=gen(6)).to(DEV)
    out = lm.generate(prompt, max_new_tokens=4, temperature=0.8, top_k=10, top_p=0.9)
    assert out.shape == (2, 9) and torch.equal(out[:, :5], prompt)
    assert int(out.max()) < V and int(out.min()) >= 0


def test_block_step_matches_forward_last_position():
    """prefill over a prompt, then single-token steps, give the same outputs as
    running the whole sequence through the block."""
    from mambaqc_b200.models import QuaternionMamba2Block
    torch.manual_seed(0)
    blk = QuaternionMamba2Block(32, d_state=8).to(DEV)
    x = torch.randn(2, 20, 32, generator=gen(7)).to(DEV)
    with torch.no_grad():
        full = blk(x)
        out, cache = blk.prefill(x[:, :2])
        assert rel_l2(out, full[:, :2]) < RTOL_F32
        for t in range(2, 20):
            y_t = blk.step(x[:, t], cache)
            assert rel_l2(y_t, full[:, t]) < RTOL_F32, t


def test_cached_greedy_generation_matches_full_recompute():
    torch.manual_seed(0)
    lm = QuaternionMamba2(V, d_model=DM, n_layers=NL, d_state=NS).to(DEV)
    prompt = torch.randint(0, V, (2, 6), generator=gen(8)).to(DEV)
    a = lm.generate(prompt, max_new_tokens=12, top_k=1)
    b = lm.generate(prompt, max_new_tokens=12, top_k=1, use_cache=True)
    assert torch.equal(a, b)
