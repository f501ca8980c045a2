"""QuaternionMamba2 language model: drop-in for
``mambaqc.models.quaternion_mamba2.QuaternionMamba2``. It is the harness of the
config-4 training step; the blocks run the fused GPU path.

Constructor arguments, submodule and parameter names (``embedding``,
``layers``, ``norm_f``, ``lm_head``), the vocabulary padding and the weight
initialisation order follow the reference (models/quaternion_mamba2.py:29-95),
so a reference state_dict loads unchanged and ``torch.manual_seed(s)`` gives the
same initial weights. ``forward(input_ids, labels)`` returns
``{"logits", "loss"}`` as the reference does (:97-167). ``generate``
re-runs the prompt plus the tokens so far through the model for each new token,
with the same sampling controls (:169-227).

Addition: ``gradient_checkpointing`` (off by default) recomputes each block in
the backward instead of keeping its activations. Without it, one block of the
base preset holds two [B, T, d_inner, N, 4] B/C activations (6.4 GB each in
bf16 at B=4, T=2048).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F
import torch.utils.checkpoint as ckpt

from mambaqc_b200.models.quaternion_mamba2_block import QuaternionMamba2Block

__all__ = ["QuaternionMamba2", "quaternion_mamba2_small", "quaternion_mamba2_base",
           "quaternion_mamba2_large"]


class QuaternionMamba2(nn.Module):
    """Embedding -> n_layers QuaternionMamba2Block -> LayerNorm -> LM head."""

    def __init__(self, vocab_size: int, d_model: int = 768, n_layers: int = 12,
                 d_state: int = 64, d_conv: int = 4, expand_factor: int = 2,
                 pad_vocab_size_multiple: int = 8, bias: bool = False, dropout: float = 0.0):
        super().__init__()
        self.vocab_size = vocab_size
        self.d_model = d_model
        self.n_layers = n_layers
        m = pad_vocab_size_multiple
        self.vocab_size_padded = -(-vocab_size // m) * m if m > 1 else vocab_size
        self.embedding = nn.Embedding(self.vocab_size_padded, d_model)
        self.dropout = nn.Dropout(dropout) if dropout > 0.0 else nn.Identity()
        self.layers = nn.ModuleList([
            QuaternionMamba2Block(d_model=d_model, d_state=d_state, d_conv=d_conv,
                                  expand_factor=expand_factor, bias=bias)
            for _ in range(n_layers)])
        self.norm_f = nn.LayerNorm(d_model)
        self.lm_head = nn.Linear(d_model, self.vocab_size_padded, bias=False)
        self.gradient_checkpointing = False
        self.apply(self._init_weights)

    @staticmethod
    def _init_weights(module: nn.Module) -> None:
        # N(0, 0.02) for linear and embedding weights, zero biases, unit LayerNorm
        if isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
        elif isinstance(module, nn.LayerNorm):
            nn.init.ones_(module.weight)
            nn.init.zeros_(module.bias)

    def forward(self, input_ids: torch.Tensor, labels: torch.Tensor | None = None):
        assert input_ids.min() >= 0, f"Negative token index: {input_ids.min().item()}"
        assert input_ids.max() < self.vocab_size, \
            f"Token index {input_ids.max().item()} >= vocab_size {self.vocab_size}"
        x = self.dropout(self.embedding(input_ids))
        for layer in self.layers:
            if self.gradient_checkpointing and self.training and torch.is_grad_enabled():
                x = ckpt.checkpoint(layer, x, use_reentrant=False)
            else:
                x = layer(x)
        logits = self.lm_head(self.norm_f(x))[..., : self.vocab_size]
        loss = None
        if labels is not None:
            valid = labels[labels != -100]
            if valid.numel() > 0:
                assert valid.min() >= 0, f"Negative label: {valid.min().item()}"
                assert valid.max() < self.vocab_size, \
                    f"Label {valid.max().item()} >= vocab_size {self.vocab_size}"
            loss = F.cross_entropy(logits.reshape(-1, self.vocab_size), labels.reshape(-1),
                                   ignore_index=-100)
        return {"logits": logits, "loss": loss}

    @torch.no_grad()
    def _next_logits_cached(self, input_ids: torch.Tensor, caches: list | None):
        """Logits of the next token. With ``caches`` None the prompt is run
        through every block's ``prefill`` and the caches are made; otherwise the
        last token alone is stepped through the blocks (recurrent decoding)."""
        if caches is None:
            x = self.embedding(input_ids)
            caches = []
            for layer in self.layers:
                x, c = layer.prefill(x)
                caches.append(c)
            x = x[:, -1]
        else:
            x = self.embedding(input_ids[:, -1])
            for layer, c in zip(self.layers, caches):
                x = layer.step(x, c)
        return self.lm_head(self.norm_f(x))[..., : self.vocab_size], caches

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 100,
                 temperature: float = 1.0, top_k: int | None = None,
                 top_p: float | None = None, use_cache: bool = False) -> torch.Tensor:
        """Sample max_new_tokens tokens after the prompt; returns [B, T + new].

        ``use_cache`` (an addition; off by default, as the reference always
        recomputes) keeps each block's conv inputs and SSM state and advances
        them one token at a time, so each new token costs one step instead of a
        pass over the whole sequence."""
        self.eval()
        caches = None
        for _ in range(max_new_tokens):
            if use_cache:
                logits, caches = self._next_logits_cached(input_ids, caches)
                nxt = logits / temperature
            else:
                nxt = self.forward(input_ids)["logits"][:, -1, :] / temperature
            if top_k is not None:
                kth = torch.topk(nxt, top_k, dim=-1).values[..., -1:]
                nxt = nxt.masked_fill(nxt < kth, float("-inf"))
            if top_p is not None:
                srt, idx = torch.sort(nxt, descending=True, dim=-1)
                cum = torch.cumsum(torch.softmax(srt, dim=-1), dim=-1)
                drop = cum > top_p
                drop[..., 1:] = drop[..., :-1].clone()   # keep the token that crosses top_p
                drop[..., 0] = False
                nxt = nxt.masked_fill(drop.scatter(-1, idx, drop), float("-inf"))
            tok = torch.multinomial(torch.softmax(nxt, dim=-1), num_samples=1)
            input_ids = torch.cat([input_ids, tok], dim=1)
        return input_ids

    def get_num_params(self, non_embedding: bool = True) -> int:
        n = sum(p.numel() for p in self.parameters())
        if non_embedding:
            n -= self.embedding.weight.numel()
            if self.lm_head.weight is not self.embedding.weight:
                n -= self.lm_head.weight.numel()
        return n

    def estimate_mfu(self, fwdbwd_per_iter: int, dt: float,
                     flops_promised: float = 2.25e15) -> float:
        """The reference's rough model-FLOPs utilisation (6 N FLOPs per token,
        times 4 for the quaternion algebra, 2048-token sequences), against
        ``flops_promised`` (default: B200 dense bf16, 2.25 PFLOP/s; the
        reference assumed an A100's 312 TFLOP/s)."""
        flops_per_iter = 6 * self.get_num_params() * 4 * 2048 * fwdbwd_per_iter
        return flops_per_iter / dt / flops_promised


def quaternion_mamba2_small(vocab_size: int) -> QuaternionMamba2:
    return QuaternionMamba2(vocab_size=vocab_size, d_model=512, n_layers=8, d_state=32)


def quaternion_mamba2_base(vocab_size: int) -> QuaternionMamba2:
    return QuaternionMamba2(vocab_size=vocab_size, d_model=768, n_layers=12, d_state=64)


def quaternion_mamba2_large(vocab_size: int) -> QuaternionMamba2:
    return QuaternionMamba2(vocab_size=vocab_size, d_model=1024, n_layers=24, d_state=64)
