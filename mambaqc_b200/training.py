"""Data-parallel training step of the LM (the config-4 harness).

One process per GPU: ``data_parallel(model)`` wraps the model in
``DistributedDataParallel``. Its gradient all-reduce runs over NCCL in buckets
that are launched while the backward is still running (``bucket_cap_mb``), and
gradients are views into those buckets (no copy). ``train_step`` runs forward +
loss under bf16 autocast (the scan state stays fp32 inside the kernels),
backward, gradient clipping and the optimizer step. It is one step of the
reference trainer without gradient accumulation:
- forward with labels under bf16 autocast, then backward (train.py:154-180);
- clipping at ``grad_clip``, the optimizer step and zeroing the gradients
  (train.py:182-206).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel

__all__ = ["data_parallel", "train_step"]


def data_parallel(model: torch.nn.Module, bucket_cap_mb: int = 64,
                  gradient_checkpointing: bool = True) -> torch.nn.Module:
    """The model wrapped for data parallelism over the default process group
    (returned unchanged when there is no group or it has one rank)."""
    if hasattr(model, "gradient_checkpointing"):
        model.gradient_checkpointing = gradient_checkpointing
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return model
    dev = next(model.parameters()).device
    return DistributedDataParallel(model, device_ids=[dev.index] if dev.type == "cuda" else None,
                                   bucket_cap_mb=bucket_cap_mb, gradient_as_bucket_view=True)


def train_step(model: torch.nn.Module, optimizer: torch.optim.Optimizer,
               input_ids: torch.Tensor, labels: torch.Tensor, grad_clip: float = 1.0,
               autocast_dtype: torch.dtype | None = torch.bfloat16) -> torch.Tensor:
    """One optimizer step on a batch; returns the loss (a device scalar, not
    synchronised)."""
    model.train()
    optimizer.zero_grad(set_to_none=True)
    if autocast_dtype is not None:
        with torch.autocast("cuda", dtype=autocast_dtype):
            loss = model(input_ids, labels=labels)["loss"]
    else:
        loss = model(input_ids, labels=labels)["loss"]
    loss.backward()
    if grad_clip is not None and grad_clip > 0:
        torch.nn.utils.clip_grad_norm_(model.parameters(), grad_clip)
    optimizer.step()
    return loss.detach()
