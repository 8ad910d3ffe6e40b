"""Embedding with the API of the reference's pgf_embedding.py (:14-124).

The gradient is deterministic: a stable radix sort of the ids followed by an ordered segment sum
(the reference's ``index_add_`` is atomic, hence order-dependent, on CUDA).
"""
from __future__ import annotations

import torch

from . import ops


@torch.no_grad()
def pgf_embedding_forward(input_ids: torch.Tensor, weight: torch.Tensor, block_size: int = 512,
                          streaming: bool = False, callback=None, out_dtype=None):
    """pgf_embedding.py:74-124; ``out_dtype`` (default: weight's) selects bf16 activations."""
    dt = out_dtype or (weight.dtype if weight.dtype in (torch.float32, torch.bfloat16) else torch.float32)
    y = ops.embedding_fwd(input_ids, weight, dtype=dt)
    if streaming:
        if callback:
            flat = y.reshape(-1, y.shape[-1])
            for start in range(0, flat.shape[0], block_size):
                end = min(start + block_size, flat.shape[0])
                callback(flat[start:end], start, end)
        return None
    return y


@torch.no_grad()
def pgf_embedding_grad(input_ids: torch.Tensor, g_out: torch.Tensor, weight: torch.Tensor,
                       block_size: int = 512, compute_input_grads: bool = False,
                       fp32_accum: bool = True):
    """pgf_embedding.py:14-71: {"grad_weight": (vocab, d)}."""
    gw = ops.embedding_bwd(input_ids.detach(), g_out.detach(), weight.shape[0])
    return {"grad_weight": gw.to(weight.dtype)}


__all__ = ["pgf_embedding_grad", "pgf_embedding_forward"]
