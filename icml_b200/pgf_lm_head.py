"""LM head with the API of the reference's pgf_lm_head.py (:45-130), plus the fused
vocab-tiled LM head + cross entropy used by the training step (the reference's callers build the
full (T, V) logits and softmax, test_multi_layer_grads.py:74-86)."""
from __future__ import annotations

import torch

from . import ops


@torch.no_grad()
def pgf_lm_head_forward(hidden: torch.Tensor, W_lm_head: torch.Tensor, block_size: int = 512,
                        streaming: bool = False, callback=None):
    """pgf_lm_head.py:96-130: logits = hidden W^T (float32)."""
    logits = ops.lm_head_fwd(hidden, W_lm_head)
    if streaming:
        if callback:
            for start in range(0, logits.shape[0], block_size):
                end = min(start + block_size, logits.shape[0])
                callback(logits[start:end], start, end)
        return None
    return logits


@torch.no_grad()
def pgf_lm_head_grad(hidden: torch.Tensor, g_logits: torch.Tensor, W_lm_head: torch.Tensor,
                     block_size: int = 512, compute_input_grads: bool = True, fp32_accum: bool = True):
    """pgf_lm_head.py:45-93: {"grad_W_lm_head"[, "grad_hidden"]}."""
    gW, gh = ops.lm_head_bwd(hidden.detach(), g_logits.detach(), W_lm_head, need_gh=compute_input_grads)
    res = {"grad_W_lm_head": gW.to(W_lm_head.dtype)}
    if compute_input_grads:
        res["grad_hidden"] = gh.to(hidden.dtype)
    return res


@torch.no_grad()
def pgf_lm_head_ce_forward(hidden: torch.Tensor, W_lm_head: torch.Tensor, targets: torch.Tensor):
    """Mean cross entropy of logits = hidden W^T against targets, without materialising the
    logits.  Returns (loss (0-d float32 tensor), lse (T,) float32 for the backward)."""
    loss_rows, lse = ops.lm_head_ce_fwd(hidden.reshape(-1, hidden.shape[-1]), W_lm_head, targets.reshape(-1))
    return loss_rows.mean(), lse


@torch.no_grad()
def pgf_lm_head_ce_grad(hidden: torch.Tensor, W_lm_head: torch.Tensor, targets: torch.Tensor,
                        lse: torch.Tensor, grad_scale: float = None, compute_input_grads: bool = True):
    """Gradients of the mean cross entropy: {"grad_W_lm_head"[, "grad_hidden"]}; grad_scale
    defaults to 1/T (the mean)."""
    h = hidden.reshape(-1, hidden.shape[-1])
    scale = (1.0 / h.shape[0]) if grad_scale is None else grad_scale
    gW, gh = ops.lm_head_ce_bwd(h, W_lm_head, targets.reshape(-1), lse, scale, need_gh=compute_input_grads)
    res = {"grad_W_lm_head": gW}
    if compute_input_grads:
        res["grad_hidden"] = gh.reshape(hidden.shape)
    return res


__all__ = ["pgf_lm_head_forward", "pgf_lm_head_grad", "pgf_lm_head_ce_forward", "pgf_lm_head_ce_grad"]
