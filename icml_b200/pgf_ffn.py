"""FFN with the API of the reference's pgf_ffn.py (pgf_ffn_forward :261-307, pgf_ffn_grad :183-258).

The CUDA operator tiles the rows itself, so ``block_size`` only shapes the ``streaming`` callback
blocks.  ``grad_W1`` is computed (the reference's block function returns it undefined).
"""
from __future__ import annotations

import torch

from . import ops


@torch.no_grad()
def pgf_ffn_forward(x: torch.Tensor, W1: torch.Tensor, b1: torch.Tensor, W2: torch.Tensor,
                    b2: torch.Tensor, block_size: int = 512, activation: str = "gelu",
                    streaming: bool = False, callback=None):
    y = ops.ffn_fwd(x, W1, b1, W2, b2, activation)
    if streaming:
        if callback:
            for start in range(0, y.shape[0], block_size):
                end = min(start + block_size, y.shape[0])
                callback(y[start:end], start, end)
        return None
    return y


@torch.no_grad()
def pgf_ffn_grad(x: torch.Tensor, g_out: torch.Tensor, W1: torch.Tensor, b1: torch.Tensor,
                 W2: torch.Tensor, b2: torch.Tensor, block_size: int = 512, activation: str = "gelu",
                 compute_input_grads: bool = False, fp32_accum: bool = True):
    if activation not in ("gelu", "relu"):
        raise ValueError(f"Unsupported activation: {activation}")
    r = ops.ffn_bwd(x.detach(), g_out.detach(), W1, b1, W2, activation, need_gx=compute_input_grads)
    out = {"grad_W1": r["grad_W1"].to(W1.dtype), "grad_b1": r["grad_b1"].to(b1.dtype),
           "grad_W2": r["grad_W2"].to(W2.dtype), "grad_b2": r["grad_b2"].to(b2.dtype)}
    if compute_input_grads:
        out["grad_x"] = r["grad_x"].to(x.dtype)
    return out


class FFNFunction(torch.autograd.Function):
    """Autograd wrapper: y = act(x W1^T + b1) W2^T + b2 with the fused CUDA backward."""

    @staticmethod
    def forward(ctx, x, W1, b1, W2, b2, activation="gelu"):
        ctx.save_for_backward(x, W1, b1, W2)
        ctx.activation = activation
        return ops.ffn_fwd(x, W1, b1, W2, b2, activation)

    @staticmethod
    def backward(ctx, gy):
        x, W1, b1, W2 = ctx.saved_tensors
        r = ops.ffn_bwd(x, gy, W1, b1, W2, ctx.activation, need_gx=ctx.needs_input_grad[0])
        return (r.get("grad_x"), r["grad_W1"], r["grad_b1"], r["grad_W2"], r["grad_b2"], None)


@torch.no_grad()
def pgf_ffn_jvp(x: torch.Tensor, x_dot: torch.Tensor, W1: torch.Tensor, W1_dot: torch.Tensor, b1: torch.Tensor,
                b1_dot: torch.Tensor, W2: torch.Tensor, W2_dot: torch.Tensor, b2: torch.Tensor, b2_dot: torch.Tensor,
                block_size: int = 512, activation: str = "gelu"):
    """pgf_ffn.py:146-180: (y, y_dot) of the FFN along every input's tangent; rows in workspace-bounded
    tiles (block_size is accepted for signature compatibility)."""
    return ops.ffn_jvp(x.detach(), x_dot.detach(), W1, W1_dot, b1, b1_dot, W2, W2_dot, b2, b2_dot, activation)


__all__ = ["pgf_ffn_grad", "pgf_ffn_forward", "pgf_ffn_jvp", "FFNFunction"]
