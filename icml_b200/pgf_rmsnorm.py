"""RMSNorm with the API of the reference's pgf_rmsnorm.py (RMSNorm, :75-214), on libpgf.so.

``block_size`` and ``fp32_accum`` are accepted for compatibility: the CUDA kernels stream
through the rows with bounded scratch and always accumulate in float32.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import ops


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        ctx.save_for_backward(x, weight)
        ctx.eps = eps
        return ops.rmsnorm_fwd(x, weight, eps)

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        gw, gx = ops.rmsnorm_bwd(x, gy, w, ctx.eps, need_gx=ctx.needs_input_grad[0])
        return gx, gw.to(w.dtype), None


class RMSNorm(nn.Module):
    """y = x / sqrt(mean(x^2) + eps) * weight (pgf_rmsnorm.py:75-87)."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _RMSNormFn.apply(x, self.weight, self.eps)

    @torch.no_grad()
    def pgf_forward(self, x: torch.Tensor, block_size: int = 512) -> torch.Tensor:
        """pgf_rmsnorm.py:89-117."""
        return ops.rmsnorm_fwd(x, self.weight, self.eps)

    @torch.no_grad()
    def pgf_jvp(self, x: torch.Tensor, x_dot: torch.Tensor, weight_dot: torch.Tensor,
                block_size: int = 512):
        """pgf_rmsnorm.py:119-155: (y, y_dot) along (x_dot, weight_dot), one pass over all rows."""
        return ops.rmsnorm_jvp(x.detach(), x_dot.detach(), self.weight, weight_dot, self.eps)

    @torch.no_grad()
    def pgf_grad(self, x: torch.Tensor, g_out: torch.Tensor, block_size: int = 512,
                 fp32_accum: bool = True, compute_input_grads: bool = False) -> dict:
        """pgf_rmsnorm.py:157-214: {"grad_weight"[, "grad_x"]}."""
        gw, gx = ops.rmsnorm_bwd(x.detach(), g_out.detach(), self.weight, self.eps,
                                 need_gx=compute_input_grads)
        res = {"grad_weight": gw.to(self.weight.dtype)}
        if compute_input_grads:
            res["grad_x"] = gx
        return res


__all__ = ["RMSNorm"]
