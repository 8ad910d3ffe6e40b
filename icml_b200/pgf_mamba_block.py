"""PGFMambaBlock / PGFMambaSequential with the API of the reference's pgf_mamba_block.py
(:16-322), on libpgf.so.

pgf_forward runs the whole sequence through the chunked CUDA scan (the reference loops over
blocks of ``block_size`` in Python; the kernels keep per-chunk boundary states instead of the
(L, B, d, N) trajectory, which is the same O(1)-in-L state memory).  pgf_backward recomputes the
forward from the layer input exactly as the reference does (:155-179) and returns the same
gradient dictionary (:137-153) and ``grad_input``.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .pgf_ffn import FFNFunction, pgf_ffn_grad
from .pgf_rmsnorm import RMSNorm
from .train_singlemamba_optimized import SingleLayerMambaPGF, _cat_weights


class PGFMambaBlock(nn.Module):
    """x -> RMSNorm -> SSM -> +x -> RMSNorm -> FFN -> +x (pgf_mamba_block.py:16-68)."""

    def __init__(self, d_model: int, d_state: int = 16, d_ff: Optional[int] = None,
                 block_size: int = 128, output_activation: Optional[str] = None,
                 ffn_activation: str = "gelu"):
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.d_ff = d_ff or 4 * d_model
        self.block_size = block_size
        self.ffn_activation = ffn_activation
        self.norm1 = RMSNorm(d_model)
        self.mamba = SingleLayerMambaPGF(d_model, d_state, output_activation=output_activation)
        self.norm2 = RMSNorm(d_model)
        self.W1 = nn.Parameter(torch.randn(self.d_ff, d_model) * 0.02)
        self.b1 = nn.Parameter(torch.zeros(self.d_ff))
        self.W2 = nn.Parameter(torch.randn(d_model, self.d_ff) * 0.02)
        self.b2 = nn.Parameter(torch.zeros(d_model))
        nn.init.xavier_uniform_(self.W1)
        nn.init.xavier_uniform_(self.W2)

    @property
    def reference_scale_grad(self) -> bool:
        return self.mamba.reference_scale_grad

    @reference_scale_grad.setter
    def reference_scale_grad(self, v: bool):
        self.mamba.reference_scale_grad = bool(v)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Autograd forward (pgf_mamba_block.py:51-68) through the CUDA autograd functions."""
        res = x
        x = self.norm1(x)
        x = self.mamba.forward_standard(x)
        x = x + res
        res = x
        h = self.norm2(x)
        B, L, D = h.shape
        f = FFNFunction.apply(h.reshape(-1, D), self.W1, self.b1, self.W2, self.b2, self.ffn_activation)
        return f.reshape(B, L, D) + res

    @torch.no_grad()
    def pgf_forward(self, x: torch.Tensor, return_ssm_states: bool = False, keep_scan: bool = False):
        """pgf_mamba_block.py:70-126.  With return_ssm_states, also the scan's boundary states (for
        pgf_backward(..., ssm_states=...), which then need not recompute them).  With keep_scan as
        well, what is returned instead is everything the backward's recompute of the scan produces
        (the scan's saved states and the residual sum y + x), so the backward runs no scan pass before
        its scan backward.  That holds, per block until its backward, about 8.5 bytes per token and
        channel of scan states (an 8-token checkpoint of the 16 states) and y + x in the activation
        dtype."""
        B, L, D = x.shape
        xn = self.norm1.pgf_forward(x, block_size=self.block_size)
        st = None
        if return_ssm_states and keep_scan:
            W, b = _cat_weights(self.mamba)
            m = self.mamba
            y, saved = ops.ssm_fwd_save(xn, W, b, m.A_log, m.D, m.scale, act=m.output_activation)
            x1, xn2 = ops.rmsnorm_fwd_res(y, x, self.norm2.weight, self.norm2.eps)
            st = {"saved": saved, "m_out": x1}
        elif return_ssm_states:
            W, b = _cat_weights(self.mamba)
            m = self.mamba
            y, st = ops.ssm_fwd_states(xn, W, b, m.A_log, m.D, m.scale, act=m.output_activation)
        else:
            y, _ = self.mamba.ssm_forward(xn)
        if not isinstance(st, dict):
            # x1 = y + x and norm2(x1) in one pass (same bits as the separate add and norm)
            x1, xn2 = ops.rmsnorm_fwd_res(y, x, self.norm2.weight, self.norm2.eps)
        # ffn(norm2(x1)) + x1 (:120-126), the skip connection added in the FFN's last epilogue
        out = ops.ffn_fwd(xn2.reshape(-1, D), self.W1, self.b1, self.W2, self.b2, self.ffn_activation,
                          residual=x1.reshape(-1, D)).reshape(B, L, D)
        return (out, st) if return_ssm_states else out

    @torch.no_grad()
    def pgf_backward(self, x: torch.Tensor, g_out: torch.Tensor, fp32_accum: bool = True,
                     ssm_states: Optional[torch.Tensor] = None) -> Dict[str, Any]:
        """pgf_mamba_block.py:128-249.  ssm_states: what pgf_forward returned for the same x -- the
        boundary states (the recompute then runs one scan pass instead of rebuilding them, :157-175),
        or, from pgf_forward(keep_scan=True), the scan's saved states and y + x (no scan recompute)."""
        B, L, D = x.shape
        g_out = g_out.to(x.dtype)
        xn1 = self.norm1.pgf_forward(x, block_size=self.block_size)              # :157
        W, b = _cat_weights(self.mamba)
        m = self.mamba
        if isinstance(ssm_states, dict):
            saved, m_out = ssm_states["saved"], ssm_states["m_out"]
            xn2 = ops.rmsnorm_fwd(m_out, self.norm2.weight, self.norm2.eps)        # :179
        else:
            # :163-178; the states it passes through are kept for the scan backward below
            y, saved = ops.ssm_fwd_save(xn1, W, b, m.A_log, m.D, m.scale, act=m.output_activation,
                                        states=ssm_states)
            m_out, xn2 = ops.rmsnorm_fwd_res(y, x, self.norm2.weight, self.norm2.eps)  # y + x, :179
        fr = pgf_ffn_grad(xn2.reshape(-1, D), g_out.reshape(-1, D), self.W1, self.b1, self.W2, self.b2,
                          block_size=self.block_size, activation=self.ffn_activation,
                          compute_input_grads=True)                              # :183-192
        # :196 and :202 (norm2's grad_x + g_out) in one pass
        gw2, g_m = ops.rmsnorm_bwd(m_out, fr["grad_x"].reshape(B, L, D), self.norm2.weight, self.norm2.eps,
                                   g_add=g_out)
        r = ops.ssm_bwd(xn1, g_m, W, b, m.A_log, m.D, m.scale, act=m.output_activation,
                        saved=saved)                                             # :206-234
        del saved
        # :237-242 and :246-249 (norm1's grad_x + g_m) in one pass
        gw1, grad_input = ops.rmsnorm_bwd(x, r["grad_u"], self.norm1.weight, self.norm1.eps, g_add=g_m)
        d, N = self.d_model, self.d_state
        gscale = r["scale"].sum().expand(d).clone() if m.reference_scale_grad else r["scale"]
        grads = {
            "W1": fr["grad_W1"], "b1": fr["grad_b1"], "W2": fr["grad_W2"], "b2": fr["grad_b2"],
            "mamba.A_log": r["A_log"], "mamba.D": r["D"], "mamba.scale": gscale,
            "mamba.dt_proj.weight": r["W_cat"][:d], "mamba.dt_proj.bias": r["b_cat"][:d],
            "mamba.B_proj.weight": r["W_cat"][d:d + N], "mamba.B_proj.bias": r["b_cat"][d:d + N],
            "mamba.C_proj.weight": r["W_cat"][d + N:], "mamba.C_proj.bias": r["b_cat"][d + N:],
            "norm1.weight": gw1, "norm2.weight": gw2,
        }
        return {"grads": grads, "grad_input": grad_input}

    @torch.no_grad()
    def pgf_forward_mamba_only(self, x_norm: torch.Tensor) -> torch.Tensor:
        """pgf_mamba_block.py:251-275."""
        y, _ = self.mamba.ssm_forward(x_norm)
        return y


class PGFMambaSequential(nn.Module):
    """pgf_mamba_block.py:277-322."""

    def __init__(self, layers: List[PGFMambaBlock]):
        super().__init__()
        self.layers = nn.ModuleList(layers)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for layer in self.layers:
            x = layer(x)
        return x

    @torch.no_grad()
    def pgf_train_step(self, x: torch.Tensor, target: torch.Tensor, loss_fn: Any) -> Dict[str, Any]:
        layer_inputs = []
        cur = x
        for layer in self.layers:
            layer_inputs.append(cur.detach().clone())
            cur = layer.pgf_forward(cur)
        loss, g_out = loss_fn(cur, target)
        all_grads = {}
        g = g_out
        for i in reversed(range(len(self.layers))):
            res = self.layers[i].pgf_backward(layer_inputs.pop(), g)
            for k, v in res["grads"].items():
                all_grads[f"layers.{i}.{k}"] = v
            g = res["grad_input"]
            del res
        return {"loss": loss, "grads": all_grads}


__all__ = ["PGFMambaBlock", "PGFMambaSequential"]
