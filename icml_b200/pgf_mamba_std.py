"""Mamba-standard variant of the PGF block, on libpgf.so.

The reference's PGFMambaBlock (pgf_mamba_block.py:16-249) wraps its own simplified SSM.  The
8-layer d_inner-512 and 24-layer d_model-1024 LM configurations use the standard Mamba mixer (in_proj, causal
depthwise conv1d + SiLU, x_proj, low-rank dt_proj, per-channel A, gate SiLU(z), out_proj); the
reference has no code for it.  `PGFMambaStdBlock` keeps the reference block's structure and PGF
API (pgf_forward / pgf_backward returning {"grads", "grad_input"}) around that mixer; parameter
names follow the common Mamba naming (in_proj, conv1d, x_proj, dt_proj, A_log, D, out_proj).
"""
from __future__ import annotations

import math
from typing import Any, Dict, Optional

import torch
import torch.nn as nn

from . import ops
from .pgf_ffn import FFNFunction, pgf_ffn_grad
from .pgf_rmsnorm import RMSNorm

_GRAD_NAMES = {"in_w": "in_proj.weight", "conv_w": "conv1d.weight", "conv_b": "conv1d.bias",
               "x_w": "x_proj.weight", "dt_w": "dt_proj.weight", "dt_b": "dt_proj.bias", "A_log": "A_log",
               "D": "D", "out_w": "out_proj.weight"}


class MambaMixer(nn.Module):
    """Standard Mamba mixer (Gu & Dao 2023) with the standard initialisation."""

    def __init__(self, d_model: int, d_state: int = 16, expand: int = 2, d_conv: int = 4,
                 dt_rank: Optional[int] = None, dt_min: float = 1e-3, dt_max: float = 1e-1):
        super().__init__()
        self.d_model, self.d_state, self.d_conv = d_model, d_state, d_conv
        self.d_inner = E = expand * d_model
        self.dt_rank = R = dt_rank or math.ceil(d_model / 16)
        self.in_proj = nn.Linear(d_model, 2 * E, bias=False)
        self.conv1d = nn.Conv1d(E, E, d_conv, groups=E, padding=d_conv - 1, bias=True)
        self.x_proj = nn.Linear(E, R + 2 * d_state, bias=False)
        self.dt_proj = nn.Linear(R, E, bias=True)
        nn.init.uniform_(self.dt_proj.weight, -R ** -0.5, R ** -0.5)
        dt = torch.exp(torch.rand(E) * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min)).clamp(min=1e-4)
        with torch.no_grad():
            self.dt_proj.bias.copy_(dt + torch.log(-torch.expm1(-dt)))
        self.A_log = nn.Parameter(torch.log(torch.arange(1, d_state + 1, dtype=torch.float32)).repeat(E, 1))
        self.D = nn.Parameter(torch.ones(E))
        self.out_proj = nn.Linear(E, d_model, bias=False)

    def params(self) -> Dict[str, torch.Tensor]:
        return {"in_w": self.in_proj.weight, "conv_w": self.conv1d.weight.view(self.d_inner, self.d_conv),
                "conv_b": self.conv1d.bias, "x_w": self.x_proj.weight, "dt_w": self.dt_proj.weight,
                "dt_b": self.dt_proj.bias, "A_log": self.A_log, "D": self.D, "out_w": self.out_proj.weight}

    def grads_to_named(self, g: Dict[str, torch.Tensor], prefix: str = "") -> Dict[str, torch.Tensor]:
        out = {}
        for k, n in _GRAD_NAMES.items():
            v = g[k]
            if k == "conv_w":
                v = v.view(self.d_inner, 1, self.d_conv)
            out[prefix + n] = v
        return out

    def forward(self, x):
        return _MixerFn.apply(x, *[self.params()[k] for k in ops.MIXER_KEYS])


class _MixerFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, *ws):
        p = dict(zip(ops.MIXER_KEYS, ws))
        ctx.save_for_backward(x, *ws)
        return ops.mamba_mixer_fwd(x, p)

    @staticmethod
    def backward(ctx, gy):
        x, *ws = ctx.saved_tensors
        g, gx = ops.mamba_mixer_bwd(x, gy, dict(zip(ops.MIXER_KEYS, ws)))
        return (gx, *[g[k].view_as(w) for k, w in zip(ops.MIXER_KEYS, ws)])


class PGFMambaStdBlock(nn.Module):
    """x -> RMSNorm -> Mamba mixer -> +x -> RMSNorm -> FFN -> +x with the PGF API of PGFMambaBlock."""

    def __init__(self, d_model: int, d_state: int = 16, d_ff: Optional[int] = None, block_size: int = 128,
                 expand: int = 2, d_conv: int = 4, dt_rank: Optional[int] = None, ffn_activation: str = "gelu"):
        super().__init__()
        self.d_model = d_model
        self.d_ff = d_ff or 4 * d_model
        self.block_size = block_size
        self.ffn_activation = ffn_activation
        self.norm1 = RMSNorm(d_model)
        self.mixer = MambaMixer(d_model, d_state, expand, d_conv, dt_rank)
        self.norm2 = RMSNorm(d_model)
        self.W1 = nn.Parameter(torch.empty(self.d_ff, d_model))
        self.b1 = nn.Parameter(torch.zeros(self.d_ff))
        self.W2 = nn.Parameter(torch.empty(d_model, self.d_ff))
        self.b2 = nn.Parameter(torch.zeros(d_model))
        nn.init.xavier_uniform_(self.W1)
        nn.init.xavier_uniform_(self.W2)

    def forward(self, x):
        x1 = self.mixer(self.norm1(x)) + x
        B, L, D = x.shape
        f = FFNFunction.apply(self.norm2(x1).reshape(-1, D), self.W1, self.b1, self.W2, self.b2, self.ffn_activation)
        return f.reshape(B, L, D) + x1

    @torch.no_grad()
    def pgf_forward(self, x: torch.Tensor, return_ssm_states: bool = False, keep_scan: bool = False):
        """With return_ssm_states, also the scan's boundary states for pgf_backward; with keep_scan as
        well, the mixer's saved buffer and mixer + x instead (the backward then runs no mixer forward)."""
        B, L, D = x.shape
        st = None
        if return_ssm_states and keep_scan:
            m, saved = ops.mamba_mixer_fwd_save(self.norm1.pgf_forward(x), self.mixer.params())
            st = {"saved": saved}
        elif return_ssm_states:
            m, st = ops.mamba_mixer_fwd(self.norm1.pgf_forward(x), self.mixer.params(), want_states=True)
        else:
            m = ops.mamba_mixer_fwd(self.norm1.pgf_forward(x), self.mixer.params())
        # x1 = mixer + x and norm2(x1) in one pass (same bits as the separate add and norm)
        x1, xn2 = ops.rmsnorm_fwd_res(m, x, self.norm2.weight, self.norm2.eps)
        if isinstance(st, dict):
            st["m_out"] = x1
        out = ops.ffn_fwd(xn2.reshape(-1, D), self.W1, self.b1, self.W2, self.b2, self.ffn_activation,
                          residual=x1.reshape(-1, D)).reshape(B, L, D)  # ffn(norm2(x1)) + x1
        return (out, st) if return_ssm_states else out

    @torch.no_grad()
    def pgf_backward(self, x: torch.Tensor, g_out: torch.Tensor, fp32_accum: bool = True,
                     ssm_states: Optional[torch.Tensor] = None) -> Dict[str, Any]:
        B, L, D = x.shape
        g_out = g_out.to(x.dtype)
        p = self.mixer.params()
        xn1 = self.norm1.pgf_forward(x)
        if isinstance(ssm_states, dict):  # from pgf_forward(keep_scan=True)
            saved, m_out = ssm_states["saved"], ssm_states["m_out"]
            xn2 = ops.rmsnorm_fwd(m_out, self.norm2.weight, self.norm2.eps)
        else:
            m_raw, saved = ops.mamba_mixer_fwd_save(xn1, p, states=ssm_states)
            m_out, xn2 = ops.rmsnorm_fwd_res(m_raw, x, self.norm2.weight, self.norm2.eps)
            del m_raw
        fr = pgf_ffn_grad(xn2.reshape(-1, D), g_out.reshape(-1, D), self.W1, self.b1, self.W2, self.b2,
                          activation=self.ffn_activation, compute_input_grads=True)
        gw2, g_m = ops.rmsnorm_bwd(m_out, fr["grad_x"].reshape(B, L, D), self.norm2.weight, self.norm2.eps,
                                   g_add=g_out)  # norm2's grad_x + g_out in one pass
        mg, gxn1 = ops.mamba_mixer_bwd(xn1, g_m, p, saved=saved)
        del saved
        gw1, grad_input = ops.rmsnorm_bwd(x, gxn1, self.norm1.weight, self.norm1.eps, g_add=g_m)
        grads = {"W1": fr["grad_W1"], "b1": fr["grad_b1"], "W2": fr["grad_W2"], "b2": fr["grad_b2"],
                 "norm1.weight": gw1, "norm2.weight": gw2}
        grads.update(self.mixer.grads_to_named(mg, "mixer."))
        return {"grads": grads, "grad_input": grad_input}


__all__ = ["MambaMixer", "PGFMambaStdBlock"]
