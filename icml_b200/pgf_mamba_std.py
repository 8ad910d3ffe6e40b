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

    #: tokens per batch row of one segment (whole PGF blocks); longer sequences run segment by segment
    segment_tokens: int = 65536

    def _segments(self, B: int, L: int):
        bs = max(int(self.block_size), 1, self.mixer.d_conv - 1)
        per_row = max(int(self.segment_tokens) // max(B, 1), bs)
        seg = -(-per_row // bs) * bs
        if L <= seg:
            return [(0, L)]
        return [(a, min(a + seg, L)) for a in range(0, L, seg)]

    def _halo_rows(self, x, a):
        """norm1 of the K-1 rows before token a (the conv context of the segment starting there)."""
        K = self.mixer.d_conv
        if a == 0 or K < 2:
            return None
        return self.norm1.pgf_forward(x[:, a - (K - 1):a].contiguous())

    @torch.no_grad()
    def pgf_forward(self, x: torch.Tensor, return_ssm_states: bool = False, keep_scan: bool = False):
        """With return_ssm_states, also the scan's boundary states for pgf_backward; with keep_scan as
        well, the mixer's saved buffer and mixer + x instead (the backward then runs no mixer forward).
        A sequence longer than one segment runs segment by segment, carrying the scan state and the
        conv's K-1-token context (the states are then a list, one entry per segment)."""
        B, L, D = x.shape
        segs = self._segments(B, L)
        if len(segs) == 1:
            return self._forward_single(x, return_ssm_states, keep_scan)
        p = self.mixer.params()
        out = torch.empty_like(x)
        states, h = [], None
        for a, e in segs:
            xs = x[:, a:e] if B == 1 else x[:, a:e].contiguous()
            xn = self.norm1.pgf_forward(xs)
            m, h, st, saved = ops.mamba_mixer_fwd_seg(xn, p, x_halo=self._halo_rows(x, a), h_init=h, want_h_final=True,
                                                      want_states=return_ssm_states and not keep_scan,
                                                      save=return_ssm_states and keep_scan)
            del xn
            x1, xn2 = ops.rmsnorm_fwd_res(m, xs, self.norm2.weight, self.norm2.eps)
            del m
            o = ops.ffn_fwd(xn2.reshape(-1, D), self.W1, self.b1, self.W2, self.b2, self.ffn_activation,
                            residual=x1.reshape(-1, D), out=out[:, a:e].view(-1, D) if B == 1 else None)
            if B != 1:
                out[:, a:e] = o.view(B, e - a, D)
            states.append({"saved": saved, "m_out": x1} if saved is not None else st)
        return (out, states) if return_ssm_states else out

    def _forward_single(self, x, return_ssm_states, keep_scan):
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
                     ssm_states: Optional[Any] = None) -> Dict[str, Any]:
        B, L, D = x.shape
        segs = self._segments(B, L)
        if isinstance(ssm_states, list) and len(segs) == 1:
            ssm_states = ssm_states[0]
        if len(segs) == 1:
            return self._backward_single(x, g_out, ssm_states)
        g_out = g_out.to(x.dtype)
        p = self.mixer.params()
        n = len(segs)
        hs = [None] * n
        if ssm_states is None:
            # the scan state entering each segment (:157-175 of the reference block, per segment)
            states = [None] * n
            h = None
            for j, (a, e) in enumerate(segs[:-1]):
                xs = x[:, a:e] if B == 1 else x[:, a:e].contiguous()
                _, h, _, _ = ops.mamba_mixer_fwd_seg(self.norm1.pgf_forward(xs), p, x_halo=self._halo_rows(x, a),
                                                     h_init=h, want_h_final=True)
                hs[j + 1] = h
        else:
            states = list(ssm_states)
        grad_input = torch.empty_like(x)
        acc: Dict[str, Any] = {}
        dh = dA = g_tail = None
        K = self.mixer.d_conv
        for j in reversed(range(n)):
            a, e = segs[j]
            xs = x[:, a:e] if B == 1 else x[:, a:e].contiguous()
            gs = g_out[:, a:e] if B == 1 else g_out[:, a:e].contiguous()
            Ls = e - a
            xn1 = self.norm1.pgf_forward(xs)
            halo = self._halo_rows(x, a)
            st = states[j]
            states[j] = None
            if isinstance(st, dict):
                saved, m_out = st["saved"], st["m_out"]
                xn2 = ops.rmsnorm_fwd(m_out, self.norm2.weight, self.norm2.eps)
            else:
                m_raw, _, _, saved = ops.mamba_mixer_fwd_seg(xn1, p, x_halo=halo, h_init=hs[j] if st is None else None,
                                                             states_in=st, save=True)
                m_out, xn2 = ops.rmsnorm_fwd_res(m_raw, xs, self.norm2.weight, self.norm2.eps)
                del m_raw
            fr = ops.ffn_bwd(xn2.reshape(-1, D), gs.reshape(-1, D), self.W1, self.b1, self.W2, self.ffn_activation,
                             need_gx=True, acc=acc.get("ffn"))
            del xn2
            acc["ffn"] = {k: fr[k] for k in ("grad_W1", "grad_b1", "grad_W2", "grad_b2")}
            gw2, g_m = ops.rmsnorm_bwd(m_out, fr["grad_x"].view(B, Ls, D), self.norm2.weight, self.norm2.eps,
                                       g_add=gs, gw_acc=acc.get("norm2"))
            del fr, m_out
            acc["norm2"] = gw2
            mg, gxn1, g_halo, dh, dA = ops.mamba_mixer_bwd_seg(xn1, g_m, p, saved, x_halo=halo, dh_end=dh, dA_end=dA,
                                                                want_carry=j > 0, want_g_halo=j > 0,
                                                                acc=acc.get("mixer"))
            del saved, xn1
            acc["mixer"] = mg
            if g_tail is not None:
                # the next segment's conv read this segment's last K-1 mixer inputs
                gxn1[:, Ls - (K - 1):] += g_tail
            g_tail = g_halo
            gw1, gin = ops.rmsnorm_bwd(xs, gxn1, self.norm1.weight, self.norm1.eps, g_add=g_m,
                                       gw_acc=acc.get("norm1"), out=grad_input[:, a:e] if B == 1 else None)
            acc["norm1"] = gw1
            if B != 1:
                grad_input[:, a:e] = gin
            del gxn1, g_m, gin
        f = acc["ffn"]
        grads = {"W1": f["grad_W1"], "b1": f["grad_b1"], "W2": f["grad_W2"], "b2": f["grad_b2"],
                 "norm1.weight": acc["norm1"], "norm2.weight": acc["norm2"]}
        grads.update(self.mixer.grads_to_named(acc["mixer"], "mixer."))
        return {"grads": grads, "grad_input": grad_input}

    def _backward_single(self, x, g_out, ssm_states):
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
