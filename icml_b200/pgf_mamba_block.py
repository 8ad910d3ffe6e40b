"""PGFMambaBlock / PGFMambaSequential with the API of the reference's pgf_mamba_block.py
(:16-322), on libpgf.so.

The reference walks the sequence in blocks of ``block_size`` tokens carrying one (B, d, N) scan
state forward (:86-112) and the adjoint pair (delta_h, dA) backward (:211-234).  Here a block's
forward and backward walk the sequence in segments of whole PGF blocks (``segment_tokens``
tokens per batch row, at least 65536 by default, so that every launch still fills the GPU), carrying
the same states between segments; inside a segment the CUDA scan runs its own chunks.  Every
per-segment buffer (projections, scan checkpoints, FFN tiles, normalised activations) is freed
before the next segment, so the memory a block's backward needs beyond its input, output and
gradient is O(segment), not O(L).  pgf_backward recomputes the forward from the layer input exactly
as the reference does (:155-179) and returns the same gradient dictionary (:137-153) and
``grad_input``.
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

    #: tokens per batch row of one scan segment (rounded up to whole PGF blocks); sequences up to this
    #: length run as one segment
    segment_tokens: int = 65536

    def _segments(self, B: int, L: int):
        """[(start, end)]: the sequence cut into segments of whole PGF blocks, each at least
        segment_tokens / B tokens long (the last one may be shorter)."""
        bs = max(int(self.block_size), 1)
        per_row = max(int(self.segment_tokens) // max(B, 1), bs)
        seg = -(-per_row // bs) * bs
        if L <= seg:
            return [(0, L)]
        return [(a, min(a + seg, L)) for a in range(0, L, seg)]

    def _forward_segment(self, x, h, want_states, keep_scan, out=None):
        """One segment of pgf_forward from scan state h (None = zero): (out, states, end state)."""
        B, L, D = x.shape
        m = self.mamba
        xn = self.norm1.pgf_forward(x, block_size=self.block_size)
        W, b = _cat_weights(m)
        st = None
        if want_states and keep_scan:
            y, saved = ops.ssm_fwd_save(xn, W, b, m.A_log, m.D, m.scale, h_init=h, act=m.output_activation)
            x1, xn2 = ops.rmsnorm_fwd_res(y, x, self.norm2.weight, self.norm2.eps)
            st = {"saved": saved, "m_out": x1}
            h_end = ops.ssm_end_state(saved, B, L, D, self.d_state)
        elif want_states:
            y, st = ops.ssm_fwd_states(xn, W, b, m.A_log, m.D, m.scale, h_init=h, act=m.output_activation)
            h_end = ops.ssm_end_state(st, B, L, D, self.d_state)
        else:
            y, h_end = ops.ssm_fwd(xn, W, b, m.A_log, m.D, m.scale, h_init=h, act=m.output_activation,
                                   want_h_final=True)
        del xn
        if not isinstance(st, dict):
            # x1 = y + x and norm2(x1) in one pass (same bits as the separate add and norm)
            x1, xn2 = ops.rmsnorm_fwd_res(y, x, self.norm2.weight, self.norm2.eps)
        del y
        # ffn(norm2(x1)) + x1 (:120-126), the skip connection added in the FFN's last epilogue
        o = ops.ffn_fwd(xn2.reshape(-1, D), self.W1, self.b1, self.W2, self.b2, self.ffn_activation,
                        residual=x1.reshape(-1, D), out=None if out is None else out.view(-1, D)).view(B, L, D)
        return o, st, h_end

    @torch.no_grad()
    def pgf_forward(self, x: torch.Tensor, return_ssm_states: bool = False, keep_scan: bool = False):
        """pgf_mamba_block.py:70-126.  With return_ssm_states, also the scan's boundary states (for
        pgf_backward(..., ssm_states=...), which then need not recompute them).  With keep_scan as
        well, what is returned instead is everything the backward's recompute of the scan produces
        (the scan's saved states and the residual sum y + x), so the backward runs no scan pass before
        its scan backward.  That holds, per block until its backward, about 8.5 bytes per token and
        channel of scan states (an 8-token checkpoint of the 16 states) and y + x in the activation
        dtype.  A sequence longer than one segment runs segment by segment (the states are then a
        list, one entry per segment)."""
        B, L, D = x.shape
        segs = self._segments(B, L)
        if len(segs) == 1:
            if return_ssm_states:
                out, st, _ = self._forward_segment(x, None, True, keep_scan)
                return out, st
            xn = self.norm1.pgf_forward(x, block_size=self.block_size)
            y, _ = self.mamba.ssm_forward(xn)
            x1, xn2 = ops.rmsnorm_fwd_res(y, x, self.norm2.weight, self.norm2.eps)
            return ops.ffn_fwd(xn2.reshape(-1, D), self.W1, self.b1, self.W2, self.b2, self.ffn_activation,
                               residual=x1.reshape(-1, D)).reshape(B, L, D)
        out = torch.empty_like(x)
        states, h = [], None
        for a, e in segs:
            xs = x[:, a:e] if B == 1 else x[:, a:e].contiguous()
            o, st, h = self._forward_segment(xs, h, return_ssm_states, keep_scan, out=out[:, a:e] if B == 1 else None)
            if B != 1:
                out[:, a:e] = o
            states.append(st)
        return (out, states) if return_ssm_states else out

    @torch.no_grad()
    def pgf_backward(self, x: torch.Tensor, g_out: torch.Tensor, fp32_accum: bool = True,
                     ssm_states: Optional[Any] = None) -> Dict[str, Any]:
        """pgf_mamba_block.py:128-249.  ssm_states: what pgf_forward returned for the same x -- the
        boundary states (the recompute then runs one scan pass instead of rebuilding them, :157-175),
        or, from pgf_forward(keep_scan=True), the scan's saved states and y + x (no scan recompute).
        A sequence longer than one segment runs its segments in reverse, carrying the adjoint and the
        first token's decay between them (:211-234) and adding each segment's parameter gradients
        into the same buffers."""
        B, L, D = x.shape
        segs = self._segments(B, L)
        if isinstance(ssm_states, list) and len(segs) == 1:
            ssm_states = ssm_states[0]
        if len(segs) == 1:
            return self._backward_single(x, g_out, ssm_states)
        g_out = g_out.to(x.dtype)
        m = self.mamba
        W, b = _cat_weights(m)
        act = m.output_activation
        n = len(segs)
        hs = [None] * n
        if ssm_states is None:
            # the scan state entering each segment (:157-175): end state of a summary pass per segment
            states = [None] * n
            h = None
            for j, (a, e) in enumerate(segs[:-1]):
                xs = x[:, a:e] if B == 1 else x[:, a:e].contiguous()
                h, _ = ops.ssm_summary(self.norm1.pgf_forward(xs, block_size=self.block_size), W, b, m.A_log,
                                       h_init=h)
                hs[j + 1] = h
        else:
            states = list(ssm_states)
        grad_input = torch.empty_like(x)
        acc: Dict[str, Any] = {}
        dh = dA = None
        for j in reversed(range(n)):
            a, e = segs[j]
            xs = x[:, a:e] if B == 1 else x[:, a:e].contiguous()
            gs = g_out[:, a:e] if B == 1 else g_out[:, a:e].contiguous()
            Ls = e - a
            xn1 = self.norm1.pgf_forward(xs, block_size=self.block_size)
            st = states[j]
            states[j] = None
            if isinstance(st, dict):
                saved, m_out = st["saved"], st["m_out"]
                xn2 = ops.rmsnorm_fwd(m_out, self.norm2.weight, self.norm2.eps)
            else:
                y, saved = ops.ssm_fwd_save(xn1, W, b, m.A_log, m.D, m.scale, act=act,
                                            h_init=hs[j] if st is None else None, states=st)
                m_out, xn2 = ops.rmsnorm_fwd_res(y, xs, self.norm2.weight, self.norm2.eps)
                del y
            fr = ops.ffn_bwd(xn2.reshape(-1, D), gs.reshape(-1, D), self.W1, self.b1, self.W2, self.ffn_activation,
                             need_gx=True, acc=acc.get("ffn"))
            del xn2
            acc["ffn"] = {k: fr[k] for k in ("grad_W1", "grad_b1", "grad_W2", "grad_b2")}
            gw2, g_m = ops.rmsnorm_bwd(m_out, fr["grad_x"].view(B, Ls, D), self.norm2.weight, self.norm2.eps,
                                       g_add=gs, gw_acc=acc.get("norm2"))
            del fr, m_out
            acc["norm2"] = gw2
            r = ops.ssm_bwd(xn1, g_m, W, b, m.A_log, m.D, m.scale, act=act, saved=saved, dh_end=dh, dA_end=dA,
                            want_carry=j > 0, acc=acc.get("ssm"))
            del saved
            acc["ssm"] = {k: r[k] for k in ("W_cat", "b_cat", "A_log", "D", "scale")}
            dh, dA = r["delta_h0"], r["dA0"]
            gw1, gin = ops.rmsnorm_bwd(xs, r["grad_u"], self.norm1.weight, self.norm1.eps, g_add=g_m,
                                       gw_acc=acc.get("norm1"), out=grad_input[:, a:e] if B == 1 else None)
            acc["norm1"] = gw1
            if B != 1:
                grad_input[:, a:e] = gin
            del r, xn1, g_m, gin
        f, sg = acc["ffn"], acc["ssm"]
        return {"grads": self._grad_dict(f["grad_W1"], f["grad_b1"], f["grad_W2"], f["grad_b2"], sg,
                                         acc["norm1"], acc["norm2"]),
                "grad_input": grad_input}

    def _grad_dict(self, gW1, gb1, gW2, gb2, r, gw1, gw2):
        d, N = self.d_model, self.d_state
        gscale = r["scale"].sum().expand(d).clone() if self.mamba.reference_scale_grad else r["scale"]
        return {
            "W1": gW1, "b1": gb1, "W2": gW2, "b2": gb2,
            "mamba.A_log": r["A_log"], "mamba.D": r["D"], "mamba.scale": gscale,
            "mamba.dt_proj.weight": r["W_cat"][:d], "mamba.dt_proj.bias": r["b_cat"][:d],
            "mamba.B_proj.weight": r["W_cat"][d:d + N], "mamba.B_proj.bias": r["b_cat"][d:d + N],
            "mamba.C_proj.weight": r["W_cat"][d + N:], "mamba.C_proj.bias": r["b_cat"][d + N:],
            "norm1.weight": gw1, "norm2.weight": gw2,
        }

    def _backward_single(self, x, g_out, ssm_states):
        """pgf_backward over one segment (the whole sequence)."""
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
        return {"grads": self._grad_dict(fr["grad_W1"], fr["grad_b1"], fr["grad_W2"], fr["grad_b2"], r, gw1, gw2),
                "grad_input": grad_input}

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
