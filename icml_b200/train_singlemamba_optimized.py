"""SingleLayerMambaPGF with the API of the reference's train_singlemamba_optimized.py (:88-765),
computed by the selective-scan kernels of libpgf.so.

Parameters, their names, shapes and initialisation are the reference's (:89-101), so state_dicts
are interchangeable and the same seed gives the same initial weights.  One deliberate
difference: the gradient of ``scale`` is the per-channel ``sum(g * y_raw)`` that autograd of
the reference forward gives; the reference's PGF path returns a scalar instead (:400, :232).
Set ``reference_scale_grad = True`` on the module to reproduce the scalar.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import ops

_ACTS = (None, "relu", "tanh")


def _adjacent(ts):
    """The tensors as one flat view when they lie back to back in one storage (as the flat optimizer
    buffer lays out a layer's projections), else None."""
    t0 = ts[0]
    st = t0.untyped_storage().data_ptr()
    off = t0.storage_offset()
    for t in ts:
        if not t.is_contiguous() or t.untyped_storage().data_ptr() != st or t.storage_offset() != off:
            return None
        off += t.numel()
    n = off - t0.storage_offset()
    return torch.empty(0, dtype=t0.dtype, device=t0.device).set_(t0.untyped_storage(), t0.storage_offset(), (n,))


@torch.no_grad()
def _cat_weights(m):
    """W_cat = [dt_proj.weight; B_proj.weight; C_proj.weight] and b_cat likewise: views of the flat
    parameter buffer when the optimizer keeps them adjacent, else concatenated copies."""
    ws = [m.dt_proj.weight, m.B_proj.weight, m.C_proj.weight]
    bs = [m.dt_proj.bias, m.B_proj.bias, m.C_proj.bias]
    W, b = _adjacent(ws), _adjacent(bs)
    W = W.view(-1, ws[0].shape[1]) if W is not None else torch.cat(ws, dim=0)
    b = b if b is not None else torch.cat(bs, dim=0)
    return W, b


def flat_order(params, module):
    """`params` with each SingleLayerMambaPGF's projection weights, then its projection biases, moved
    next to each other (at the first one's place), so a flat buffer in this order holds W_cat and
    b_cat contiguously."""
    params = list(params)
    for m in module.modules():
        if isinstance(m, SingleLayerMambaPGF):
            group = [m.dt_proj.weight, m.B_proj.weight, m.C_proj.weight, m.dt_proj.bias, m.B_proj.bias,
                     m.C_proj.bias]
            ids = {id(p) for p in group}
            at = min(i for i, p in enumerate(params) if id(p) in ids)
            rest = [p for p in params if id(p) not in ids]
            before = [p for p in params[:at] if id(p) not in ids]
            params = before + group + rest[len(before):]
    return params


class SSMFunction(torch.autograd.Function):
    """Autograd wrapper of the SSM layer: forward_standard's math (:731-765) with the CUDA
    forward and PGF backward."""

    @staticmethod
    def forward(ctx, u, dt_w, dt_b, B_w, B_b, C_w, C_b, A_log, D, scale, act):
        W = torch.cat([dt_w, B_w, C_w], 0)
        b = torch.cat([dt_b, B_b, C_b], 0)
        y, _ = ops.ssm_fwd(u, W, b, A_log, D, scale, act=act)
        ctx.save_for_backward(u, W, b, A_log, D, scale)
        ctx.act = act
        ctx.split = (dt_w.shape[0], B_w.shape[0], C_w.shape[0])
        return y

    @staticmethod
    def backward(ctx, gy):
        u, W, b, A_log, D, scale = ctx.saved_tensors
        r = ops.ssm_bwd(u, gy, W, b, A_log, D, scale, act=ctx.act)
        gw = torch.split(r["W_cat"], ctx.split, 0)
        gb = torch.split(r["b_cat"], ctx.split, 0)
        return (r["grad_u"], gw[0], gb[0], gw[1], gb[1], gw[2], gb[2], r["A_log"], r["D"], r["scale"],
                None)


class SingleLayerMambaPGF(nn.Module):
    def __init__(self, d_model, d_state=16, output_activation=None):
        super().__init__()
        if output_activation not in _ACTS:
            raise ValueError(f"output_activation must be one of {_ACTS}")
        self.d_model = d_model
        self.d_state = d_state
        self.output_activation = output_activation
        self.A_log = nn.Parameter(torch.log(torch.arange(1, d_state + 1).float() * 0.1))
        self.D = nn.Parameter(torch.ones(d_model))
        self.dt_proj = nn.Linear(d_model, d_model)
        self.B_proj = nn.Linear(d_model, d_state)
        self.C_proj = nn.Linear(d_model, d_state)
        self.scale = nn.Parameter(torch.ones(d_model))
        self.reference_scale_grad = False

    # --- (:116-124)
    def _project(self, u):
        W, b = _cat_weights(self)
        shp = u.shape
        out = ops.gemm(u.reshape(-1, shp[-1]), W, bias=b).reshape(*shp[:-1], -1)
        d, N = self.d_model, self.d_state
        return out[..., :d], out[..., d:d + N], out[..., d + N:]

    def ssm_forward(self, u, h0=None, want_h_final=False):
        """Block forward from state h0 (B,d,N): y (B,L,d) and optionally the final state."""
        W, b = _cat_weights(self)
        return ops.ssm_fwd(u, W, b, self.A_log, self.D, self.scale, h_init=h0,
                           act=self.output_activation, want_h_final=want_h_final)

    # --- (:350-472)
    @torch.no_grad()
    def _pass2_block_direct_grad(self, u_block, g_out_block, h0_block, delta_h_next, dA_next,
                                 fp32_accum=True):
        """Returns (A_log, D, scale, dt_w, dt_b, B_w, B_b, C_w, C_b, delta_h[0], dA[0], grad_u)."""
        W, b = _cat_weights(self)
        r = ops.ssm_bwd(u_block, g_out_block, W, b, self.A_log, self.D, self.scale, h_init=h0_block,
                        dh_end=delta_h_next, dA_end=dA_next, act=self.output_activation,
                        want_carry=True)
        d, N = self.d_model, self.d_state
        gw, gb = r["W_cat"], r["b_cat"]
        gscale = r["scale"].sum() if self.reference_scale_grad else r["scale"]
        return (r["A_log"], r["D"], gscale, gw[:d], gb[:d], gw[d:d + N], gb[d:d + N], gw[d + N:],
                gb[d + N:], r["delta_h0"], r["dA0"], r["grad_u"])

    # --- (:474-561)
    def pgf_train_step(self, u, target_y, optimizer, block_size):
        """MSE-target PGF step: loss = mean((y - target)^2); writes .grad and steps."""
        with torch.no_grad():
            y, _ = self.ssm_forward(u)
            diff = (y.float() - target_y.float())
            loss = (diff * diff).mean()
            g = (diff * (2.0 / diff.numel())).to(u.dtype)
            W, b = _cat_weights(self)
            r = ops.ssm_bwd(u, g, W, b, self.A_log, self.D, self.scale, act=self.output_activation)
        optimizer.zero_grad()
        d, N = self.d_model, self.d_state
        self.A_log.grad = r["A_log"]
        self.D.grad = r["D"]
        self.scale.grad = (r["scale"].sum().expand_as(self.scale).clone()
                           if self.reference_scale_grad else r["scale"])
        self.dt_proj.weight.grad, self.dt_proj.bias.grad = r["W_cat"][:d], r["b_cat"][:d]
        self.B_proj.weight.grad, self.B_proj.bias.grad = r["W_cat"][d:d + N], r["b_cat"][d:d + N]
        self.C_proj.weight.grad, self.C_proj.bias.grad = r["W_cat"][d + N:], r["b_cat"][d + N:]
        optimizer.step()
        return loss.item()

    # --- (:563-685)
    @torch.no_grad()
    def compute_state_hvp(self, u, target_y, v_h, block_size):
        """State HVP trajectory (L, B, D, N) of the MSE loss against target_y along v_h (B, D, N) on the
        initial state, for the whole sequence at once (block_size is accepted for signature
        compatibility; the kernels chunk the sequence themselves)."""
        W, b = _cat_weights(self)
        B_, L_, D = u.shape
        v = v_h if v_h is not None else torch.zeros(B_, D, self.d_state, device=u.device)
        return ops.ssm_state_hvp(u, target_y, W, b, self.A_log, self.D, self.scale, v, act=self.output_activation)

    # --- (:731-765)
    def forward_standard(self, u):
        return SSMFunction.apply(u, self.dt_proj.weight, self.dt_proj.bias, self.B_proj.weight,
                                 self.B_proj.bias, self.C_proj.weight, self.C_proj.bias, self.A_log,
                                 self.D, self.scale, self.output_activation)

    def forward(self, u):
        return self.forward_standard(u)


__all__ = ["SingleLayerMambaPGF", "SSMFunction"]
