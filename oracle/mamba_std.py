"""CPU oracle of the Mamba-standard variant of the PGF block.  TEST INFRASTRUCTURE ONLY.

The reference (zhry915/icml) has no code for this variant: its SSM (train_singlemamba_optimized.py:
88-124) has no in_proj/out_proj, no convolution, no gate and a shared A.  The 8-layer
d_inner-512 and 24-layer d_model-1024 LM configurations describe the standard Mamba mixer (Gu & Dao, "Mamba:
Linear-Time Sequence Modeling with Selective State Spaces", 2023, Algorithm 2 / Section 3.4):

    xz = x W_in^T                      (2E outputs, no bias); xi, z = xz[:E], xz[E:]
    xc = causal depthwise conv1d(xi)   (kernel K, per-channel weights and bias)
    u  = silu(xc)
    [dt_low | B | C] = u W_x^T          (R + 2N outputs, no bias)
    delta = softplus(dt_low W_dt^T + b_dt)
    h_t = exp(delta_t A) * h_{t-1} + delta_t B_t u_t,   A = -exp(A_log)  (per channel, E x N)
    y_t = C_t . h_t + D u_t;  y = y * silu(z);  out = y W_out^T   (no bias)

restated here from that published description in plain PyTorch.  The reference has no such code,
so the restatement cannot be pinned to it; instead tests/test_oracle_mamba_std.py checks it against
an independent implementation of the same mixer, the pure-PyTorch path of transformers'
MambaMixer (`slow_forward`, transformers 5.5.0): outputs and every gradient agree to float32
rounding (relative 2e-7 to 7e-7) at the single-block configuration.  The block around it is the reference's PGFMambaBlock
(pgf_mamba_block.py:51-68): x -> RMSNorm -> mixer -> +x -> RMSNorm -> FFN -> +x.
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch
import torch.nn.functional as F

from . import pgf_oracle as O

STD_KEYS = ("in_w", "conv_w", "conv_b", "x_w", "dt_w", "dt_b", "A_log", "D", "out_w")


def std_init(d_model: int, d_state: int = 16, expand: int = 2, d_conv: int = 4, dt_rank: Optional[int] = None,
             generator: Optional[torch.Generator] = None, dtype=torch.float64,
             dt_min: float = 1e-3, dt_max: float = 1e-1) -> Dict[str, torch.Tensor]:
    """Standard Mamba initialisation: Linear/conv weights uniform(+-1/sqrt(fan_in)), dt_proj weight
    uniform(+-dt_rank^-1/2), dt_proj bias = softplus^-1 of dt ~ log-uniform[dt_min, dt_max],
    A_log = log(1..N) per channel, D = 1."""
    E = expand * d_model
    R = dt_rank or math.ceil(d_model / 16)
    g = generator

    def U(shape, bound):
        return ((torch.rand(*shape, generator=g, dtype=torch.float64) * 2 - 1) * bound).to(dtype)

    dt = torch.exp(torch.rand(E, generator=g, dtype=torch.float64) * (math.log(dt_max) - math.log(dt_min))
                   + math.log(dt_min)).clamp_(min=1e-4)
    return {
        "in_w": U((2 * E, d_model), 1 / math.sqrt(d_model)),
        "conv_w": U((E, d_conv), 1 / math.sqrt(d_conv)),
        "conv_b": U((E,), 1 / math.sqrt(d_conv)),
        "x_w": U((R + 2 * d_state, E), 1 / math.sqrt(E)),
        "dt_w": U((E, R), R ** -0.5),
        "dt_b": (dt + torch.log(-torch.expm1(-dt))).to(dtype),
        "A_log": torch.log(torch.arange(1, d_state + 1, dtype=torch.float64)).repeat(E, 1).to(dtype),
        "D": torch.ones(E, dtype=dtype),
        "out_w": U((d_model, E), 1 / math.sqrt(E)),
    }


def causal_conv(xi: torch.Tensor, w: torch.Tensor, b: torch.Tensor,
                prefix: Optional[torch.Tensor] = None) -> torch.Tensor:
    """xc[t, e] = b[e] + sum_k w[e, k] xi[t - (K-1) + k, e]; `prefix` (B, K-1, E) are the tokens
    before t = 0 (zeros when absent)."""
    Bsz, L, E = xi.shape
    K = w.shape[1]
    pre = prefix if prefix is not None else xi.new_zeros(Bsz, K - 1, E)
    xp = torch.cat([pre, xi], 1)
    out = b.expand(Bsz, L, E).clone()
    for k in range(K):
        out = out + w[:, k] * xp[:, k:k + L]
    return out


def mixer_forward(p: Dict[str, torch.Tensor], x: torch.Tensor, h0: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The standard Mamba mixer, (B, L, d) -> (B, L, d), sequential scan over time."""
    E = p["D"].shape[0]
    N = p["A_log"].shape[1]
    R = p["dt_w"].shape[1]
    xz = x @ p["in_w"].t()
    xi, z = xz[..., :E], xz[..., E:]
    u = F.silu(causal_conv(xi, p["conv_w"], p["conv_b"]))
    xd = u @ p["x_w"].t()
    dt_low, Bm, Cm = xd[..., :R], xd[..., R:R + N], xd[..., R + N:]
    delta = F.softplus(dt_low @ p["dt_w"].t() + p["dt_b"])
    A = -torch.exp(p["A_log"])
    Bsz, L, _ = x.shape
    h = x.new_zeros(Bsz, E, N) if h0 is None else h0
    ys = []
    for t in range(L):
        dA = torch.exp(delta[:, t, :, None] * A)
        h = dA * h + delta[:, t, :, None] * Bm[:, t, None, :] * u[:, t, :, None]
        ys.append((h * Cm[:, t, None, :]).sum(-1) + p["D"] * u[:, t])
    y = torch.stack(ys, 1) * F.silu(z)
    return y @ p["out_w"].t()


def block_init(d_model: int, d_state: int = 16, d_ff: Optional[int] = None, expand: int = 2, d_conv: int = 4,
               dt_rank: Optional[int] = None, generator=None, dtype=torch.float64) -> Dict[str, torch.Tensor]:
    d_ff = d_ff or 4 * d_model
    a1 = math.sqrt(6.0 / (d_model + d_ff))
    g = generator
    bp = {"norm1.weight": torch.ones(d_model, dtype=dtype), "norm2.weight": torch.ones(d_model, dtype=dtype),
          "W1": ((torch.rand(d_ff, d_model, generator=g, dtype=torch.float64) * 2 - 1) * a1).to(dtype),
          "b1": torch.zeros(d_ff, dtype=dtype),
          "W2": ((torch.rand(d_model, d_ff, generator=g, dtype=torch.float64) * 2 - 1) * a1).to(dtype),
          "b2": torch.zeros(d_model, dtype=dtype)}
    for k, v in std_init(d_model, d_state, expand, d_conv, dt_rank, g, dtype).items():
        bp["mixer." + k] = v
    return bp


def block_forward(bp: Dict[str, torch.Tensor], x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x -> RMSNorm -> mixer -> +x -> RMSNorm -> FFN(GELU-tanh) -> +x (pgf_mamba_block.py:51-68)."""
    p = {k[6:]: v for k, v in bp.items() if k.startswith("mixer.")}
    x1 = mixer_forward(p, O.rmsnorm_forward(x, bp["norm1.weight"], eps)) + x
    Bsz, L, d = x.shape
    f = O.ffn_forward(O.rmsnorm_forward(x1, bp["norm2.weight"], eps).reshape(-1, d), bp["W1"], bp["b1"], bp["W2"],
                      bp["b2"], "gelu")
    return f.reshape(Bsz, L, d) + x1


def block_grads(bp: Dict[str, torch.Tensor], x: torch.Tensor, g: torch.Tensor, eps: float = 1e-6):
    """Autograd of block_forward: (y, {param name: grad}, grad_input)."""
    params = {k: v.detach().clone().requires_grad_(True) for k, v in bp.items()}
    xx = x.detach().clone().requires_grad_(True)
    y = block_forward(params, xx, eps)
    y.backward(g)
    return y.detach(), {k: v.grad for k, v in params.items()}, xx.grad


def lm_grads(emb, lm_head, final_norm, blocks, ids, targets, eps: float = 1e-6):
    """Autograd of the LM: embedding -> blocks -> final RMSNorm -> LM head -> mean CE."""
    emb = emb.detach().clone().requires_grad_(True)
    lm = lm_head.detach().clone().requires_grad_(True) if lm_head is not None else None
    fn = final_norm.detach().clone().requires_grad_(True)
    bl = [{k: v.detach().clone().requires_grad_(True) for k, v in bp.items()} for bp in blocks]
    x = F.embedding(ids, emb)
    for bp in bl:
        x = block_forward(bp, x, eps)
    x = O.rmsnorm_forward(x, fn, eps)
    W = lm if lm is not None else emb
    loss = F.cross_entropy((x @ W.t()).reshape(-1, W.shape[0]), targets.reshape(-1))
    loss.backward()
    grads = {"emb": emb.grad, "final_norm": fn.grad}
    if lm is not None:
        grads["lm_head"] = lm.grad
    for i, bp in enumerate(bl):
        for k, v in bp.items():
            grads[f"layers.{i}.{k}"] = v.grad
    return loss.detach(), grads
