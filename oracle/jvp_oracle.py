"""CPU oracle for the forward-mode (JVP) PGF operators.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU arms of
``bench.py`` may import this module; the product path never calls it.

Restates, in plain PyTorch, the reference's forward-mode operators:
* ``RMSNorm.pgf_jvp`` / ``_rmsnorm_jvp_jit`` (pgf_rmsnorm.py:54-72, 119-155);
* ``pgf_ffn_jvp`` / ``_ffn_block_jvp_jit`` (pgf_ffn.py:120-180);
* ``FrechetMambaOperator.pgf_forward`` (pgf_mamba.py:69-139): the block-wise JVP of a selective
  scan with a learned initial state and a softplus output, carried across blocks as a
  (primal, tangent) state pair.

The reference differentiates with ``torch.func.jvp``; the restatement writes the tangent
recurrence out by hand (the derivative of every step of pgf_mamba.py:89-110 with the parameters
held fixed), so a float64 run is a truth independent of autograd.  Parity pin:
``tests/golden/jvp.pt`` (outputs of the reference itself, made by ``tests/golden/make_golden.py``),
checked in ``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F

from .pgf_oracle import gelu_tanh, gelu_tanh_prime

Tensor = torch.Tensor


def rmsnorm_jvp(x: Tensor, x_dot: Tensor, w: Tensor, w_dot: Tensor, eps: float = 1e-6) -> Tuple[Tensor, Tensor]:
    """(y, y_dot) of y = x / rms(x) * w along (x_dot, w_dot).  pgf_rmsnorm.py:54-72."""
    rms = torch.sqrt(torch.mean(x * x, dim=-1, keepdim=True) + eps)
    rms_dot = torch.mean(x * x_dot, dim=-1, keepdim=True) / rms
    y = (x / rms) * w
    y_dot = ((x_dot * rms - x * rms_dot) / (rms * rms)) * w + (x / rms) * w_dot
    return y, y_dot


def ffn_jvp(x: Tensor, x_dot: Tensor, W1: Tensor, W1_dot: Tensor, b1: Tensor, b1_dot: Tensor, W2: Tensor,
            W2_dot: Tensor, b2: Tensor, b2_dot: Tensor, activation: str = "gelu") -> Tuple[Tensor, Tensor]:
    """(y, y_dot) of y = act(x W1^T + b1) W2^T + b2 along every input's tangent.  pgf_ffn.py:120-142."""
    z1 = x @ W1.t() + b1
    z1_dot = x_dot @ W1.t() + x @ W1_dot.t() + b1_dot
    if activation == "gelu":
        h, h_dot = gelu_tanh(z1), gelu_tanh_prime(z1) * z1_dot
    else:
        h, h_dot = torch.relu(z1), (z1 > 0).to(z1.dtype) * z1_dot
    y = h @ W2.t() + b2
    y_dot = h_dot @ W2.t() + h @ W2_dot.t() + b2_dot
    return y, y_dot


# --------------------------------------------------------------------------
# FrechetMambaOperator  (pgf_mamba.py:33-166)
# --------------------------------------------------------------------------

def frechet_init(d_model: int, d_state: int = 16, init_window: int = 3,
                 generator: Optional[torch.Generator] = None) -> Dict[str, Tensor]:
    """Parameters with the shapes of pgf_mamba.py:38-49 (A_log of A ~ -1 + 0.1 N(0,1); nn.Linear-like
    uniform weights).  Names follow _get_params_dict (:51-59) plus the init estimator."""
    g = generator

    def lin(o, i):
        bound = 1.0 / (i ** 0.5)
        return ((torch.rand(o, i, generator=g) * 2 - 1) * bound, (torch.rand(o, generator=g) * 2 - 1) * bound)

    A_init = torch.randn(d_state, generator=g) * 0.1 - 1.0
    dt_w, dt_b = lin(d_model, d_model)
    B_w, B_b = lin(d_state, d_model)
    C_w, C_b = lin(d_state, d_model)
    ie_w, ie_b = lin(d_model * d_state, d_model * init_window)
    return {"A_log": torch.log(-A_init), "dt_w": dt_w, "dt_b": dt_b, "B_w": B_w, "B_b": B_b, "C_w": C_w,
            "C_b": C_b, "D_w": torch.ones(d_model), "scale": torch.tensor(2.0), "init_w": ie_w, "init_b": ie_b,
            "init_window": torch.tensor(init_window)}


def frechet_initial_state(p: Dict[str, Tensor], u: Tensor, du: Tensor) -> Tuple[Tensor, Tensor]:
    """(h0, h0_dot): init_estimator on the first init_window tokens, zero when L < init_window
    (pgf_mamba.py:61-66, its tangent at :80-81; the estimator is affine, so the tangent is W du)."""
    L, D = u.shape
    w = int(p["init_window"])
    N = p["A_log"].shape[0]
    if L < w:
        z = torch.zeros(D, N, dtype=u.dtype)
        return z, z.clone()
    h0 = (p["init_w"] @ u[:w].flatten() + p["init_b"]).view(D, N)
    h0_dot = (p["init_w"] @ du[:w].flatten()).view(D, N)
    return h0, h0_dot


def frechet_jvp(p: Dict[str, Tensor], u: Tensor, du: Tensor, h0: Optional[Tensor] = None,
                h0_dot: Optional[Tensor] = None) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    """(y, y_dot, h_end, h_end_dot) of the operator's scan along (h0_dot, du), token by token.

    Per token (pgf_mamba.py:89-110): dt = softplus(u W_dt^T + b_dt), B, C = u W^T + b, A = -exp(A_log),
    z = dt A, dA = exp(z), dB = phi_1(z) B, h = dA h + dB u,
    y = softplus(C . h + D u) * max(scale, 0.5).
    Tangents with the parameters fixed: dt' = sigmoid(.) (du W_dt^T), z' = dt' A, dA' = dA z',
    dB' = phi_1'(z) z' B + phi_1(z) B',  h' = dA h' + dA' h_prev + dB' u + dB du,
    y' = sigmoid(y_raw) (C' . h + C . h' + D du) * max(scale, 0.5).
    phi_1(z) = expm1(z)/z here; the reference divides by (z + 1e-9) (:7-12), a relative difference
    below 1.5e-9/|z|.
    """
    L, D = u.shape
    N = p["A_log"].shape[0]
    if h0 is None:
        h0, h0_dot = frechet_initial_state(p, u, du)
    A = -torch.exp(p["A_log"])
    pre = u @ p["dt_w"].t() + p["dt_b"]
    pre_dot = du @ p["dt_w"].t()
    dt, dt_dot = F.softplus(pre), torch.sigmoid(pre) * pre_dot
    Bm, Bm_dot = u @ p["B_w"].t() + p["B_b"], du @ p["B_w"].t()
    Cm, Cm_dot = u @ p["C_w"].t() + p["C_b"], du @ p["C_w"].t()
    s = torch.clamp(p["scale"], min=0.5)
    h, hd = h0.clone(), h0_dot.clone()
    ys, yds = [], []
    for t in range(L):
        z = dt[t].unsqueeze(-1) * A                 # (D, N)
        zd = dt_dot[t].unsqueeze(-1) * A
        e = torch.exp(z)
        p1 = torch.where(z.abs() < 1e-12, torch.ones_like(z), torch.expm1(z) / torch.where(z == 0, torch.ones_like(z), z))
        p1p = torch.where(z.abs() < 1e-6, 0.5 + z / 3.0, (e - p1) / torch.where(z == 0, torch.ones_like(z), z))
        b = p1 * Bm[t] * u[t].unsqueeze(-1)
        bd = (p1p * zd * Bm[t] + p1 * Bm_dot[t]) * u[t].unsqueeze(-1) + p1 * Bm[t] * du[t].unsqueeze(-1)
        hd = e * hd + e * zd * h + bd
        h = e * h + b
        y_raw = h @ Cm[t] + p["D_w"] * u[t]
        y_raw_dot = h @ Cm_dot[t] + hd @ Cm[t] + p["D_w"] * du[t]
        ys.append(F.softplus(y_raw) * s)
        yds.append(torch.sigmoid(y_raw) * y_raw_dot * s)
    return torch.stack(ys), torch.stack(yds), h, hd
