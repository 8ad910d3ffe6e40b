"""Drop-in for the reference's forward-mode operator module (pgf_mamba.py): the Frechet operator's
PGF forward computes the sequence output and its directional derivative (JVP) on libpgf's
kernels (pgf_frechet_jvp: chunked scan of the (state, tangent) pair; float32).

Same module, class, method and parameter names as the reference, constructed in the same order,
so a seeded construction gives the reference's initial weights.  The reference's two module-level
torch helpers (its phi_1 discretisation and log-shifted cumsum scan, pgf_mamba.py:7-31) are not
provided: nothing outside that file calls them, and here the scan kernels do that work.
``mamba_atomic_step`` (one token) runs the same kernels as ``pgf_forward`` on a one-token sequence.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.nn as nn

from . import ops


class FrechetMambaOperator(nn.Module):
    """pgf_mamba.py:33-166."""

    def __init__(self, d_model: int, d_state: int = 16, init_window: int = 3):
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.init_window = init_window
        A_init = torch.randn(self.d_state) * 0.1 - 1.0
        self.A_log = nn.Parameter(torch.log(-A_init))
        self.dt_proj = nn.Linear(d_model, d_model)
        self.B_proj = nn.Linear(d_model, self.d_state)
        self.C_proj = nn.Linear(d_model, self.d_state)
        self.D = nn.Parameter(torch.ones(d_model))
        self.redshift_scale = nn.Parameter(torch.tensor(2.0))
        self.init_estimator = nn.Linear(d_model * init_window, d_model * d_state)

    def _get_params_dict(self):
        return {"A_log": self.A_log, "dt_w": self.dt_proj.weight, "dt_b": self.dt_proj.bias,
                "B_w": self.B_proj.weight, "B_b": self.B_proj.bias, "C_w": self.C_proj.weight,
                "C_b": self.C_proj.bias, "D_w": self.D, "scale": self.redshift_scale}

    def _cat(self):
        W = torch.cat([self.dt_proj.weight, self.B_proj.weight, self.C_proj.weight], 0).detach()
        b = torch.cat([self.dt_proj.bias, self.B_proj.bias, self.C_proj.bias], 0).detach()
        return W, b

    @torch.no_grad()
    def _initial_pair(self, u_seq: torch.Tensor, du_seq: torch.Tensor):
        """(h0, h0_dot) of pgf_mamba.py:61-66, 79-81: the estimator is affine, so the tangent is W du."""
        L, D = u_seq.shape
        if L < self.init_window:
            return None, None
        W = self.init_estimator.weight
        b = self.init_estimator.bias
        pre = torch.stack([u_seq[:self.init_window].reshape(-1), du_seq[:self.init_window].reshape(-1)])
        out = ops.gemm(pre, W, b_trans=False, out_dtype=torch.float32)  # (2, D*N) = pre W^T
        h0 = (out[0] + b).view(D, self.d_state)
        h0_dot = out[1].view(D, self.d_state)
        return h0, h0_dot

    def estimate_initial_state(self, u_seq: torch.Tensor) -> torch.Tensor:
        L, D = u_seq.shape
        if L < self.init_window:
            return torch.zeros(D, self.d_state, device=u_seq.device)
        return self.init_estimator(u_seq[:self.init_window].flatten()).view(D, self.d_state)

    @torch.no_grad()
    def pgf_forward(self, u_seq: torch.Tensor, du_seq: torch.Tensor, block_size: int = 64, streaming: bool = False,
                    callback: Optional[Callable] = None):
        """pgf_mamba.py:69-139: (y, y_dot) of the whole sequence; with streaming, callback(y_blk,
        dy_blk, start, end) per block of block_size tokens and None returned."""
        u = u_seq.detach().float()
        du = du_seq.detach().float()
        h0, h0_dot = self._initial_pair(u, du)
        W, b = self._cat()
        y, dy = ops.frechet_jvp(u, du, W, b, self.A_log, self.D, self.redshift_scale, h0, h0_dot)
        if streaming:
            if callback is not None:
                L = u.shape[0]
                for s in range(0, L, block_size):
                    e = min(s + block_size, L)
                    callback(y[s:e], dy[s:e], s, e)
            return None
        return y, dy

    @torch.no_grad()
    def forward(self, u_seq: torch.Tensor) -> torch.Tensor:
        """pgf_mamba.py:140-149 (the standard forward): y of the same scan (zero tangent)."""
        y, _ = self.pgf_forward(u_seq, torch.zeros_like(u_seq))
        return y

    @torch.no_grad()
    def mamba_atomic_step(self, u_t, h_prev, params):
        """One token from state h_prev (pgf_mamba.py:151-163): (y_t, h_t), computed as a one-token
        sequence by the scan kernels of pgf_forward (CUDA tensors)."""
        W = torch.cat([params["dt_w"], params["B_w"], params["C_w"]], 0).detach()
        b = torch.cat([params["dt_b"], params["B_b"], params["C_b"]], 0).detach()
        u = u_t.detach().float().reshape(1, -1)
        h0 = h_prev.detach().float()
        y, _, h, _ = ops.frechet_jvp(u, torch.zeros_like(u), W, b, params["A_log"], params["D_w"], params["scale"],
                                     h0, torch.zeros_like(h0), want_state=True)
        return y[0], h


__all__ = ["FrechetMambaOperator"]
