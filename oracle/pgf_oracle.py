"""CPU oracle for the PGF block-wise recompute-and-backpropagate training step.

TEST INFRASTRUCTURE ONLY.  This module is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline / reference arm of ``bench.py``
may import it.  The product path (``icml_b200``) never calls it and fails loudly
when its CUDA library is missing.

It restates, in plain PyTorch on the CPU, the algorithm of the reference
implementation (zhry915/icml, a flat directory of Python files).  Every function
cites the reference ``file:line`` it follows.  Two deliberate deviations, both
switchable:

* ``pgf_ffn._process_single_block_grad`` in the reference returns
  ``grad_W1_contrib`` without ever computing it (pgf_ffn.py:101-117, a NameError
  as shipped).  The oracle computes ``grad_W1 = grad_z^T @ x`` as the comment at
  pgf_ffn.py:103 describes.
* The reference's PGF gradient of ``mamba.scale`` is a scalar
  ``(g_out * y_raw).sum()`` (train_singlemamba_optimized.py:400) broadcast into a
  ``(d_model,)`` parameter.  ``scale_grad="autograd"`` (default) returns the
  per-channel sum ``(g_out * y_raw).sum((0, 1))``, which is what autograd of the
  reference forward (``forward_standard``, :731-765) gives;
  ``scale_grad="reference"`` reproduces the reference's scalar broadcast.

All functions take an explicit ``dtype``-agnostic tensor input: run them on
float64 tensors to get a high-precision truth, or on float32 tensors to mimic
the reference bit-for-bit in operation order.

Parity pin: ``tests/golden/*.pt`` hold outputs of the reference itself (imported
read-only in the development container by ``tests/golden/make_golden.py``);
``tests/test_oracle_golden.py`` checks this restatement against them.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

Tensor = torch.Tensor

# --------------------------------------------------------------------------
# L1 math primitives  (train_singlemamba_optimized.py:13-84)
# --------------------------------------------------------------------------


def phi_1(z: Tensor) -> Tensor:
    """phi_1(z) = expm1(z)/z, 1 where |z| < 1e-12.  train_singlemamba_optimized.py:13-19."""
    eps = 1e-12
    mask = z.abs() < eps
    z_safe = torch.where(mask, torch.full_like(z, eps), z)
    res = torch.expm1(z_safe) / z_safe
    return torch.where(mask, torch.ones_like(res), res)


def phi_1_prime(z: Tensor) -> Tensor:
    """phi_1'(z) = ((z-1)e^z+1)/z^2, 1/2 where |z| < 1e-9.  train_singlemamba_optimized.py:21-27."""
    eps = 1e-9
    mask = z.abs() < eps
    z_safe = torch.where(mask, torch.full_like(z, eps), z)
    res = ((z_safe - 1) * torch.exp(z_safe) + 1) / (z_safe ** 2)
    return torch.where(mask, torch.full_like(res, 0.5), res)


def scan_linear(a: Tensor, b: Tensor, h0: Tensor) -> Tensor:
    """h_t = a_t*h_{t-1} + b_t over dim 0, returns the whole trajectory.
    train_singlemamba_optimized.py:41-52 (_scan_linear_recursive)."""
    out = torch.empty_like(a)
    h = h0
    for t in range(a.shape[0]):
        h = a[t] * h + b[t]
        out[t] = h
    return out


def scan_linear_reverse(a_fwd: Tensor, b_fwd: Tensor, h_next: Tensor) -> Tensor:
    """z_t = a_t*z_{t+1} + b_t, t = L-1..0.  train_singlemamba_optimized.py:75-84."""
    L = a_fwd.shape[0]
    out = torch.empty_like(a_fwd)
    z = h_next
    for i in range(L):
        t = L - 1 - i
        z = a_fwd[t] * z + b_fwd[t]
        out[t] = z
    return out


# --------------------------------------------------------------------------
# SSM core  (SingleLayerMambaPGF, train_singlemamba_optimized.py:88-765)
# Parameter dict keys: A_log (N,), D (d,), scale (d,), dt_w (d,d), dt_b (d,),
#                      B_w (N,d), B_b (N,), C_w (N,d), C_b (N,)
# --------------------------------------------------------------------------

SSM_KEYS = ("A_log", "D", "scale", "dt_w", "dt_b", "B_w", "B_b", "C_w", "C_b")


def ssm_init(d_model: int, d_state: int = 16, generator: Optional[torch.Generator] = None,
             dtype=torch.float32) -> Dict[str, Tensor]:
    """Parameters initialised as SingleLayerMambaPGF.__init__ (train_singlemamba_optimized.py:89-101):
    A_log = log(0.1*[1..N]), D = 1, scale = 1, nn.Linear default (kaiming-uniform, bound 1/sqrt(fan_in))."""
    bound = 1.0 / math.sqrt(d_model)

    def lin(o, i):
        w = (torch.rand(o, i, generator=generator) * 2 - 1) * bound
        b = (torch.rand(o, generator=generator) * 2 - 1) * bound
        return w.to(dtype), b.to(dtype)

    dt_w, dt_b = lin(d_model, d_model)
    B_w, B_b = lin(d_state, d_model)
    C_w, C_b = lin(d_state, d_model)
    return {
        "A_log": torch.log(torch.arange(1, d_state + 1, dtype=torch.float32) * 0.1).to(dtype),
        "D": torch.ones(d_model, dtype=dtype),
        "scale": torch.ones(d_model, dtype=dtype),
        "dt_w": dt_w, "dt_b": dt_b, "B_w": B_w, "B_b": B_b, "C_w": C_w, "C_b": C_b,
    }


def ssm_project(p: Dict[str, Tensor], u: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
    """[dt_in | B | C] = u @ [W_dt; W_B; W_C]^T + b.  train_singlemamba_optimized.py:116-124."""
    d = p["D"].shape[0]
    N = p["A_log"].shape[0]
    W = torch.cat([p["dt_w"], p["B_w"], p["C_w"]], dim=0)
    b = torch.cat([p["dt_b"], p["B_b"], p["C_b"]], dim=0)
    out = F.linear(u, W, b)
    return out[..., :d], out[..., d:d + N], out[..., d + N:]


def _discretise(p, u_block, dt_input, B_vec):
    """dt = softplus(dt_in); dtA = dt*A; dA = exp(dtA); b = phi_1(dtA)*B*u, time-major (L,B,d,N).
    pgf_mamba_block.py:92-101 / train_singlemamba_optimized.py:379-383."""
    N = p["A_log"].shape[0]
    A = -torch.exp(p["A_log"])
    dt = F.softplus(dt_input.transpose(0, 1))
    dtA = dt.unsqueeze(-1) * A.view(1, 1, 1, N)
    dA = torch.exp(dtA)
    dB = phi_1(dtA) * B_vec.transpose(0, 1).unsqueeze(2)
    b = dB * u_block.transpose(0, 1).unsqueeze(-1)
    return dt, dtA, dA, b


def ssm_forward(p: Dict[str, Tensor], u: Tensor, block_size: int,
                h0: Optional[Tensor] = None, act: Optional[str] = None) -> Tuple[Tensor, List[Tensor], Tensor]:
    """Block-streamed SSM forward with boundary-state hand-off.
    pgf_mamba_block.py:80-112 (PGFMambaBlock.pgf_forward, Mamba part) and :157-175 (boundary states).
    Returns (y (B,L,d), [h0 of every block], h at the end)."""
    Bsz, L, d = u.shape
    N = p["A_log"].shape[0]
    h = torch.zeros(Bsz, d, N, dtype=u.dtype) if h0 is None else h0
    ys, h0s = [], []
    for start in range(0, L, block_size):
        end = min(start + block_size, L)
        h0s.append(h.clone())
        ub = u[:, start:end]
        dt_in, Bv, Cv = ssm_project(p, ub)
        _, _, dA, b = _discretise(p, ub, dt_in, Bv)
        traj = scan_linear(dA, b, h)
        h = traj[-1].clone()
        hc = (Cv.transpose(0, 1).unsqueeze(2) * traj).sum(-1)
        hc = _act(act, hc)
        y_raw = hc + p["D"] * ub.transpose(0, 1)
        ys.append((y_raw * p["scale"]).transpose(0, 1))
    return torch.cat(ys, dim=1), h0s, h


def _act(act, x):
    if act is None:
        return x
    if act == "relu":
        return F.relu(x)
    if act == "tanh":
        return torch.tanh(x)
    raise ValueError(act)


def _act_prime(act, x):
    """train_singlemamba_optimized.py:103-114."""
    if act is None:
        return torch.ones_like(x)
    if act == "relu":
        return (x > 0).to(x.dtype)
    if act == "tanh":
        return 1.0 - torch.tanh(x) ** 2
    raise ValueError(act)


def _act_double_prime(act, x):
    """train_singlemamba_optimized.py:103-114."""
    if act == "tanh":
        t = torch.tanh(x)
        return -2.0 * t * (1.0 - t * t)
    return torch.zeros_like(x)


def ssm_state_hvp(p: Dict[str, Tensor], u: Tensor, target: Tensor, v_h: Tensor,
                  act: Optional[str] = None) -> Tensor:
    """State HVP trajectory (L, B, d, N) of SingleLayerMambaPGF.compute_state_hvp
    (train_singlemamba_optimized.py:563-685 with _pass2_block's HVP branch :249-275), over the
    whole sequence instead of blocks (the block hand-offs are the same recurrences):
      xi_t = dA_t xi_{t-1}, xi_{-1} = v_h;
      S_t = hf_t (C_t . xi_t) C_t,  hf = l'' (no activation) or l'' act'(C.h)^2 + grad_y act''(C.h),
      l'' = 2 scale_const, grad_y = scale_const (y_pred - target), scale_const = 2 / (L d B);
      zeta_t = dA_{t+1} zeta_{t+1} + S_t with dA_L = 1, zeta_L = 0 (the output).
    h is the forward trajectory from a zero state (:580-596)."""
    Bsz, L, d = u.shape
    dt_in, Bv, Cv = ssm_project(p, u)
    _, _, dA, b = _discretise(p, u, dt_in, Bv)                     # (L, B, d, N)
    Ct = Cv.transpose(0, 1)                                          # (L, B, N)
    scale_const = 2.0 / (L * d * Bsz)
    l2 = 2.0 * scale_const
    if act is None:
        hf = torch.full((L, Bsz, d), l2, dtype=u.dtype)
    else:
        traj = scan_linear(dA, b, torch.zeros(Bsz, d, dA.shape[-1], dtype=u.dtype))
        hc = (Ct.unsqueeze(2) * traj).sum(-1)                        # (L, B, d)
        y_pred = (_act(act, hc) + p["D"] * u.transpose(0, 1)) * p["scale"]
        grad_y = scale_const * (y_pred - target.transpose(0, 1))
        hf = l2 * _act_prime(act, hc) ** 2 + grad_y * _act_double_prime(act, hc)
    xi = scan_linear(dA, torch.zeros_like(dA), v_h)
    S = (hf * (Ct.unsqueeze(2) * xi).sum(-1)).unsqueeze(-1) * Ct.unsqueeze(2)
    a_fwd = torch.cat([dA[1:], torch.ones_like(dA[:1])], 0)
    return scan_linear_reverse(a_fwd, S, torch.zeros_like(v_h))


def ssm_block_grad(p: Dict[str, Tensor], u_block: Tensor, g_block: Tensor, h0: Tensor,
                   delta_h_next: Tensor, dA_next: Tensor, act: Optional[str] = None) -> Dict[str, Tensor]:
    """One block of the PGF backward: recompute from h0, reverse adjoint scan, all grads.
    train_singlemamba_optimized.py:350-472 (_pass2_block_direct_grad).

    Returns a dict with A_log, D, scale_ref (the reference's scalar, :400),
    scale (per-channel autograd value), dt_w, dt_b, B_w, B_b, C_w, C_b, delta_h0, dA0, grad_u,
    and the per-token intermediates grad_dt_in, grad_B, grad_C, grad_u_scan."""
    Bsz, L, d = u_block.shape
    N = p["A_log"].shape[0]
    dt_in, Bv, Cv = ssm_project(p, u_block)
    dt_in_t = dt_in.transpose(0, 1)
    B_t = Bv.transpose(0, 1)
    C_t = Cv.transpose(0, 1)
    u_t = u_block.transpose(0, 1)
    g_t = g_block.transpose(0, 1)
    A = -torch.exp(p["A_log"])
    dt = F.softplus(dt_in_t)
    dtA = dt.unsqueeze(-1) * A.view(1, 1, 1, N)
    dA = torch.exp(dtA)
    b = phi_1(dtA) * B_t.unsqueeze(2) * u_t.unsqueeze(-1)
    h_traj = scan_linear(dA, b, h0)

    delta_in_direct = g_t * p["scale"]                        # :391
    h_contrib = (C_t.unsqueeze(2) * h_traj).sum(-1)           # :392
    delta_in_h = delta_in_direct * _act_prime(act, h_contrib)  # :393-398
    y_raw = _act(act, h_contrib) + p["D"] * u_t
    grad_scale_ref = (g_t * y_raw).sum()                       # :400 (scalar, reference)
    grad_scale = (g_t * y_raw).sum(dim=(0, 1))                 # autograd value

    C_contrib = delta_in_h.unsqueeze(-1) * C_t.unsqueeze(2)    # :402
    a_fwd = torch.empty_like(dA)                               # :404-406
    a_fwd[:-1] = dA[1:]
    a_fwd[-1] = dA_next
    delta_h = scan_linear_reverse(a_fwd, C_contrib, delta_h_next)  # :408

    h_prev = torch.empty_like(h_traj)                          # :410-412
    h_prev[0] = h0
    h_prev[1:] = h_traj[:-1]
    B_exp = B_t.unsqueeze(2)
    u_exp = u_t.unsqueeze(-1)
    p1p = phi_1_prime(dtA)
    term_common = p1p * dtA * B_exp * u_exp                    # :416
    J_Alog = dtA * dA * h_prev + term_common                   # :418
    grad_A_log = (delta_h * J_Alog).sum(dim=(0, 1, 2))        # :425
    A_view = A.view(1, 1, 1, N)
    J_dt = A_view * dA * h_prev + p1p * A_view * B_exp * u_exp  # :427-428
    g_dt = (delta_h * J_dt).sum(-1)
    grad_dt_in = g_dt * torch.sigmoid(dt_in_t)                 # :430
    p1 = phi_1(dtA)
    grad_B = (delta_h * (p1 * u_exp)).sum(dim=2)               # :432-433
    grad_C = (delta_in_h.unsqueeze(-1) * h_traj).sum(dim=2)    # :435
    grad_D = (delta_in_direct * u_t).sum(dim=(0, 1))           # :436

    grad_stack = torch.cat([grad_dt_in, grad_B, grad_C], dim=2)  # :439-451
    u_flat = u_t.reshape(-1, d)
    gs_flat = grad_stack.reshape(-1, d + 2 * N)
    gw = (u_flat.t() @ gs_flat).t()
    gb = gs_flat.sum(0)

    grad_u_rec = (delta_h * (p1 * B_exp)).sum(-1)              # :454-455
    grad_u_direct = delta_in_direct * p["D"]                   # :457
    W_cat = torch.cat([p["dt_w"], p["B_w"], p["C_w"]], dim=0)
    grad_u_proj = torch.matmul(grad_stack, W_cat)              # :459-461
    grad_u = (grad_u_direct + grad_u_rec + grad_u_proj).transpose(0, 1)  # :463
    return {
        "A_log": grad_A_log, "D": grad_D, "scale": grad_scale, "scale_ref": grad_scale_ref,
        "dt_w": gw[:d], "dt_b": gb[:d], "B_w": gw[d:d + N], "B_b": gb[d:d + N],
        "C_w": gw[d + N:], "C_b": gb[d + N:],
        "delta_h0": delta_h[0].clone(), "dA0": dA[0].clone(), "grad_u": grad_u,
        "grad_dt_in": grad_dt_in.transpose(0, 1), "grad_B": grad_B.transpose(0, 1),
        "grad_C": grad_C.transpose(0, 1),
        "grad_u_scan": (grad_u_direct + grad_u_rec).transpose(0, 1),
    }


def ssm_backward(p: Dict[str, Tensor], u: Tensor, g: Tensor, block_size: int,
                 act: Optional[str] = None, scale_grad: str = "autograd") -> Tuple[Dict[str, Tensor], Tensor]:
    """Whole-sequence SSM backward: boundary-state recompute, then blocks in reverse carrying
    (delta_h, dA).  pgf_mamba_block.py:157-175 and :206-234.  Returns (param grads, grad_u)."""
    Bsz, L, d = u.shape
    N = p["A_log"].shape[0]
    _, h0s, _ = ssm_forward(p, u, block_size, act=act)
    grads = {k: torch.zeros_like(p[k]) for k in SSM_KEYS}
    grad_u = torch.zeros_like(u)
    dh = torch.zeros(Bsz, d, N, dtype=u.dtype)
    dAn = torch.ones(Bsz, d, N, dtype=u.dtype)
    nblk = len(h0s)
    for i in reversed(range(nblk)):
        s = i * block_size
        e = min(s + block_size, L)
        r = ssm_block_grad(p, u[:, s:e], g[:, s:e], h0s[i], dh, dAn, act=act)
        for k in SSM_KEYS:
            if k == "scale":
                grads[k] += r["scale"] if scale_grad == "autograd" else r["scale_ref"]
            else:
                grads[k] += r[k]
        dh, dAn = r["delta_h0"], r["dA0"]
        grad_u[:, s:e] = r["grad_u"]
    return grads, grad_u


def ssm_forward_standard(p: Dict[str, Tensor], u: Tensor, act: Optional[str] = None) -> Tensor:
    """Autograd twin of the SSM.  train_singlemamba_optimized.py:731-765."""
    y, _, _ = ssm_forward(p, u, u.shape[1], act=act)
    return y


# --------------------------------------------------------------------------
# RMSNorm  (pgf_rmsnorm.py:9-51, 75-117, 157-214)
# --------------------------------------------------------------------------


def rmsnorm_forward(x: Tensor, w: Tensor, eps: float = 1e-6) -> Tensor:
    """y = x / sqrt(mean(x^2)+eps) * w.  pgf_rmsnorm.py:10-18 / 83-87."""
    rms = torch.sqrt(torch.mean(x * x, dim=-1, keepdim=True) + eps)
    return (x / rms) * w


def rmsnorm_grad(x: Tensor, g: Tensor, w: Tensor, eps: float = 1e-6) -> Tuple[Tensor, Tensor]:
    """(grad_weight, grad_x).  pgf_rmsnorm.py:22-51."""
    d = x.shape[-1]
    x2 = x.reshape(-1, d)
    g2 = g.reshape(-1, d)
    rms = torch.sqrt(torch.mean(x2 * x2, dim=-1, keepdim=True) + eps)
    rinv = rms.reciprocal()
    gw = (g2 * (x2 * rinv)).sum(0)
    gwt = g2 * w.unsqueeze(0)
    term1 = gwt * rinv
    dot = (gwt * x2).sum(-1, keepdim=True)
    term2 = (x2 * dot) * (rinv * rinv * rinv) / float(d)
    return gw, (term1 - term2).reshape(x.shape)


# --------------------------------------------------------------------------
# FFN  (pgf_ffn.py:16-117, 183-307)
# --------------------------------------------------------------------------

_GELU_C = 0.7978845608
_GELU_A = 0.044715


def gelu_tanh(x: Tensor) -> Tensor:
    """pgf_ffn.py:16-18."""
    return 0.5 * x * (1.0 + torch.tanh(_GELU_C * (x + _GELU_A * x * x * x)))


def gelu_tanh_prime(x: Tensor) -> Tensor:
    """pgf_ffn.py:21-26."""
    t = torch.tanh(_GELU_C * (x + _GELU_A * x * x * x))
    sech2 = 1.0 - t * t
    return 0.5 * (1.0 + t) + 0.5 * x * sech2 * (_GELU_C * (1.0 + 3.0 * _GELU_A * x * x))


def ffn_forward(x: Tensor, W1: Tensor, b1: Tensor, W2: Tensor, b2: Tensor, activation: str = "gelu") -> Tensor:
    """y = act(x W1^T + b1) W2^T + b2.  pgf_ffn.py:34-55."""
    z = x @ W1.t() + b1
    h = gelu_tanh(z) if activation == "gelu" else torch.relu(z)
    return h @ W2.t() + b2


def ffn_grad(x: Tensor, g: Tensor, W1: Tensor, b1: Tensor, W2: Tensor, b2: Tensor,
             activation: str = "gelu") -> Dict[str, Tensor]:
    """pgf_ffn.py:58-117, with the missing grad_W1 = grad_z^T x (comment at :103)."""
    z = x @ W1.t() + b1
    if activation == "gelu":
        h, hp = gelu_tanh(z), gelu_tanh_prime(z)
    elif activation == "relu":
        h, hp = F.relu(z), (z > 0).to(z.dtype)
    else:
        raise ValueError(activation)
    gW2 = g.t() @ h
    gb2 = g.sum(0)
    gz = (g @ W2) * hp
    gW1 = gz.t() @ x
    gb1 = gz.sum(0)
    gx = gz @ W1
    return {"grad_W1": gW1, "grad_b1": gb1, "grad_W2": gW2, "grad_b2": gb2, "grad_x": gx}


# --------------------------------------------------------------------------
# Embedding / LM head / CE  (pgf_embedding.py, pgf_lm_head.py, test_multi_layer_grads.py:74-86)
# --------------------------------------------------------------------------


def embedding_forward(ids: Tensor, W: Tensor) -> Tensor:
    """pgf_embedding.py:7-11, 74-124."""
    return F.embedding(ids, W)


def embedding_grad(ids: Tensor, g: Tensor, W: Tensor) -> Tensor:
    """Dense (V,d) gradient by index_add_ in token order.  pgf_embedding.py:14-71."""
    gw = torch.zeros_like(W)
    gw.index_add_(0, ids.reshape(-1), g.reshape(-1, g.shape[-1]))
    return gw


def lm_head_forward(h: Tensor, W: Tensor) -> Tensor:
    """logits = h W^T.  pgf_lm_head.py:14-22, 96-130."""
    return h @ W.t()


def lm_head_grad(h: Tensor, g_logits: Tensor, W: Tensor) -> Tuple[Tensor, Tensor]:
    """(grad_W, grad_h).  pgf_lm_head.py:25-93."""
    return g_logits.t() @ h, g_logits @ W


def ce_loss_and_grad(logits: Tensor, targets: Tensor) -> Tuple[Tensor, Tensor]:
    """Mean cross entropy and (softmax - onehot)/T.  test_multi_layer_grads.py:74-86,
    train_wikitext_rebuttal.py:116-125."""
    V = logits.shape[-1]
    lf = logits.reshape(-1, V)
    tf = targets.reshape(-1)
    loss = F.cross_entropy(lf, tf)
    g = F.softmax(lf, dim=-1)
    g[torch.arange(g.shape[0]), tf] -= 1.0
    g /= lf.shape[0]
    return loss, g.reshape(logits.shape)


# --------------------------------------------------------------------------
# Block assembly  (PGFMambaBlock, pgf_mamba_block.py:16-275)
# Block param keys: norm1.weight, norm2.weight, W1, b1, W2, b2, mamba.<SSM_KEYS>
# --------------------------------------------------------------------------


def block_ssm_params(bp: Dict[str, Tensor]) -> Dict[str, Tensor]:
    """Map the block state_dict names (pgf_mamba_block.py:137-153) onto SSM_KEYS."""
    m = {
        "A_log": "mamba.A_log", "D": "mamba.D", "scale": "mamba.scale",
        "dt_w": "mamba.dt_proj.weight", "dt_b": "mamba.dt_proj.bias",
        "B_w": "mamba.B_proj.weight", "B_b": "mamba.B_proj.bias",
        "C_w": "mamba.C_proj.weight", "C_b": "mamba.C_proj.bias",
    }
    return {k: bp[v] for k, v in m.items()}


BLOCK_GRAD_NAMES = ("W1", "b1", "W2", "b2", "mamba.A_log", "mamba.D", "mamba.scale",
                    "mamba.dt_proj.weight", "mamba.dt_proj.bias", "mamba.B_proj.weight",
                    "mamba.B_proj.bias", "mamba.C_proj.weight", "mamba.C_proj.bias",
                    "norm1.weight", "norm2.weight")


def block_pgf_forward(bp: Dict[str, Tensor], x: Tensor, block_size: int, eps: float = 1e-6,
                      ffn_activation: str = "gelu", act: Optional[str] = None) -> Tensor:
    """x -> RMSNorm -> SSM -> +x -> RMSNorm -> FFN -> +x.  pgf_mamba_block.py:70-126."""
    Bsz, L, d = x.shape
    xn = rmsnorm_forward(x, bp["norm1.weight"], eps)
    y, _, _ = ssm_forward(block_ssm_params(bp), xn, block_size, act=act)
    x1 = y + x
    xn2 = rmsnorm_forward(x1, bp["norm2.weight"], eps)
    f = ffn_forward(xn2.reshape(-1, d), bp["W1"], bp["b1"], bp["W2"], bp["b2"], ffn_activation)
    return f.reshape(Bsz, L, d) + x1


def block_pgf_backward(bp: Dict[str, Tensor], x: Tensor, g_out: Tensor, block_size: int,
                       eps: float = 1e-6, ffn_activation: str = "gelu", act: Optional[str] = None,
                       scale_grad: str = "autograd") -> Dict[str, object]:
    """pgf_mamba_block.py:128-249.  Returns {"grads": {15 names}, "grad_input": (B,L,d)}."""
    Bsz, L, d = x.shape
    sp = block_ssm_params(bp)
    xn1 = rmsnorm_forward(x, bp["norm1.weight"], eps)                      # :157
    y, _, _ = ssm_forward(sp, xn1, block_size, act=act)                    # :163-178
    m_out = y + x
    xn2 = rmsnorm_forward(m_out, bp["norm2.weight"], eps)                  # :179
    fr = ffn_grad(xn2.reshape(-1, d), g_out.reshape(-1, d), bp["W1"], bp["b1"], bp["W2"], bp["b2"],
                  ffn_activation)                                          # :183-192
    gn2w, gn2x = rmsnorm_grad(m_out, fr["grad_x"].reshape(Bsz, L, d), bp["norm2.weight"], eps)  # :196-200
    g_m = gn2x + g_out                                                     # :202
    sg, gu = ssm_backward(sp, xn1, g_m, block_size, act=act, scale_grad=scale_grad)  # :206-234
    gn1w, gn1x = rmsnorm_grad(x, gu, bp["norm1.weight"], eps)              # :237-242
    grads = {
        "W1": fr["grad_W1"], "b1": fr["grad_b1"], "W2": fr["grad_W2"], "b2": fr["grad_b2"],
        "mamba.A_log": sg["A_log"], "mamba.D": sg["D"], "mamba.scale": sg["scale"],
        "mamba.dt_proj.weight": sg["dt_w"], "mamba.dt_proj.bias": sg["dt_b"],
        "mamba.B_proj.weight": sg["B_w"], "mamba.B_proj.bias": sg["B_b"],
        "mamba.C_proj.weight": sg["C_w"], "mamba.C_proj.bias": sg["C_b"],
        "norm1.weight": gn1w, "norm2.weight": gn2w,
    }
    return {"grads": grads, "grad_input": gn1x + g_m}                      # :246-249


def block_init(d_model: int, d_state: int = 16, d_ff: Optional[int] = None,
               generator: Optional[torch.Generator] = None, dtype=torch.float32) -> Dict[str, Tensor]:
    """PGFMambaBlock.__init__ (pgf_mamba_block.py:21-49): RMSNorm weights 1, SSM as ssm_init,
    W1/W2 xavier-uniform, b1/b2 zero."""
    d_ff = d_ff or 4 * d_model
    sp = ssm_init(d_model, d_state, generator, dtype)
    a1 = math.sqrt(6.0 / (d_model + d_ff))
    W1 = ((torch.rand(d_ff, d_model, generator=generator) * 2 - 1) * a1).to(dtype)
    W2 = ((torch.rand(d_model, d_ff, generator=generator) * 2 - 1) * a1).to(dtype)
    bp = {
        "norm1.weight": torch.ones(d_model, dtype=dtype), "norm2.weight": torch.ones(d_model, dtype=dtype),
        "W1": W1, "b1": torch.zeros(d_ff, dtype=dtype), "W2": W2, "b2": torch.zeros(d_model, dtype=dtype),
        "mamba.A_log": sp["A_log"], "mamba.D": sp["D"], "mamba.scale": sp["scale"],
        "mamba.dt_proj.weight": sp["dt_w"], "mamba.dt_proj.bias": sp["dt_b"],
        "mamba.B_proj.weight": sp["B_w"], "mamba.B_proj.bias": sp["B_b"],
        "mamba.C_proj.weight": sp["C_w"], "mamba.C_proj.bias": sp["C_b"],
    }
    return bp


def block_forward_autograd(bp: Dict[str, Tensor], x: Tensor, eps: float = 1e-6,
                           ffn_activation: str = "gelu", act: Optional[str] = None) -> Tensor:
    """Autograd twin.  pgf_mamba_block.py:51-68."""
    return block_pgf_forward(bp, x, x.shape[1], eps, ffn_activation, act)


# --------------------------------------------------------------------------
# LM training step  (train_wikitext_rebuttal.py:98-149, test_multi_layer_grads.py:88-126)
# --------------------------------------------------------------------------


def lm_pgf_step(emb: Tensor, lm_head: Tensor, blocks: List[Dict[str, Tensor]], ids: Tensor,
                targets: Tensor, block_size: int, eps: float = 1e-6,
                scale_grad: str = "autograd") -> Tuple[Tensor, Dict[str, Tensor]]:
    """PGF forward over all layers (stashing layer inputs), CE, LM head grad, layers in reverse,
    embedding grad.  Returns (loss, grads) with names emb, lm_head, layers.<i>.<name>."""
    Bsz, L = ids.shape
    d = emb.shape[1]
    x = embedding_forward(ids, emb)
    inputs = []
    for bp in blocks:
        inputs.append(x.clone())
        x = block_pgf_forward(bp, x, block_size, eps)
    logits = lm_head_forward(x.reshape(-1, d), lm_head)
    loss, g_logits = ce_loss_and_grad(logits, targets.reshape(-1))
    gW, gh = lm_head_grad(x.reshape(-1, d), g_logits, lm_head)
    grads = {"lm_head": gW}
    g = gh.reshape(Bsz, L, d)
    for i in reversed(range(len(blocks))):
        r = block_pgf_backward(blocks[i], inputs[i], g, block_size, eps, scale_grad=scale_grad)
        for k, v in r["grads"].items():
            grads[f"layers.{i}.{k}"] = v
        g = r["grad_input"]
    grads["emb"] = embedding_grad(ids, g, emb)
    return loss, grads


def lm_autograd_step(emb: Tensor, lm_head: Tensor, blocks: List[Dict[str, Tensor]], ids: Tensor,
                     targets: Tensor, eps: float = 1e-6) -> Tuple[Tensor, Dict[str, Tensor]]:
    """Plain autograd over the same model.  train_wikitext_rebuttal.py:79-96."""
    emb = emb.detach().clone().requires_grad_(True)
    lm_head = lm_head.detach().clone().requires_grad_(True)
    bl = [{k: v.detach().clone().requires_grad_(True) for k, v in bp.items()} for bp in blocks]
    x = F.embedding(ids, emb)
    for bp in bl:
        x = block_forward_autograd(bp, x, eps)
    logits = x @ lm_head.t()
    loss = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1))
    loss.backward()
    grads = {"emb": emb.grad, "lm_head": lm_head.grad}
    for i, bp in enumerate(bl):
        for k, v in bp.items():
            grads[f"layers.{i}.{k}"] = v.grad
    return loss.detach(), grads


def zipf_tokens(n: int, vocab: int, s: float = 1.1, generator: Optional[torch.Generator] = None) -> Tensor:
    """Synthetic token ids ~ Zipf(s) over ranks 1..vocab by inverse CDF (seeded)."""
    ranks = torch.arange(1, vocab + 1, dtype=torch.float64)
    pmf = ranks.pow(-s)
    cdf = torch.cumsum(pmf / pmf.sum(), 0)
    u = torch.rand(n, generator=generator, dtype=torch.float64)
    return torch.searchsorted(cdf, u).clamp_(max=vocab - 1)
