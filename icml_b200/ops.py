"""Tensor-level wrappers over the C-ABI of libpgf.so.

Every function takes CUDA tensors, allocates outputs and scratch from the torch caching
allocator (so peak-memory accounting stays in ``torch.cuda.max_memory_allocated``), launches on
the current stream and returns new tensors.  Activations are float32 or bfloat16; parameters and
parameter gradients are float32.  Nothing here runs on the CPU: a CPU tensor is an error.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from ._lib import Epilogue, check, lib

F32, BF16 = 0, 1
ACT = {None: 0, "none": 0, "gelu": 1, "relu": 2, "tanh": 3}
EPI = {"none": 0, "gelu": 1, "relu": 2, "dgelu": 3, "drelu": 4}


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise TypeError(f"unsupported activation dtype {t.dtype} (float32 or bfloat16)")


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("icml_b200 operators run on CUDA tensors only (no CPU path)")


def _c(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    return None if t is None else t.contiguous()


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _f32(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    return None if t is None else t.detach().float().contiguous()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


# --------------------------------------------------------------------------- RMSNorm
def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    _cuda(x, w)
    x = _c(x)
    w = _f32(w)
    dim = x.shape[-1]
    rows = x.numel() // dim
    y = torch.empty_like(x)
    check(lib().pgf_rmsnorm_fwd(_p(x), _p(w), _p(y), rows, dim, eps, _dt(x), _stream()), "rmsnorm_fwd")
    return y


def rmsnorm_fwd_res(x: torch.Tensor, res: torch.Tensor, w: torch.Tensor, eps: float):
    """(x + res, RMSNorm(x + res) * w) in one pass; bitwise the separate add and norm."""
    _cuda(x, res, w)
    x, res = _c(x), _c(res.to(x.dtype))
    w = _f32(w)
    dim = x.shape[-1]
    rows = x.numel() // dim
    sm = torch.empty_like(x)
    y = torch.empty_like(x)
    check(lib().pgf_rmsnorm_fwd_res(_p(x), _p(res), _p(w), _p(sm), _p(y), rows, dim, eps, _dt(x), _stream()),
          "rmsnorm_fwd_res")
    return sm, y


def _out_buf(out: Optional[torch.Tensor], shape, dtype, device, name: str) -> torch.Tensor:
    """`out` (contiguous, of this shape and dtype, e.g. a view into a larger buffer) or a new tensor."""
    if out is None:
        return torch.empty(*shape, dtype=dtype, device=device)
    if tuple(out.shape) != tuple(shape) or out.dtype != dtype or not out.is_contiguous() or out.device != device:
        raise ValueError(f"{name}: out must be contiguous {tuple(shape)} {dtype} on {device}")
    return out


def _out_like(out: Optional[torch.Tensor], ref: torch.Tensor, name: str) -> torch.Tensor:
    return _out_buf(out, ref.shape, ref.dtype, ref.device, name)


def _acc_buffer(acc: Optional[torch.Tensor], shape, device, name: str):
    """(buffer, accumulate flag): `acc` (float32, `shape`) to add into, or a new buffer to write."""
    if acc is None:
        return torch.empty(*shape, dtype=torch.float32, device=device), 0
    if tuple(acc.shape) != tuple(shape) or acc.dtype != torch.float32 or not acc.is_contiguous():
        raise ValueError(f"{name}: accumulator must be contiguous float32 {tuple(shape)}")
    return acc, 1


def rmsnorm_bwd(x: torch.Tensor, g: torch.Tensor, w: torch.Tensor, eps: float,
                need_gx: bool = True, g_add: Optional[torch.Tensor] = None,
                gw_acc: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None
                ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """(grad weight, grad x); with g_add, grad x + g_add (fused, bitwise the separate add).  gw_acc:
    add grad weight into this float32 buffer instead (it is returned); out: write grad x there."""
    _cuda(x, g, w)
    x, g = _c(x), _c(g.to(x.dtype))
    w = _f32(w)
    dim = x.shape[-1]
    rows = x.numel() // dim
    gw, accum = _acc_buffer(gw_acc, (dim,), x.device, "rmsnorm_bwd")
    gx = _out_like(out, x, "rmsnorm_bwd") if (need_gx or g_add is not None) else None
    L = lib()
    nb = L.pgf_rmsnorm_bwd_workspace(rows, dim)
    ws = _ws(nb, x.device)
    if g_add is not None:
        ga = _c(g_add.to(x.dtype))
        check(L.pgf_rmsnorm_bwd_add(_p(x), _p(g), _p(w), _p(ga), _p(gx), _p(gw), accum, rows, dim, eps, _dt(x),
                                    _p(ws), ws.numel(), _stream()), "rmsnorm_bwd_add")
    else:
        check(L.pgf_rmsnorm_bwd(_p(x), _p(g), _p(w), _p(gx), _p(gw), accum, rows, dim, eps, _dt(x),
                                _p(ws), ws.numel(), _stream()), "rmsnorm_bwd")
    return gw, gx


# --------------------------------------------------------------------------- embedding
def embedding_fwd(ids: torch.Tensor, W: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    _cuda(ids, W)
    ids = _c(ids.long())
    W = _f32(W)
    V, d = W.shape
    y = torch.empty(*ids.shape, d, dtype=dtype, device=W.device)
    check(lib().pgf_embedding_fwd(_p(ids), _p(W), _p(y), ids.numel(), V, d, _dt(y), _stream()),
          "embedding_fwd")
    return y


def embedding_bwd(ids: torch.Tensor, g: torch.Tensor, vocab: int) -> torch.Tensor:
    _cuda(ids, g)
    ids = _c(ids.long())
    d = g.shape[-1]
    g = _c(g)
    n = ids.numel()
    gw = torch.empty(vocab, d, dtype=torch.float32, device=g.device)
    L = lib()
    ws = _ws(L.pgf_embedding_bwd_workspace(n, vocab, d), g.device)
    check(L.pgf_embedding_bwd(_p(ids), _p(g), _p(gw), 0, n, vocab, d, _dt(g), _p(ws), ws.numel(),
                              _stream()), "embedding_bwd")
    return gw


# --------------------------------------------------------------------------- dense products
def gemm(A: torch.Tensor, B: torch.Tensor, *, a_trans=False, b_trans=False, out_dtype=torch.float32,
         bias=None, epilogue="none", aux=None, aux_out=None, addend=None, alpha=1.0,
         out: Optional[torch.Tensor] = None, accumulate=False, split_k=True) -> torch.Tensor:
    """D = epi(alpha * opA @ opB^T): opA = A (M,K) or A^T when a_trans; opB = B (N,K) or B^T.
    split_k: give the product split-K scratch (used only when the output has few tiles)."""
    _cuda(A, B)
    A, B = _c(A), _c(B)
    M, K = (A.shape[1], A.shape[0]) if a_trans else A.shape
    N, K2 = (B.shape[1], B.shape[0]) if b_trans else B.shape
    assert K == K2, (A.shape, B.shape, a_trans, b_trans)
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=A.device)
    e = Epilogue()
    e.kind = EPI[epilogue]
    e.alpha = alpha
    keep = []  # keeps converted operands alive until the launch
    if bias is not None:
        keep.append(_f32(bias))
        e.bias = keep[-1].data_ptr()
    if aux is not None:
        e.aux, e.aux_dtype, e.ld_aux = aux.data_ptr(), _dt(aux), aux.shape[-1]
    if aux_out is not None:
        e.aux_out, e.aux_out_dtype, e.ld_aux_out = aux_out.data_ptr(), _dt(aux_out), aux_out.shape[-1]
    if addend is not None:
        e.addend, e.addend_dtype, e.ld_addend = addend.data_ptr(), _dt(addend), addend.shape[-1]
    e.accumulate = int(accumulate)
    L = lib()
    nws = L.pgf_gemm_workspace(M, N, K) if split_k else 0
    ws = _ws(nws, A.device) if nws else None
    check(L.pgf_gemm_ex(M, N, K, _p(A), _dt(A), A.shape[1], int(a_trans), _p(B), _dt(B), B.shape[1],
                        int(b_trans), _p(out), _dt(out), out.shape[1], e, _p(ws) if ws is not None else None,
                        ws.numel() if ws is not None else 0, _stream()), "gemm")
    return out


def colsum(X: torch.Tensor) -> torch.Tensor:
    _cuda(X)
    X = _c(X)
    M, N = X.shape
    out = torch.empty(N, dtype=torch.float32, device=X.device)
    L = lib()
    ws = _ws(L.pgf_colsum_workspace(M, N), X.device)
    check(L.pgf_colsum(_p(X), _dt(X), M, N, N, _p(out), 0, _p(ws), ws.numel(), _stream()), "colsum")
    return out


# --------------------------------------------------------------------------- FFN
def ffn_fwd(x, W1, b1, W2, b2, activation="gelu", residual=None, out=None) -> torch.Tensor:
    """FFN(x); with `residual` (rows x d_out, x's dtype), FFN(x) + residual from the same kernel.
    out: write the result there (contiguous rows x d_out in x's dtype)."""
    _cuda(x, W1)
    x = _c(x)
    W1, b1, W2, b2 = _f32(W1), _f32(b1), _f32(W2), _f32(b2)
    rows, d_in = x.shape
    d_h, d_out = W1.shape[0], W2.shape[0]
    y = _out_buf(out, (rows, d_out), x.dtype, x.device, "ffn_fwd")
    L = lib()
    ws = _ws(L.pgf_ffn_workspace(rows, d_in, d_h, d_out, _dt(x), 0), x.device)
    if residual is not None:
        res = _c(residual.to(x.dtype))
        if res.shape != (rows, d_out):
            raise ValueError(f"ffn_fwd: residual shape {tuple(res.shape)} != {(rows, d_out)}")
        check(L.pgf_ffn_fwd_res(_p(x), _p(W1), _p(b1), _p(W2), _p(b2), _p(res), _p(y), rows, d_in, d_h, d_out,
                                ACT[activation], _dt(x), _p(ws), ws.numel(), _stream()), "ffn_fwd_res")
        return y
    check(L.pgf_ffn_fwd(_p(x), _p(W1), _p(b1), _p(W2), _p(b2), _p(y), rows, d_in, d_h, d_out,
                        ACT[activation], _dt(x), _p(ws), ws.numel(), _stream()), "ffn_fwd")
    return y


def ffn_jvp(x, x_dot, W1, W1_dot, b1, b1_dot, W2, W2_dot, b2, b2_dot, activation="gelu"):
    """(y, y_dot) of the FFN along every input's tangent (pgf_ffn.py:120-180)."""
    _cuda(x, x_dot, W1)
    x, x_dot = _c(x), _c(x_dot.to(x.dtype))
    W1, W1_dot, b1, b1_dot = _f32(W1), _f32(W1_dot), _f32(b1), _f32(b1_dot)
    W2, W2_dot, b2, b2_dot = _f32(W2), _f32(W2_dot), _f32(b2), _f32(b2_dot)
    rows, d_in = x.shape
    d_h, d_out = W1.shape[0], W2.shape[0]
    y = torch.empty(rows, d_out, dtype=x.dtype, device=x.device)
    y_dot = torch.empty_like(y)
    L = lib()
    ws = _ws(L.pgf_ffn_jvp_workspace(rows, d_in, d_h, d_out, _dt(x)), x.device)
    check(L.pgf_ffn_jvp(_p(x), _p(x_dot), _p(W1), _p(W1_dot), _p(b1), _p(b1_dot), _p(W2), _p(W2_dot), _p(b2),
                        _p(b2_dot), _p(y), _p(y_dot), rows, d_in, d_h, d_out, ACT[activation], _dt(x), _p(ws),
                        ws.numel(), _stream()), "ffn_jvp")
    return y, y_dot


def rmsnorm_jvp(x, x_dot, w, w_dot, eps: float):
    """(y, y_dot) of RMSNorm along (x_dot, w_dot) (pgf_rmsnorm.py:54-72)."""
    _cuda(x, x_dot, w)
    x, x_dot = _c(x), _c(x_dot.to(x.dtype))
    w, w_dot = _f32(w), _f32(w_dot)
    dim = x.shape[-1]
    rows = x.numel() // dim
    y, y_dot = torch.empty_like(x), torch.empty_like(x)
    check(lib().pgf_rmsnorm_jvp(_p(x), _p(x_dot), _p(w), _p(w_dot), _p(y), _p(y_dot), rows, dim, eps, _dt(x),
                                _stream()), "rmsnorm_jvp")
    return y, y_dot


def frechet_jvp(u, u_dot, W_cat, b_cat, A_log, Dp, scale, h0=None, h0_dot=None, want_state=False):
    """(y, y_dot[, h_end, h_end_dot]) of the Frechet operator's scan over one (L, D) float32
    sequence along (h0_dot, u_dot) (pgf_mamba.py:69-139)."""
    _cuda(u, u_dot, W_cat)
    if u.dtype != torch.float32:
        raise TypeError("frechet_jvp: float32 sequences only")
    u, u_dot = _c(u), _c(u_dot.to(u.dtype))
    W_cat, b_cat, A_log, Dp = _f32(W_cat), _f32(b_cat), _f32(A_log), _f32(Dp)
    scale = _f32(scale.reshape(1))
    L_, D = u.shape
    N = A_log.shape[0]
    y, y_dot = torch.empty_like(u), torch.empty_like(u)
    he = torch.empty(D, N, device=u.device) if want_state else None
    hde = torch.empty(D, N, device=u.device) if want_state else None
    lb = lib()
    ws = _ws(lb.pgf_frechet_jvp_workspace(L_, D, N), u.device)
    check(lb.pgf_frechet_jvp(_p(u), _p(u_dot), _p(W_cat), _p(b_cat), _p(A_log), _p(Dp), _p(scale), _p(_f32(h0)),
                             _p(_f32(h0_dot)), _p(y), _p(y_dot), _p(he), _p(hde), L_, D, N, _p(ws), ws.numel(),
                             _stream()), "frechet_jvp")
    return (y, y_dot, he, hde) if want_state else (y, y_dot)


def ssm_state_hvp(u, target, W_cat, b_cat, A_log, Dp, scale, v_h, act=None):
    """(L, B, D, N) state-HVP trajectory of the MSE loss (train_singlemamba_optimized.py:563-685)."""
    _cuda(u, target, W_cat)
    u, target = _f32(u), _f32(target)
    W_cat, b_cat, A_log, Dp, scale, v_h = (_f32(t) for t in (W_cat, b_cat, A_log, Dp, scale, v_h))
    Bsz, L_, D = u.shape
    N = A_log.shape[0]
    out = torch.empty(L_, Bsz, D, N, device=u.device)
    lb = lib()
    ws = _ws(lb.pgf_ssm_state_hvp_workspace(Bsz, L_, D, N, ACT[act]), u.device)
    check(lb.pgf_ssm_state_hvp(_p(u), _p(target), _p(W_cat), _p(b_cat), _p(A_log), _p(Dp), _p(scale), _p(v_h),
                               _p(out), Bsz, L_, D, N, ACT[act], _p(ws), ws.numel(), _stream()), "ssm_state_hvp")
    return out


def ffn_bwd(x, g, W1, b1, W2, activation="gelu", need_gx=True, acc=None) -> Dict[str, torch.Tensor]:
    """Gradients of the FFN; acc: a dict of float32 grad_W1 / grad_b1 / grad_W2 / grad_b2 buffers to
    add into (those buffers are returned)."""
    _cuda(x, g, W1)
    x, g = _c(x), _c(g.to(x.dtype))
    W1, b1, W2 = _f32(W1), _f32(b1), _f32(W2)
    rows, d_in = x.shape
    d_h, d_out = W1.shape[0], W2.shape[0]
    dev = x.device
    acc = acc or {}
    gW1, accum = _acc_buffer(acc.get("grad_W1"), (d_h, d_in), dev, "ffn_bwd")
    gb1, a1 = _acc_buffer(acc.get("grad_b1"), (d_h,), dev, "ffn_bwd")
    gW2, a2 = _acc_buffer(acc.get("grad_W2"), (d_out, d_h), dev, "ffn_bwd")
    gb2, a3 = _acc_buffer(acc.get("grad_b2"), (d_out,), dev, "ffn_bwd")
    if len({accum, a1, a2, a3}) != 1:
        raise ValueError("ffn_bwd: give all four accumulators or none")
    gx = torch.empty_like(x) if need_gx else None
    L = lib()
    ws = _ws(L.pgf_ffn_workspace(rows, d_in, d_h, d_out, _dt(x), 1), dev)
    check(L.pgf_ffn_bwd(_p(x), _p(g), _p(W1), _p(b1), _p(W2), _p(gW1), _p(gb1), _p(gW2), _p(gb2),
                        _p(gx), accum, rows, d_in, d_h, d_out, ACT[activation], _dt(x), _p(ws),
                        ws.numel(), _stream()), "ffn_bwd")
    r = {"grad_W1": gW1, "grad_b1": gb1, "grad_W2": gW2, "grad_b2": gb2}
    if need_gx:
        r["grad_x"] = gx
    return r


# --------------------------------------------------------------------------- LM head
def lm_head_fwd(h, W) -> torch.Tensor:
    _cuda(h, W)
    h = _c(h)
    W = _f32(W)
    T, d = h.shape
    V = W.shape[0]
    logits = torch.empty(T, V, dtype=torch.float32, device=h.device)
    L = lib()
    ws = _ws(L.pgf_lm_head_workspace(T, V, d, _dt(h)), h.device)
    check(L.pgf_lm_head_fwd(_p(h), _p(W), _p(logits), T, V, d, _dt(h), _p(ws), ws.numel(), _stream()),
          "lm_head_fwd")
    return logits


def lm_head_bwd(h, g_logits, W, need_gh=True):
    _cuda(h, g_logits, W)
    h = _c(h)
    g_logits = _f32(g_logits)
    W = _f32(W)
    T, d = h.shape
    V = W.shape[0]
    gW = torch.empty(V, d, dtype=torch.float32, device=h.device)
    gh = torch.empty_like(h) if need_gh else None
    L = lib()
    ws = _ws(L.pgf_lm_head_workspace(T, V, d, _dt(h)), h.device)
    check(L.pgf_lm_head_bwd(_p(h), _p(g_logits), _p(W), _p(gW), _p(gh), 0, T, V, d, _dt(h), _p(ws),
                            ws.numel(), _stream()), "lm_head_bwd")
    return gW, gh


def lm_head_ce_fwd(h, W, targets):
    """Per-row CE loss and log-sum-exp of logits = h W^T, vocab-tiled (logits never stored)."""
    _cuda(h, W, targets)
    h = _c(h)
    W = _f32(W)
    targets = _c(targets.long())
    T, d = h.shape
    V = W.shape[0]
    loss_rows = torch.empty(T, dtype=torch.float32, device=h.device)
    lse = torch.empty(T, dtype=torch.float32, device=h.device)
    L = lib()
    ws = _ws(L.pgf_lm_head_ce_workspace(T, V, d, _dt(h)), h.device)
    check(L.pgf_lm_head_ce_fwd(_p(h), _p(W), _p(targets), _p(loss_rows), _p(lse), T, V, d, _dt(h),
                               _p(ws), ws.numel(), _stream()), "lm_head_ce_fwd")
    return loss_rows, lse


def lm_head_ce_bwd(h, W, targets, lse, grad_scale: float, need_gh=True):
    _cuda(h, W, targets, lse)
    h = _c(h)
    W = _f32(W)
    targets = _c(targets.long())
    T, d = h.shape
    V = W.shape[0]
    gW = torch.empty(V, d, dtype=torch.float32, device=h.device)
    gh = torch.empty_like(h) if need_gh else None
    L = lib()
    ws = _ws(L.pgf_lm_head_ce_workspace(T, V, d, _dt(h)), h.device)
    lse = _c(lse)
    check(L.pgf_lm_head_ce_bwd(_p(h), _p(W), _p(targets), _p(lse), grad_scale, _p(gW), _p(gh), 0,
                               T, V, d, _dt(h), _p(ws), ws.numel(), _stream()), "lm_head_ce_bwd")
    return gW, gh


# --------------------------------------------------------------------------- selective scan
def ssm_fwd(u, W_cat, b_cat, A_log, Dp, scale, h_init=None, act=None, want_h_final=False):
    """y (Bsz,L,D) in u's dtype, and the state after the last token when asked."""
    _cuda(u, W_cat)
    u = _c(u)
    Bsz, L_, D = u.shape
    N = A_log.shape[0]
    y = torch.empty_like(u)
    hf = torch.empty(Bsz, D, N, dtype=torch.float32, device=u.device) if want_h_final else None
    Lb = lib()
    ws = _ws(Lb.pgf_ssm_workspace(Bsz, L_, D, N, _dt(u), 0), u.device)
    W_cat, b_cat, A_log, Dp, scale, h_init = (_f32(t) for t in (W_cat, b_cat, A_log, Dp, scale, h_init))
    check(Lb.pgf_ssm_fwd(_p(u), _p(W_cat), _p(b_cat), _p(A_log), _p(Dp), _p(scale), _p(h_init),
                         _p(y), _p(hf), Bsz, L_, D, N, ACT[act], _dt(u), _p(ws), ws.numel(),
                         _stream()), "ssm_fwd")
    return y, hf


def ssm_fwd_states(u, W_cat, b_cat, A_log, Dp, scale, h_init=None, act=None):
    """ssm_fwd that also returns the boundary states of every chunk (for ssm_fwd_save(states=...))."""
    _cuda(u, W_cat)
    u = _c(u)
    Bsz, L_, D = u.shape
    N = A_log.shape[0]
    y = torch.empty_like(u)
    Lb = lib()
    states = torch.empty(Lb.pgf_ssm_states_size(Bsz, L_, D, N) // 4, dtype=torch.float32, device=u.device)
    ws = _ws(Lb.pgf_ssm_workspace(Bsz, L_, D, N, _dt(u), 0), u.device)
    W_cat, b_cat, A_log, Dp, scale, h_init = (_f32(t) for t in (W_cat, b_cat, A_log, Dp, scale, h_init))
    check(Lb.pgf_ssm_fwd_states(_p(u), _p(W_cat), _p(b_cat), _p(A_log), _p(Dp), _p(scale), _p(h_init), _p(y),
                                _p(states), Bsz, L_, D, N, ACT[act], _dt(u), _p(ws), ws.numel(), _stream()),
          "ssm_fwd_states")
    return y, states


def ssm_fwd_save(u, W_cat, b_cat, A_log, Dp, scale, h_init=None, act=None, states=None):
    """ssm_fwd that also returns the saved scan states (boundary states + 8-token checkpoints)
    for ssm_bwd(..., saved=...) on the same inputs.  With `states` (from ssm_fwd_states on the
    same inputs) the boundary states are not recomputed: one pass over the sequence."""
    _cuda(u, W_cat)
    u = _c(u)
    Bsz, L_, D = u.shape
    N = A_log.shape[0]
    y = torch.empty_like(u)
    Lb = lib()
    saved = torch.empty(Lb.pgf_ssm_saved_size(Bsz, L_, D, N) // 4, dtype=torch.float32, device=u.device)
    ws = _ws(Lb.pgf_ssm_workspace(Bsz, L_, D, N, _dt(u), 0), u.device)
    W_cat, b_cat, A_log, Dp, scale, h_init = (_f32(t) for t in (W_cat, b_cat, A_log, Dp, scale, h_init))
    if states is not None:
        if h_init is not None:
            raise ValueError("ssm_fwd_save: states already include the initial state")
        check(Lb.pgf_ssm_fwd_save_states(_p(u), _p(W_cat), _p(b_cat), _p(A_log), _p(Dp), _p(scale), _p(states),
                                         _p(y), _p(saved), Bsz, L_, D, N, ACT[act], _dt(u), _p(ws), ws.numel(),
                                         _stream()), "ssm_fwd_save_states")
        return y, saved
    check(Lb.pgf_ssm_fwd_save(_p(u), _p(W_cat), _p(b_cat), _p(A_log), _p(Dp), _p(scale), _p(h_init),
                              _p(y), _p(saved), Bsz, L_, D, N, ACT[act], _dt(u), _p(ws), ws.numel(),
                              _stream()), "ssm_fwd_save")
    return y, saved


def ssm_end_state(states: torch.Tensor, Bsz: int, L_: int, D: int, N: int) -> torch.Tensor:
    """The state after the last token, (Bsz, D, N), from the boundary states that ssm_fwd_states
    returns or the saved buffer of ssm_fwd_save (both begin with the (Bsz, chunks + 1, D, N) chunk
    start states, the last of which is the end state)."""
    n1 = lib().pgf_ssm_states_size(Bsz, L_, D, N) // (4 * Bsz * D * N)
    return states[:Bsz * n1 * D * N].view(Bsz, n1, D, N)[:, n1 - 1]


def ssm_bwd(u, g, W_cat, b_cat, A_log, Dp, scale, h_init=None, dh_end=None, dA_end=None, act=None,
            want_carry=False, saved=None, acc=None):
    """All gradients of the SSM layer over [0, L) plus the carries (delta_h[0], dA[0]).  With
    `saved` (from ssm_fwd_save on the same inputs) the forward passes are not recomputed.  acc: a dict
    of float32 W_cat / b_cat / A_log / D / scale buffers to add the parameter gradients into."""
    _cuda(u, g, W_cat)
    u, g = _c(u), _c(g.to(u.dtype))
    Bsz, L_, D = u.shape
    N = A_log.shape[0]
    dev = u.device
    W_cat, b_cat = _f32(W_cat), _f32(b_cat)
    acc = acc or {}
    gW, accum = _acc_buffer(acc.get("W_cat"), tuple(W_cat.shape), dev, "ssm_bwd")
    gb, a1 = _acc_buffer(acc.get("b_cat"), tuple(b_cat.shape), dev, "ssm_bwd")
    gA, a2 = _acc_buffer(acc.get("A_log"), (N,), dev, "ssm_bwd")
    gD, a3 = _acc_buffer(acc.get("D"), (D,), dev, "ssm_bwd")
    gS, a4 = _acc_buffer(acc.get("scale"), (D,), dev, "ssm_bwd")
    if len({accum, a1, a2, a3, a4}) != 1:
        raise ValueError("ssm_bwd: give all five accumulators or none")
    gu = torch.empty_like(u)
    dh0 = torch.empty(Bsz, D, N, dtype=torch.float32, device=dev) if want_carry else None
    dA0 = torch.empty(Bsz, D, N, dtype=torch.float32, device=dev) if want_carry else None
    Lb = lib()
    ws = _ws(Lb.pgf_ssm_workspace(Bsz, L_, D, N, _dt(u), 1), dev)
    A_log, Dp, scale, h_init, dh_end, dA_end = (_f32(t) for t in (A_log, Dp, scale, h_init, dh_end, dA_end))
    fn = Lb.pgf_ssm_bwd if saved is None else Lb.pgf_ssm_bwd_saved
    check(fn(_p(u), _p(g), _p(W_cat), _p(b_cat), _p(A_log), _p(Dp),
                         _p(scale), _p(h_init if saved is None else saved), _p(dh_end), _p(dA_end),
                         _p(gW), _p(gb), _p(gA), _p(gD), _p(gS), _p(gu), _p(dh0), _p(dA0), accum,
                         Bsz, L_, D, N, ACT[act], _dt(u), _p(ws), ws.numel(), _stream()), "ssm_bwd")
    return {"W_cat": gW, "b_cat": gb, "A_log": gA, "D": gD, "scale": gS, "grad_u": gu,
            "delta_h0": dh0, "dA0": dA0}


def ssm_summary(u, W_cat, b_cat, A_log, h_init=None):
    """(state after the segment from h_init, sum of dt per (batch, channel))."""
    _cuda(u, W_cat)
    u = _c(u)
    Bsz, L_, D = u.shape
    N = A_log.shape[0]
    hf = torch.empty(Bsz, D, N, dtype=torch.float32, device=u.device)
    sdt = torch.empty(Bsz, D, dtype=torch.float32, device=u.device)
    Lb = lib()
    ws = _ws(Lb.pgf_ssm_workspace(Bsz, L_, D, N, _dt(u), 0), u.device)
    W_cat, b_cat, A_log, h_init = (_f32(t) for t in (W_cat, b_cat, A_log, h_init))
    check(Lb.pgf_ssm_summary(_p(u), _p(W_cat), _p(b_cat), _p(A_log), _p(h_init), _p(hf), _p(sdt), Bsz, L_,
                             D, N, _dt(u), _p(ws), ws.numel(), _stream()), "ssm_summary")
    return hf, sdt


def ssm_bwd_summary(u, g, W_cat, b_cat, A_log, scale, h_init=None, act=None):
    """(adjoint at the first token for a zero end carry, first token's decay, sum of dt but the first)."""
    _cuda(u, g, W_cat)
    u, g = _c(u), _c(g.to(u.dtype))
    Bsz, L_, D = u.shape
    N = A_log.shape[0]
    dev = u.device
    dh0 = torch.empty(Bsz, D, N, dtype=torch.float32, device=dev)
    dA0 = torch.empty(Bsz, D, N, dtype=torch.float32, device=dev)
    sdx = torch.empty(Bsz, D, dtype=torch.float32, device=dev)
    Lb = lib()
    ws = _ws(Lb.pgf_ssm_workspace(Bsz, L_, D, N, _dt(u), 1), dev)
    W_cat, b_cat, A_log, scale, h_init = (_f32(t) for t in (W_cat, b_cat, A_log, scale, h_init))
    check(Lb.pgf_ssm_bwd_summary(_p(u), _p(g), _p(W_cat), _p(b_cat), _p(A_log), _p(scale), _p(h_init),
                                 _p(dh0), _p(dA0), _p(sdx), Bsz, L_, D, N, ACT[act], _dt(u), _p(ws),
                                 ws.numel(), _stream()), "ssm_bwd_summary")
    return dh0, dA0, sdx


def ssm_fwd_begin(u, W_cat, b_cat, A_log):
    """Sequence sharding, forward part 1: (h_seg, sum_dt, state) -- this segment's end state and sum
    of dt from a zero start (what the ranks exchange) and the state ssm_fwd_finish continues from."""
    _cuda(u, W_cat)
    u = _c(u)
    Bsz, L_, D = u.shape
    N = A_log.shape[0]
    hseg = torch.empty(Bsz, D, N, dtype=torch.float32, device=u.device)
    sdt = torch.empty(Bsz, D, dtype=torch.float32, device=u.device)
    Lb = lib()
    ws = _ws(Lb.pgf_ssm_workspace(Bsz, L_, D, N, _dt(u), 0), u.device)
    W_cat, b_cat, A_log = (_f32(t) for t in (W_cat, b_cat, A_log))
    check(Lb.pgf_ssm_fwd_begin(_p(u), _p(W_cat), _p(b_cat), _p(A_log), _p(hseg), _p(sdt), Bsz, L_, D, N, _dt(u),
                               _p(ws), ws.numel(), _stream()), "ssm_fwd_begin")
    return hseg, sdt, {"u": u, "W_cat": W_cat, "b_cat": b_cat, "A_log": A_log, "ws": ws}


def ssm_fwd_finish(state, Dp, scale, h_init=None, act=None, want_states=False):
    """Sequence sharding, forward part 2: y from the state entering the segment.  With want_states,
    (y, states): the segment's boundary states for ssm_fwd_save(states=...) in the backward."""
    u = state["u"]
    Bsz, L_, D = u.shape
    N = state["A_log"].shape[0]
    y = torch.empty_like(u)
    Dp, scale, h_init = (_f32(t) for t in (Dp, scale, h_init))
    ws = state["ws"]
    Lb = lib()
    args = (_p(u), _p(state["W_cat"]), _p(state["b_cat"]), _p(state["A_log"]), _p(Dp), _p(scale), _p(h_init), _p(y))
    tail = (Bsz, L_, D, N, ACT[act], _dt(u), _p(ws), ws.numel(), _stream())
    if want_states:
        states = torch.empty(Lb.pgf_ssm_states_size(Bsz, L_, D, N) // 4, dtype=torch.float32, device=u.device)
        check(Lb.pgf_ssm_fwd_finish_states(*args, _p(states), *tail), "ssm_fwd_finish_states")
        return y, states
    check(Lb.pgf_ssm_fwd_finish(*args, None, *tail), "ssm_fwd_finish")
    return y


def ssm_bwd_begin(u, g, W_cat, b_cat, A_log, scale, saved, h_init=None, act=None):
    """Sequence sharding, backward part 1 (after ssm_fwd_save with the segment's h_init): (adjoint at
    the first token for a zero end carry, its decay, sum of dt but the first, state)."""
    _cuda(u, g, W_cat)
    u, g = _c(u), _c(g.to(u.dtype))
    Bsz, L_, D = u.shape
    N = A_log.shape[0]
    dev = u.device
    dh0 = torch.empty(Bsz, D, N, dtype=torch.float32, device=dev)
    dA0 = torch.empty(Bsz, D, N, dtype=torch.float32, device=dev)
    sdx = torch.empty(Bsz, D, dtype=torch.float32, device=dev)
    Lb = lib()
    ws = _ws(Lb.pgf_ssm_workspace(Bsz, L_, D, N, _dt(u), 1), dev)
    W_cat, b_cat, A_log, scale, h_init = (_f32(t) for t in (W_cat, b_cat, A_log, scale, h_init))
    check(Lb.pgf_ssm_bwd_begin(_p(u), _p(g), _p(W_cat), _p(b_cat), _p(A_log), _p(scale), _p(h_init), _p(saved),
                               _p(dh0), _p(dA0), _p(sdx), Bsz, L_, D, N, ACT[act], _dt(u), _p(ws), ws.numel(),
                               _stream()), "ssm_bwd_begin")
    return dh0, dA0, sdx, {"u": u, "g": g, "W_cat": W_cat, "b_cat": b_cat, "A_log": A_log, "scale": scale,
                           "h_init": h_init, "saved": saved, "act": act, "ws": ws}


def ssm_bwd_finish(state, Dp, dh_end=None, dA_end=None):
    """Sequence sharding, backward part 2: every gradient for the carry entering from the right."""
    u, g = state["u"], state["g"]
    Bsz, L_, D = u.shape
    N = state["A_log"].shape[0]
    dev = u.device
    gW = torch.empty_like(state["W_cat"])
    gb = torch.empty_like(state["b_cat"])
    gA = torch.empty(N, dtype=torch.float32, device=dev)
    gD = torch.empty(D, dtype=torch.float32, device=dev)
    gS = torch.empty(D, dtype=torch.float32, device=dev)
    gu = torch.empty_like(u)
    Dp, dh_end, dA_end = (_f32(t) for t in (Dp, dh_end, dA_end))
    ws = state["ws"]
    check(lib().pgf_ssm_bwd_finish(_p(u), _p(g), _p(state["W_cat"]), _p(state["b_cat"]), _p(state["A_log"]),
                                   _p(Dp), _p(state["scale"]), _p(state["h_init"]), _p(state["saved"]),
                                   _p(dh_end), _p(dA_end), _p(gW), _p(gb), _p(gA), _p(gD), _p(gS), _p(gu), None,
                                   None, 0, Bsz, L_, D, N, ACT[state["act"]], _dt(u), _p(ws), ws.numel(),
                                   _stream()), "ssm_bwd_finish")
    return {"W_cat": gW, "b_cat": gb, "A_log": gA, "D": gD, "scale": gS, "grad_u": gu}


def ssm_compose_ranks_fwd(gathered, rank: int, A_log, Bsz: int, D: int, N: int) -> torch.Tensor:
    """State entering segment `rank` of a sharded sequence, from every rank's [h_seg | sum_dt]
    summary gathered as rows of `gathered` (P, stride).  A_log (N,) or, per channel, (D, N)."""
    _cuda(gathered, A_log)
    g, A = _c(gathered.float()), _f32(A_log)
    P, stride = g.shape
    h = torch.empty(Bsz, D, N, dtype=torch.float32, device=g.device)
    check(lib().pgf_ssm_compose_ranks_fwd(_p(g), stride, P, rank, _p(A), int(A.dim() == 2), _p(h), Bsz, D, N,
                                          _stream()), "ssm_compose_ranks_fwd")
    return h


def ssm_compose_ranks_bwd(gathered, rank: int, A_log, Bsz: int, D: int, N: int):
    """(dh_end, dA_end) entering segment `rank` from the right, from every rank's
    [dh_start | dA_start | sum_dt_excl] summary gathered as rows of `gathered` (P, stride)."""
    _cuda(gathered, A_log)
    g, A = _c(gathered.float()), _f32(A_log)
    P, stride = g.shape
    dh = torch.empty(Bsz, D, N, dtype=torch.float32, device=g.device)
    dA = torch.empty(Bsz, D, N, dtype=torch.float32, device=g.device)
    check(lib().pgf_ssm_compose_ranks_bwd(_p(g), stride, P, rank, _p(A), int(A.dim() == 2), _p(dh), _p(dA), Bsz, D,
                                          N, _stream()), "ssm_compose_ranks_bwd")
    return dh, dA


# --------------------------------------------------------------------------- Mamba-standard mixer
MIXER_KEYS = ("in_w", "conv_w", "conv_b", "x_w", "dt_w", "dt_b", "A_log", "D", "out_w")


def _mixer_dims(x, p):
    Bsz, L_, d = x.shape
    E, N = p["A_log"].shape
    R = p["dt_w"].shape[1]
    K = p["conv_w"].shape[1]
    return Bsz, L_, d, E, R, N, K


def mamba_mixer_fwd(x, p, want_states: bool = False):
    """Standard Mamba mixer forward; p: dict of MIXER_KEYS float32 tensors.  want_states: also the
    scan's boundary states, for mamba_mixer_fwd_save(states=...)."""
    _cuda(x, p["in_w"])
    x = _c(x)
    Bsz, L_, d, E, R, N, K = _mixer_dims(x, p)
    q = {k: _f32(p[k]) for k in MIXER_KEYS}
    out = torch.empty_like(x)
    Lb = lib()
    ws = _ws(Lb.pgf_mamba_mixer_workspace(Bsz, L_, d, E, R, N, K, _dt(x), 0), x.device)
    if want_states:
        st = torch.empty(Lb.pgf_mamba_mixer_states_size(Bsz, L_, d, E, R, N, K) // 4, device=x.device)
        check(Lb.pgf_mamba_mixer_fwd_states(_p(x), *[_p(q[k]) for k in MIXER_KEYS], _p(out), _p(st), Bsz, L_, d, E,
                                            R, N, K, _dt(x), _p(ws), ws.numel(), _stream()), "mamba_mixer_fwd_states")
        return out, st
    check(Lb.pgf_mamba_mixer_fwd(_p(x), *[_p(q[k]) for k in MIXER_KEYS], _p(out), Bsz, L_, d, E, R, N, K,
                                 _dt(x), _p(ws), ws.numel(), _stream()), "mamba_mixer_fwd")
    return out


def mamba_mixer_fwd_save(x, p, states: Optional[torch.Tensor] = None):
    """Mixer forward that keeps its intermediates: (out, saved) for mamba_mixer_bwd(saved=...).
    With `states` (from mamba_mixer_fwd(want_states=True) on the same x) the scan's boundary states
    are not rebuilt."""
    _cuda(x, p["in_w"])
    x = _c(x)
    Bsz, L_, d, E, R, N, K = _mixer_dims(x, p)
    q = {k: _f32(p[k]) for k in MIXER_KEYS}
    out = torch.empty_like(x)
    Lb = lib()
    saved = _ws(Lb.pgf_mamba_mixer_saved_size(Bsz, L_, d, E, R, N, K, _dt(x)), x.device)
    ws = _ws(Lb.pgf_mamba_mixer_workspace(Bsz, L_, d, E, R, N, K, _dt(x), 0), x.device)
    if states is not None:
        check(Lb.pgf_mamba_mixer_fwd_save_states(_p(x), *[_p(q[k]) for k in MIXER_KEYS], _p(states), _p(out),
                                                 _p(saved), saved.numel(), Bsz, L_, d, E, R, N, K, _dt(x), _p(ws),
                                                 ws.numel(), _stream()), "mamba_mixer_fwd_save_states")
        return out, saved
    check(Lb.pgf_mamba_mixer_fwd_save(_p(x), *[_p(q[k]) for k in MIXER_KEYS], _p(out), _p(saved), saved.numel(),
                                      Bsz, L_, d, E, R, N, K, _dt(x), _p(ws), ws.numel(), _stream()),
          "mamba_mixer_fwd_save")
    return out, saved


def mamba_mixer_bwd(x, g, p, saved: Optional[torch.Tensor] = None):
    """(grads dict over MIXER_KEYS, grad_x) of the standard Mamba mixer; `saved` from
    mamba_mixer_fwd_save on the same x and weights skips the forward re-run."""
    _cuda(x, g, p["in_w"])
    x, g = _c(x), _c(g.to(x.dtype))
    Bsz, L_, d, E, R, N, K = _mixer_dims(x, p)
    q = {k: _f32(p[k]) for k in MIXER_KEYS}
    grads = {k: torch.empty_like(q[k]) for k in MIXER_KEYS}
    gx = torch.empty_like(x)
    Lb = lib()
    ws = _ws(Lb.pgf_mamba_mixer_workspace(Bsz, L_, d, E, R, N, K, _dt(x), 1), x.device)
    if saved is None:
        check(Lb.pgf_mamba_mixer_bwd(_p(x), _p(g), *[_p(q[k]) for k in MIXER_KEYS],
                                     *[_p(grads[k]) for k in MIXER_KEYS], _p(gx), 0, Bsz, L_, d, E, R, N, K,
                                     _dt(x), _p(ws), ws.numel(), _stream()), "mamba_mixer_bwd")
    else:
        check(Lb.pgf_mamba_mixer_bwd_saved(_p(x), _p(g), *[_p(q[k]) for k in MIXER_KEYS],
                                           *[_p(grads[k]) for k in MIXER_KEYS], _p(gx), 0, _p(saved),
                                           saved.numel(), Bsz, L_, d, E, R, N, K, _dt(x), _p(ws), ws.numel(),
                                           _stream()), "mamba_mixer_bwd_saved")
    return grads, gx


# --------------------------------------------------------------------------- mixer over segments
def _mixer_prep(x, p):
    _cuda(x, p["in_w"])
    x = _c(x)
    dims = _mixer_dims(x, p)
    q = {k: _f32(p[k]) for k in MIXER_KEYS}
    return x, dims, q


def _halo(x_halo, x):
    return None if x_halo is None else _c(x_halo.to(x.dtype))


def mamba_mixer_fwd_seg(x, p, x_halo=None, h_init=None, states_in=None, want_h_final=False, want_states=False,
                        save=False):
    """The mixer over one segment of a longer sequence: x_halo (Bsz, K-1, d) the mixer inputs of the
    K-1 tokens before it (conv context), h_init the scan state entering it, states_in the boundary
    states of an earlier call with want_states on the same input.  Returns (out, h_final, states,
    saved) (None where not asked)."""
    x, (Bsz, L_, d, E, R, N, K), q = _mixer_prep(x, p)
    Lb = lib()
    out = torch.empty_like(x)
    hf = torch.empty(Bsz, E, N, device=x.device) if want_h_final else None
    st = torch.empty(Lb.pgf_mamba_mixer_states_size(Bsz, L_, d, E, R, N, K) // 4, device=x.device) if want_states \
        else None
    saved = _ws(Lb.pgf_mamba_mixer_saved_size(Bsz, L_, d, E, R, N, K, _dt(x)), x.device) if save else None
    ws = _ws(Lb.pgf_mamba_mixer_workspace(Bsz, L_, d, E, R, N, K, _dt(x), 0), x.device)
    check(Lb.pgf_mamba_mixer_fwd_seg(_p(x), *[_p(q[k]) for k in MIXER_KEYS], _p(_halo(x_halo, x)), _p(_f32(h_init)),
                                     _p(states_in), _p(out), _p(hf), _p(st), _p(saved),
                                     saved.numel() if saved is not None else 0, Bsz, L_, d, E, R, N, K, _dt(x), _p(ws),
                                     ws.numel(), _stream()), "mamba_mixer_fwd_seg")
    return out, hf, st, saved


def mamba_mixer_end_state(states, Bsz, L_, d, E, R, N, K):
    """The scan state after the segment, (Bsz, E, N), from the boundary states of mamba_mixer_fwd_seg."""
    n1 = lib().pgf_mamba_mixer_states_size(Bsz, L_, d, E, R, N, K) // (4 * Bsz * E * N)
    return states.view(Bsz, n1, E, N)[:, n1 - 1]


def mamba_mixer_fwd_begin(x, p, x_halo=None):
    """Sequence sharding, forward part 1: (h_seg, sum_dt, state) -- the segment's summary from a zero
    start and the state mamba_mixer_fwd_finish continues from."""
    x, (Bsz, L_, d, E, R, N, K), q = _mixer_prep(x, p)
    Lb = lib()
    hs = torch.empty(Bsz, E, N, device=x.device)
    sdt = torch.empty(Bsz, E, device=x.device)
    ws = _ws(Lb.pgf_mamba_mixer_workspace(Bsz, L_, d, E, R, N, K, _dt(x), 0), x.device)
    xh = _halo(x_halo, x)
    check(Lb.pgf_mamba_mixer_fwd_begin(_p(x), *[_p(q[k]) for k in MIXER_KEYS], _p(xh), _p(hs), _p(sdt), Bsz, L_, d, E,
                                       R, N, K, _dt(x), _p(ws), ws.numel(), _stream()), "mamba_mixer_fwd_begin")
    return hs, sdt, {"x": x, "q": q, "x_halo": xh, "ws": ws, "dims": (Bsz, L_, d, E, R, N, K)}


def mamba_mixer_fwd_finish(state, h_init, want_states=False):
    """Sequence sharding, forward part 2: the output from the state entering the segment (and, with
    want_states, its boundary states for mamba_mixer_fwd_seg(states_in=...))."""
    x, q, ws = state["x"], state["q"], state["ws"]
    Bsz, L_, d, E, R, N, K = state["dims"]
    out = torch.empty_like(x)
    st = torch.empty(lib().pgf_mamba_mixer_states_size(Bsz, L_, d, E, R, N, K) // 4, device=x.device) \
        if want_states else None
    check(lib().pgf_mamba_mixer_fwd_finish(_p(x), *[_p(q[k]) for k in MIXER_KEYS], _p(state["x_halo"]),
                                           _p(_f32(h_init)), _p(out), _p(st), Bsz, L_, d, E, R, N, K, _dt(x), _p(ws),
                                           ws.numel(), _stream()), "mamba_mixer_fwd_finish")
    return (out, st) if want_states else out


def mamba_mixer_bwd_seg(x, g, p, saved, x_halo=None, dh_end=None, dA_end=None, want_carry=False, want_g_halo=False,
                        acc=None):
    """Gradients of the mixer over one segment (saved: from mamba_mixer_fwd_seg(save=True) on the same
    input with the segment's h_init and x_halo).  Returns (grads, grad_x, grad_x_halo, dh_start,
    dA_start); acc: a dict over MIXER_KEYS of float32 buffers to add the parameter gradients into."""
    x, (Bsz, L_, d, E, R, N, K), q = _mixer_prep(x, p)
    g = _c(g.to(x.dtype))
    acc = acc or {}
    bufs = [_acc_buffer(acc.get(k), tuple(q[k].shape), x.device, "mamba_mixer_bwd_seg") for k in MIXER_KEYS]
    if len({a for _, a in bufs}) != 1:
        raise ValueError("mamba_mixer_bwd_seg: give all accumulators or none")
    grads = {k: b for k, (b, _) in zip(MIXER_KEYS, bufs)}
    accum = bufs[0][1]
    gx = torch.empty_like(x)
    xh = _halo(x_halo, x)
    gh = torch.empty_like(xh) if (want_g_halo and xh is not None) else None
    dh0 = torch.empty(Bsz, E, N, device=x.device) if want_carry else None
    dA0 = torch.empty(Bsz, E, N, device=x.device) if want_carry else None
    Lb = lib()
    ws = _ws(Lb.pgf_mamba_mixer_workspace(Bsz, L_, d, E, R, N, K, _dt(x), 1), x.device)
    check(Lb.pgf_mamba_mixer_bwd_seg(_p(x), _p(g), *[_p(q[k]) for k in MIXER_KEYS], _p(xh), _p(saved), saved.numel(),
                                     _p(_f32(dh_end)), _p(_f32(dA_end)), *[_p(grads[k]) for k in MIXER_KEYS], _p(gx),
                                     _p(gh), _p(dh0), _p(dA0), accum, Bsz, L_, d, E, R, N, K, _dt(x), _p(ws),
                                     ws.numel(), _stream()), "mamba_mixer_bwd_seg")
    return grads, gx, gh, dh0, dA0


def mamba_mixer_bwd_begin(x, g, p, saved, x_halo=None):
    """Sequence sharding, backward part 1: (dh_start, dA_start, sum_dt_excl, state) for a zero end carry."""
    x, (Bsz, L_, d, E, R, N, K), q = _mixer_prep(x, p)
    g = _c(g.to(x.dtype))
    Lb = lib()
    dh0 = torch.empty(Bsz, E, N, device=x.device)
    dA0 = torch.empty(Bsz, E, N, device=x.device)
    sdx = torch.empty(Bsz, E, device=x.device)
    ws = _ws(Lb.pgf_mamba_mixer_workspace(Bsz, L_, d, E, R, N, K, _dt(x), 1), x.device)
    xh = _halo(x_halo, x)
    check(Lb.pgf_mamba_mixer_bwd_begin(_p(x), _p(g), *[_p(q[k]) for k in MIXER_KEYS], _p(xh), _p(saved),
                                       saved.numel(), _p(dh0), _p(dA0), _p(sdx), Bsz, L_, d, E, R, N, K, _dt(x),
                                       _p(ws), ws.numel(), _stream()), "mamba_mixer_bwd_begin")
    return dh0, dA0, sdx, {"x": x, "g": g, "q": q, "x_halo": xh, "saved": saved, "ws": ws,
                           "dims": (Bsz, L_, d, E, R, N, K)}


def mamba_mixer_bwd_finish(state, dh_end=None, dA_end=None, want_g_halo=False):
    """Sequence sharding, backward part 2: (grads, grad_x, grad_x_halo) for the carry from the right."""
    x, g, q, ws, saved, xh = state["x"], state["g"], state["q"], state["ws"], state["saved"], state["x_halo"]
    Bsz, L_, d, E, R, N, K = state["dims"]
    grads = {k: torch.empty_like(q[k]) for k in MIXER_KEYS}
    gx = torch.empty_like(x)
    gh = torch.empty_like(xh) if (want_g_halo and xh is not None) else None
    check(lib().pgf_mamba_mixer_bwd_finish(_p(x), _p(g), *[_p(q[k]) for k in MIXER_KEYS], _p(xh), _p(saved),
                                           saved.numel(), _p(_f32(dh_end)), _p(_f32(dA_end)),
                                           *[_p(grads[k]) for k in MIXER_KEYS], _p(gx), _p(gh), 0, Bsz, L_, d, E, R,
                                           N, K, _dt(x), _p(ws), ws.numel(), _stream()), "mamba_mixer_bwd_finish")
    return grads, gx, gh
