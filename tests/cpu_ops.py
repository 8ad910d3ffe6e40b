"""CPU implementation of the operator namespace that icml_b200.seqpar drives, built on the oracle.

Test infrastructure: it lets the sequence-sharding host logic (segment summaries, all-gathers,
carry composition, gradient all-reduce) run on gloo CPU ranks and be compared with the
single-process oracle.  Signatures follow icml_b200.ops.
"""
import torch
import torch.nn.functional as F

from oracle import pgf_oracle as O


def _params(W_cat, b_cat, A_log, Dp=None, scale=None):
    N = A_log.shape[0]
    d = W_cat.shape[1]
    return {"A_log": A_log.detach(), "D": (Dp if Dp is not None else torch.ones(d)).detach(),
            "scale": (scale if scale is not None else torch.ones(d)).detach(),
            "dt_w": W_cat[:d].detach(), "dt_b": b_cat[:d].detach(), "B_w": W_cat[d:d + N].detach(),
            "B_b": b_cat[d:d + N].detach(), "C_w": W_cat[d + N:].detach(), "C_b": b_cat[d + N:].detach()}


def _dt(u, W_cat, b_cat):
    d = W_cat.shape[1]
    return F.softplus((u @ W_cat.t() + b_cat)[..., :d])


def rmsnorm_fwd(x, w, eps):
    return O.rmsnorm_forward(x, w.detach(), eps)


def rmsnorm_fwd_res(x, res, w, eps):
    s = x + res
    return s, O.rmsnorm_forward(s, w.detach(), eps)


def rmsnorm_bwd(x, g, w, eps, need_gx=True, g_add=None):
    gw, gx = O.rmsnorm_grad(x, g, w.detach(), eps)
    if g_add is not None:
        return gw, gx + g_add
    return gw, (gx if need_gx else None)


def ssm_summary(u, W_cat, b_cat, A_log, h_init=None):
    p = _params(W_cat, b_cat, A_log)
    _, _, h = O.ssm_forward(p, u, u.shape[1], h0=h_init)
    return h, _dt(u, W_cat, b_cat).sum(1)


def ssm_fwd(u, W_cat, b_cat, A_log, Dp, scale, h_init=None, act=None, want_h_final=False):
    p = _params(W_cat, b_cat, A_log, Dp, scale)
    y, _, h = O.ssm_forward(p, u, u.shape[1], h0=h_init, act=act)
    return y, (h if want_h_final else None)


def ssm_fwd_states(u, W_cat, b_cat, A_log, Dp, scale, h_init=None, act=None):
    """The boundary-state buffer's stand-in is the state that entered the segment."""
    y, _ = ssm_fwd(u, W_cat, b_cat, A_log, Dp, scale, h_init=h_init, act=act)
    return y, {"h_init": h_init}


def ssm_fwd_save(u, W_cat, b_cat, A_log, Dp, scale, h_init=None, act=None, states=None):
    if states is not None:
        assert h_init is None
        h_init = states["h_init"]
    y, _ = ssm_fwd(u, W_cat, b_cat, A_log, Dp, scale, h_init=h_init, act=act)
    return y, None


def ssm_bwd_summary(u, g, W_cat, b_cat, A_log, scale, h_init=None, act=None):
    p = _params(W_cat, b_cat, A_log, None, scale)
    B, L, d = u.shape
    N = A_log.shape[0]
    h0 = h_init if h_init is not None else torch.zeros(B, d, N, dtype=u.dtype)
    r = O.ssm_block_grad(p, u, g, h0, torch.zeros(B, d, N, dtype=u.dtype), torch.ones(B, d, N, dtype=u.dtype),
                         act=act)
    return r["delta_h0"], r["dA0"], _dt(u, W_cat, b_cat)[:, 1:].sum(1)


def ssm_fwd_begin(u, W_cat, b_cat, A_log):
    h, sdt = ssm_summary(u, W_cat, b_cat, A_log)
    return h, sdt, {"u": u, "W_cat": W_cat, "b_cat": b_cat, "A_log": A_log}


def ssm_fwd_finish(state, Dp, scale, h_init=None, act=None, want_states=False):
    y, _ = ssm_fwd(state["u"], state["W_cat"], state["b_cat"], state["A_log"], Dp, scale, h_init=h_init, act=act)
    return (y, {"h_init": h_init}) if want_states else y


def ssm_bwd_begin(u, g, W_cat, b_cat, A_log, scale, saved, h_init=None, act=None):
    dh0, dA0, sdx = ssm_bwd_summary(u, g, W_cat, b_cat, A_log, scale, h_init=h_init, act=act)
    return dh0, dA0, sdx, {"u": u, "g": g, "W_cat": W_cat, "b_cat": b_cat, "A_log": A_log, "scale": scale,
                           "h_init": h_init, "saved": saved, "act": act}


def ssm_bwd_finish(state, Dp, dh_end=None, dA_end=None):
    return ssm_bwd(state["u"], state["g"], state["W_cat"], state["b_cat"], state["A_log"], Dp, state["scale"],
                   h_init=state["h_init"], dh_end=dh_end, dA_end=dA_end, act=state["act"], saved=state["saved"])


def ssm_bwd(u, g, W_cat, b_cat, A_log, Dp, scale, h_init=None, dh_end=None, dA_end=None, act=None,
            want_carry=False, saved=None):
    p = _params(W_cat, b_cat, A_log, Dp, scale)
    B, L, d = u.shape
    N = A_log.shape[0]
    z = torch.zeros(B, d, N, dtype=u.dtype)
    r = O.ssm_block_grad(p, u, g, h_init if h_init is not None else z, dh_end if dh_end is not None else z,
                         dA_end if dA_end is not None else torch.ones_like(z), act=act)
    return {"W_cat": torch.cat([r["dt_w"], r["B_w"], r["C_w"]], 0),
            "b_cat": torch.cat([r["dt_b"], r["B_b"], r["C_b"]], 0),
            "A_log": r["A_log"], "D": r["D"], "scale": r["scale"], "grad_u": r["grad_u"],
            "delta_h0": r["delta_h0"], "dA0": r["dA0"]}


def ffn_fwd(x, W1, b1, W2, b2, activation="gelu", residual=None):
    y = O.ffn_forward(x, W1.detach(), b1.detach(), W2.detach(), b2.detach(), activation)
    return y if residual is None else y + residual


def ffn_bwd(x, g, W1, b1, W2, activation="gelu", need_gx=True):
    r = O.ffn_grad(x, g, W1.detach(), b1.detach(), W2.detach(), torch.zeros(W2.shape[0]), activation)
    if not need_gx:
        r.pop("grad_x")
    return r


def embedding_fwd(ids, W, dtype=torch.float32):
    return O.embedding_forward(ids, W.detach()).to(dtype)


def embedding_bwd(ids, g, vocab):
    return torch.zeros(vocab, g.shape[-1], dtype=g.dtype).index_add_(0, ids.reshape(-1), g.reshape(-1, g.shape[-1]))


def lm_head_ce_fwd(h, W, targets):
    logits = h @ W.detach().t()
    lse = torch.logsumexp(logits, -1)
    return lse - logits[torch.arange(h.shape[0]), targets], lse


def lm_head_ce_bwd(h, W, targets, lse, grad_scale, need_gh=True):
    logits = h @ W.detach().t()
    G = torch.exp(logits - lse[:, None])
    G[torch.arange(h.shape[0]), targets] -= 1.0
    G *= grad_scale
    return G.t() @ h, (G @ W.detach() if need_gh else None)


def ssm_compose_ranks_fwd(gathered, rank, A_log, Bsz, D, N):
    """State entering segment `rank`: fold H <- exp(A sum_dt_j) H + h_seg_j over ranks j < rank, from
    rows [h_seg (Bsz,D,N) | sum_dt (Bsz,D)] of `gathered` (the host statement of the kernel's fold)."""
    A = -torch.exp(A_log.detach().to(gathered.dtype))
    A = A if A.dim() == 2 else A.expand(D, N)
    n = Bsz * D * N
    H = torch.zeros(Bsz, D, N, dtype=gathered.dtype)
    for j in range(rank):
        h_loc = gathered[j, :n].view(Bsz, D, N)
        sdt = gathered[j, n:n + Bsz * D].view(Bsz, D, 1)
        H = torch.exp(A * sdt) * H + h_loc
    return H


def ssm_compose_ranks_bwd(gathered, rank, A_log, Bsz, D, N):
    """(dh_end, dA_end) for segment `rank` from rows [dh_start | dA_start | sum_dt_excl]: from the last
    rank down to rank + 1, X = aE G; G <- exp(A sum_dt_excl_j) X + dh_start_j; aE <- dA_start_j."""
    A = -torch.exp(A_log.detach().to(gathered.dtype))
    A = A if A.dim() == 2 else A.expand(D, N)
    n = Bsz * D * N
    G = torch.zeros(Bsz, D, N, dtype=gathered.dtype)
    aE = torch.ones(Bsz, D, N, dtype=gathered.dtype)
    for j in range(gathered.shape[0] - 1, rank, -1):
        d_loc = gathered[j, :n].view(Bsz, D, N)
        dA0 = gathered[j, n:2 * n].view(Bsz, D, N)
        sdx = gathered[j, 2 * n:2 * n + Bsz * D].view(Bsz, D, 1)
        G = torch.exp(A * sdx) * (aE * G) + d_loc
        aE = dA0
    return G, aE


# --------------------------------------------------------------------------- Mamba-standard mixer
def _std_params(p):
    return {k: v.detach() for k, v in p.items()}


def _std_run(p, x, halo=None, h0=None, first_leaf=False):
    """The oracle's standard mixer (oracle/mamba_std.py) over one segment with the conv context rows
    `halo` (mixer inputs of the K-1 tokens before it) and the entering state h0: (out, h_final,
    delta, state after the first token)."""
    from oracle import mamba_std as MS
    E = p["D"].shape[0]
    N = p["A_log"].shape[1]
    R = p["dt_w"].shape[1]
    xz = x @ p["in_w"].t()
    xi, z = xz[..., :E], xz[..., E:]
    pre = halo @ p["in_w"][:E].t() if halo is not None else None
    u = F.silu(MS.causal_conv(xi, p["conv_w"], p["conv_b"], pre))
    xd = u @ p["x_w"].t()
    dt_low, Bm, Cm = xd[..., :R], xd[..., R:R + N], xd[..., R + N:]
    delta = F.softplus(dt_low @ p["dt_w"].t() + p["dt_b"])
    A = -torch.exp(p["A_log"])
    Bsz, L, _ = x.shape
    h = x.new_zeros(Bsz, E, N) if h0 is None else h0
    ys, first = [], None
    for t in range(L):
        h = torch.exp(delta[:, t, :, None] * A) * h + delta[:, t, :, None] * Bm[:, t, None, :] * u[:, t, :, None]
        if t == 0 and first_leaf:
            h.retain_grad()
            first = h
        ys.append((h * Cm[:, t, None, :]).sum(-1) + p["D"] * u[:, t])
    y = torch.stack(ys, 1) * F.silu(z)
    return y @ p["out_w"].t(), h, delta, first


def mamba_mixer_fwd_begin(x, p, x_halo=None):
    q = _std_params(p)
    with torch.no_grad():
        _, hf, delta, _ = _std_run(q, x, x_halo)
    return hf, delta.sum(1), {"x": x, "p": q, "x_halo": x_halo}


def mamba_mixer_fwd_finish(state, h_init, want_states=False):
    with torch.no_grad():
        out, _, _, _ = _std_run(state["p"], state["x"], state["x_halo"], h_init)
    return (out, {"h_init": h_init}) if want_states else out


def mamba_mixer_fwd_seg(x, p, x_halo=None, h_init=None, states_in=None, want_h_final=False, want_states=False,
                        save=False):
    if states_in is not None:
        h_init = states_in["h_init"]
    with torch.no_grad():
        out, hf, _, _ = _std_run(_std_params(p), x, x_halo, h_init)
    return out, hf, {"h_init": h_init}, {"h_init": h_init}


@torch.enable_grad()
def _std_grads(x, g, p, saved, x_halo, dh_end=None, dA_end=None):
    q = {k: v.detach().clone().requires_grad_(True) for k, v in p.items()}
    xx = x.detach().clone().requires_grad_(True)
    hh = x_halo.detach().clone().requires_grad_(True) if x_halo is not None else None
    out, hf, delta, first = _std_run(q, xx, hh, saved["h_init"], first_leaf=True)
    loss = (out * g).sum()
    if dh_end is not None:
        loss = loss + (hf * (dA_end * dh_end)).sum()
    loss.backward()
    A = -torch.exp(q["A_log"].detach())
    return q, xx, hh, first, delta.detach(), A


def mamba_mixer_bwd_begin(x, g, p, saved, x_halo=None):
    q, xx, hh, first, delta, A = _std_grads(x, g, p, saved, x_halo)
    dA0 = torch.exp(delta[:, 0, :, None] * A)
    return first.grad.detach(), dA0, delta[:, 1:].sum(1), {"x": x, "g": g, "p": p, "saved": saved, "x_halo": x_halo}


def mamba_mixer_bwd_finish(state, dh_end=None, dA_end=None, want_g_halo=False):
    q, xx, hh, _, _, _ = _std_grads(state["x"], state["g"], state["p"], state["saved"], state["x_halo"], dh_end,
                                    dA_end)
    grads = {k: v.grad.detach() for k, v in q.items()}
    return grads, xx.grad.detach(), (hh.grad.detach() if (want_g_halo and hh is not None) else None)
