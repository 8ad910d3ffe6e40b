"""Sequence-sharded PGF training step: one long sequence split into contiguous segments, one per rank.

Every operator of the block is token-local except the selective scan, whose recurrence
h_t = exp(dt_t A) h_{t-1} + b_t is affine.  A rank's segment therefore summarises, from a zero
start, to (h_loc, sum_dt): its end state and its total decay exp(A_n * sum_dt).  One all-gather of
those per layer gives every rank the state entering its segment (an exclusive prefix over the
ranks before it); it then runs its segment from that state.  The backward mirrors it: from a zero
carry each rank computes the adjoint at its first token, its first token's decay and the decay of
the rest of its segment; one all-gather per layer gives every rank the carry entering its segment
from the right (the reference's block hand-off, pgf_mamba_block.py:86-112 and :207-234, across
GPUs).  Parameter and embedding gradients are partial sums, all-reduced once per step.

The functions take an `ops` namespace (default: the CUDA operators of icml_b200.ops) so the same
host logic can be exercised with other implementations of the operators.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from . import ops as cuda_ops


@dataclass
class SeqGroup:
    """A process group whose ranks hold consecutive segments of the same sequences."""
    group: Any = None
    rank: int = 0
    world: int = 1

    @staticmethod
    def from_default() -> "SeqGroup":
        if not dist.is_initialized():
            return SeqGroup()
        return SeqGroup(None, dist.get_rank(), dist.get_world_size())

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        """(world, *t.shape) stack of every rank's tensor, in rank order."""
        t = t.contiguous()
        if self.world == 1:
            return t.unsqueeze(0)
        out = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(out, t, group=self.group)
        return torch.stack(out, 0)

    def all_gather_flat(self, ts) -> torch.Tensor:
        """(world, n): each rank's tensors, flattened to float32 and concatenated, in rank order --
        one collective for the whole summary."""
        flat = torch.cat([t.reshape(-1).float() for t in ts])
        if self.world == 1:
            return flat.unsqueeze(0)
        out = torch.empty(self.world * flat.numel(), dtype=flat.dtype, device=flat.device)
        dist.all_gather_into_tensor(out, flat, group=self.group)
        return out.view(self.world, -1)

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t


def _wb(m):
    from .train_singlemamba_optimized import _cat_weights
    return _cat_weights(m)


def _is_std(block) -> bool:
    return hasattr(block, "mixer")


def _prev_rows(sp: SeqGroup, rows: torch.Tensor) -> Optional[torch.Tensor]:
    """The previous rank's `rows` (same shape on every rank), or None on rank 0: the conv context a
    Mamba-standard segment needs from the segment before it."""
    g = sp.all_gather_flat([rows])
    return g[sp.rank - 1].view_as(rows).to(rows.dtype) if sp.rank > 0 else None


def _next_rows(sp: SeqGroup, rows: Optional[torch.Tensor], like: torch.Tensor) -> Optional[torch.Tensor]:
    """The next rank's `rows` (zeros stand in where a rank has none), or None on the last rank."""
    g = sp.all_gather_flat([rows if rows is not None else torch.zeros_like(like)])
    return g[sp.rank + 1].view_as(like).to(like.dtype) if sp.rank + 1 < sp.world else None


@torch.no_grad()
def std_block_forward(block, x: torch.Tensor, sp: SeqGroup, ops=cuda_ops):
    """PGFMambaStdBlock.pgf_forward on this rank's segment: the conv's K-1 context rows come from the
    previous rank, the scan state entering the segment from the composed summaries of all earlier
    ranks (per-channel A).  Returns (y, (conv context rows, boundary states) for std_block_backward)."""
    B, L, D = x.shape
    m = block.mixer
    p = m.params()
    K = m.d_conv
    xn = ops.rmsnorm_fwd(x, block.norm1.weight, block.norm1.eps)
    halo = _prev_rows(sp, xn[:, L - (K - 1):].contiguous()) if (sp.world > 1 and K > 1) else None
    hs, sdt, st = ops.mamba_mixer_fwd_begin(xn, p, x_halo=halo)
    h_in = ops.ssm_compose_ranks_fwd(sp.all_gather_flat([hs, sdt]), sp.rank, m.A_log, B, m.d_inner, m.d_state)
    y, states = ops.mamba_mixer_fwd_finish(st, h_in, want_states=True)
    del st
    x1, xn2 = ops.rmsnorm_fwd_res(y, x, block.norm2.weight, block.norm2.eps)
    f = ops.ffn_fwd(xn2.reshape(-1, D), block.W1, block.b1, block.W2, block.b2, block.ffn_activation,
                    residual=x1.reshape(-1, D))
    return f.reshape(B, L, D), (halo, states)


@torch.no_grad()
def std_block_backward(block, x: torch.Tensor, g_out: torch.Tensor, ctx, sp: SeqGroup, ops=cuda_ops):
    """PGFMambaStdBlock.pgf_backward on this rank's segment (local partial parameter gradients): the
    adjoint carry from the right comes from the composed summaries of the later ranks, and the
    gradient of the next rank's conv context rows is added to this segment's last K-1 rows."""
    B, L, D = x.shape
    m = block.mixer
    p = m.params()
    K = m.d_conv
    halo, states = ctx
    g_out = g_out.to(x.dtype)
    xn1 = ops.rmsnorm_fwd(x, block.norm1.weight, block.norm1.eps)
    m_raw, _, _, saved = ops.mamba_mixer_fwd_seg(xn1, p, x_halo=halo, states_in=states, save=True)
    m_out, xn2 = ops.rmsnorm_fwd_res(m_raw, x, block.norm2.weight, block.norm2.eps)
    del m_raw
    fr = ops.ffn_bwd(xn2.reshape(-1, D), g_out.reshape(-1, D), block.W1, block.b1, block.W2, block.ffn_activation,
                     need_gx=True)
    gn2w, g_m = ops.rmsnorm_bwd(m_out, fr["grad_x"].reshape(B, L, D), block.norm2.weight, block.norm2.eps,
                                g_add=g_out)
    d_loc, dA0, sdx, bst = ops.mamba_mixer_bwd_begin(xn1, g_m, p, saved, x_halo=halo)
    dh_end, dA_end = ops.ssm_compose_ranks_bwd(sp.all_gather_flat([d_loc, dA0, sdx]), sp.rank, m.A_log, B, m.d_inner,
                                               m.d_state)
    mg, gxn1, g_halo = ops.mamba_mixer_bwd_finish(bst, dh_end=dh_end, dA_end=dA_end, want_g_halo=halo is not None)
    del bst, saved
    if sp.world > 1 and K > 1:
        tail = gxn1[:, L - (K - 1):]
        g_next = _next_rows(sp, g_halo, tail)
        if g_next is not None:
            gxn1[:, L - (K - 1):] = tail + g_next
    gn1w, grad_input = ops.rmsnorm_bwd(x, gxn1, block.norm1.weight, block.norm1.eps, g_add=g_m)
    grads = {"W1": fr["grad_W1"], "b1": fr["grad_b1"], "W2": fr["grad_W2"], "b2": fr["grad_b2"],
             "norm1.weight": gn1w, "norm2.weight": gn2w}
    grads.update(m.grads_to_named(mg, "mixer."))
    return {"grads": grads, "grad_input": grad_input}


@torch.no_grad()
def block_forward(block, x: torch.Tensor, sp: SeqGroup, ops=cuda_ops):
    """PGFMambaBlock.pgf_forward on this rank's segment; returns (y, state entering the segment,
    the scan's boundary states for block_backward)."""
    if _is_std(block):
        y, ctx = std_block_forward(block, x, sp, ops)
        return y, None, ctx
    B, L, D = x.shape
    m = block.mamba
    W, b = _wb(m)
    xn = ops.rmsnorm_fwd(x, block.norm1.weight, block.norm1.eps)
    if sp.world > 1:
        # the zero-start pass gives the segment summary; the output pass continues from it
        h_loc, sdt, st = ops.ssm_fwd_begin(xn, W, b, m.A_log)
        h_in = ops.ssm_compose_ranks_fwd(sp.all_gather_flat([h_loc, sdt]), sp.rank, m.A_log, B, D, m.d_state)
        y, states = ops.ssm_fwd_finish(st, m.D, m.scale, h_init=h_in, act=m.output_activation, want_states=True)
        del st
    else:
        h_in = None
        y, states = ops.ssm_fwd_states(xn, W, b, m.A_log, m.D, m.scale, act=m.output_activation)
    x1, xn2 = ops.rmsnorm_fwd_res(y, x, block.norm2.weight, block.norm2.eps)  # y + x, then norm2
    f = ops.ffn_fwd(xn2.reshape(-1, D), block.W1, block.b1, block.W2, block.b2, block.ffn_activation,
                    residual=x1.reshape(-1, D))  # ffn(norm2(x1)) + x1
    return f.reshape(B, L, D), h_in, states


@torch.no_grad()
def block_backward(block, x: torch.Tensor, g_out: torch.Tensor, h_in: Optional[torch.Tensor], sp: SeqGroup,
                   ops=cuda_ops, states=None) -> Dict[str, Any]:
    """PGFMambaBlock.pgf_backward on this rank's segment (local partial parameter gradients).  With
    `states` from block_forward on the same input, the scan's forward is one pass."""
    if _is_std(block):
        return std_block_backward(block, x, g_out, states, sp, ops)
    B, L, D = x.shape
    m = block.mamba
    W, b = _wb(m)
    g_out = g_out.to(x.dtype)
    xn1 = ops.rmsnorm_fwd(x, block.norm1.weight, block.norm1.eps)
    if states is not None:
        y, saved = ops.ssm_fwd_save(xn1, W, b, m.A_log, m.D, m.scale, act=m.output_activation, states=states)
    else:
        y, saved = ops.ssm_fwd_save(xn1, W, b, m.A_log, m.D, m.scale, h_init=h_in, act=m.output_activation)
    m_out, xn2 = ops.rmsnorm_fwd_res(y, x, block.norm2.weight, block.norm2.eps)
    fr = ops.ffn_bwd(xn2.reshape(-1, D), g_out.reshape(-1, D), block.W1, block.b1, block.W2,
                     block.ffn_activation, need_gx=True)
    gn2w, g_m = ops.rmsnorm_bwd(m_out, fr["grad_x"].reshape(B, L, D), block.norm2.weight, block.norm2.eps,
                                g_add=g_out)  # norm2's grad_x + g_out
    if sp.world > 1:
        # the reverse chunk pass gives the segment's adjoint summary; the gradients continue from it
        d_loc, dA0, sdx, st = ops.ssm_bwd_begin(xn1, g_m, W, b, m.A_log, m.scale, saved, h_init=h_in,
                                                act=m.output_activation)
        dh_end, dA_end = ops.ssm_compose_ranks_bwd(sp.all_gather_flat([d_loc, dA0, sdx]), sp.rank, m.A_log, B, D,
                                                   m.d_state)
        r = ops.ssm_bwd_finish(st, m.D, dh_end=dh_end, dA_end=dA_end)
        del st
    else:
        r = ops.ssm_bwd(xn1, g_m, W, b, m.A_log, m.D, m.scale, h_init=h_in, act=m.output_activation, saved=saved)
    del saved
    gn1w, grad_input = ops.rmsnorm_bwd(x, r["grad_u"], block.norm1.weight, block.norm1.eps, g_add=g_m)
    d, N = m.d_model, m.d_state
    gscale = r["scale"].sum().expand(d).clone() if m.reference_scale_grad else r["scale"]
    grads = {
        "W1": fr["grad_W1"], "b1": fr["grad_b1"], "W2": fr["grad_W2"], "b2": fr["grad_b2"],
        "mamba.A_log": r["A_log"], "mamba.D": r["D"], "mamba.scale": gscale,
        "mamba.dt_proj.weight": r["W_cat"][:d], "mamba.dt_proj.bias": r["b_cat"][:d],
        "mamba.B_proj.weight": r["W_cat"][d:d + N], "mamba.B_proj.bias": r["b_cat"][d:d + N],
        "mamba.C_proj.weight": r["W_cat"][d + N:], "mamba.C_proj.bias": r["b_cat"][d + N:],
        "norm1.weight": gn1w, "norm2.weight": gn2w,
    }
    return {"grads": grads, "grad_input": grad_input}


@torch.no_grad()
def lm_forward_backward(model, input_ids: torch.Tensor, targets: torch.Tensor, sp: SeqGroup,
                        ops=cuda_ops, total_tokens: Optional[int] = None, reducer=None):
    """The PGF LM step on this rank's segment of every sequence.  Returns (global mean loss, grads):
    gradients are summed over ranks (all-reduce), the loss is the mean over all ranks' tokens.  With
    `reducer` (an optim.OverlappedGradReduce with SUM) the gradients are summed layer by layer into the
    flat optimizer's gradient buffer while the backward goes on, and the returned ones stay local."""
    B, L = input_ids.shape
    d = model.d_model
    T_total = total_tokens if total_tokens is not None else B * L * sp.world
    x = ops.embedding_fwd(input_ids, model.emb_weight, dtype=model.act_dtype)
    stash: List[Tuple[torch.Tensor, Optional[torch.Tensor], Any]] = []
    for layer in model.backbone.layers:
        y, h_in, states = block_forward(layer, x, sp, ops)
        stash.append((x, h_in, states))
        x = y
    xf = ops.rmsnorm_fwd(x, model.final_norm.weight, model.final_norm.eps) if model.final_norm is not None else x
    h = xf.reshape(-1, d)
    tg = targets.reshape(-1)
    loss_rows, lse = ops.lm_head_ce_fwd(h, model.lm_head_weight, tg)
    gW, gh = ops.lm_head_ce_bwd(h, model.lm_head_weight, tg, lse, 1.0 / T_total)
    grads = {"lm_head": gW}
    g = gh.reshape(B, L, d)
    if model.final_norm is not None:
        grads["final_norm"], g = ops.rmsnorm_bwd(x, g, model.final_norm.weight, model.final_norm.eps)
    del x, xf, h, gh
    for i in reversed(range(model.n_layers)):
        xi, h_in, states = stash.pop()
        res = block_backward(model.backbone.layers[i], xi, g, h_in, sp, ops, states=states)
        for k, v in res["grads"].items():
            grads[f"layers.{i}.{k}"] = v
        if reducer is not None:
            reducer.layer(i, res["grads"])
        g = res["grad_input"]
    grads["emb"] = ops.embedding_bwd(input_ids, g, model.vocab_size)
    if getattr(model, "tied", False):
        grads["emb"] = grads["emb"] + grads.pop("lm_head")
    loss_sum = loss_rows.sum().reshape(1).float()
    if reducer is not None:
        reducer.finish(grads, extra=loss_sum)
    elif sp.world > 1:
        names = sorted(grads)
        flat = torch.cat([grads[k].reshape(-1).float() for k in names] + [loss_sum])
        sp.all_reduce_(flat)
        o = 0
        for k in names:
            n = grads[k].numel()
            grads[k] = flat[o:o + n].view_as(grads[k])
            o += n
        loss_sum = flat[o:o + 1]
    return loss_sum[0] / T_total, grads


__all__ = ["SeqGroup", "block_forward", "block_backward", "lm_forward_backward"]
