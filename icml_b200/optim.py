"""AdamW over one flat float32 parameter buffer, on libpgf's kernels (pgf_adamw_step, pgf_grad_norm).

The reference steps ``torch.optim.AdamW(params, lr=1e-3, weight_decay=0.01)`` after every PGF step
(train_wikitext_rebuttal.py:77,148).  ``FlatAdamW`` is that optimizer with the same arithmetic, over
a single contiguous buffer: the parameters become views into it (their ``.data`` is re-pointed)
and one multi-tensor kernel updates every parameter and both moments in a single HBM pass, reading
each gradient where the backward left it.  Clipping, or a caller that reduces gradients across
GPUs, gathers them into one flat gradient buffer first (one launch).  ``max_grad_norm`` adds the global-norm clipping
of ``torch.nn.utils.clip_grad_norm_`` (a deterministic two-level sum of squares; the clip factor
stays on the device).  The step count lives on the device, so the whole step can be captured in a
CUDA graph.
"""
from __future__ import annotations

import ctypes
from typing import Iterable, List, Optional, Sequence

import torch

from ._lib import check, lib
from .ops import _stream


class FlatAdamW:
    def __init__(self, params: Iterable[torch.nn.Parameter], lr: float = 1e-3, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.01, max_grad_norm: Optional[float] = None):
        self.params: List[torch.nn.Parameter] = list(params)
        if not self.params:
            raise ValueError("FlatAdamW: no parameters")
        dev = self.params[0].device
        if dev.type != "cuda":
            raise RuntimeError("FlatAdamW runs on libpgf's CUDA kernels; parameters must be on a GPU")
        for p in self.params:
            if p.dtype != torch.float32 or p.device != dev:
                raise ValueError("FlatAdamW: parameters must be float32 on one device")
        self.lr, self.betas, self.eps, self.weight_decay = lr, tuple(betas), eps, weight_decay
        self.max_grad_norm = max_grad_norm
        # 4-element (16-byte) aligned slots, so every slice starts where the vector loads can
        self.offsets = []
        off = 0
        for p in self.params:
            self.offsets.append(off)
            off += (p.numel() + 3) // 4 * 4
        self.n = off
        self.flat = torch.zeros(self.n, device=dev, dtype=torch.float32)
        with torch.no_grad():
            for p, o in zip(self.params, self.offsets):
                view = self.flat[o:o + p.numel()].view_as(p)
                view.copy_(p)
                p.data = view
        self.grad = torch.zeros_like(self.flat)
        self.exp_avg = torch.zeros_like(self.flat)
        self.exp_avg_sq = torch.zeros_like(self.flat)
        self.step_count = torch.zeros(1, device=dev, dtype=torch.float32)
        self.grad_norm = torch.zeros(1, device=dev, dtype=torch.float32)
        self.clip = torch.ones(1, device=dev, dtype=torch.float32)
        self._norm_ws = torch.empty(max(lib().pgf_grad_norm_workspace(self.n), 8), device=dev, dtype=torch.uint8)
        self._keep: List[torch.Tensor] = []

    def zero_grad(self, set_to_none: bool = True):
        for p in self.params:
            p.grad = None

    def _table(self, grads: Optional[Sequence[Optional[torch.Tensor]]]):
        """Host arrays (gradient pointers, flat offsets, sizes) for the multi-tensor calls."""
        gs = [p.grad for p in self.params] if grads is None else list(grads)
        ptrs = []
        for p, g in zip(self.params, gs):
            if g is None:
                ptrs.append(None)
                continue
            if g.dtype != torch.float32 or g.device != p.device or g.shape != p.shape:
                raise ValueError("FlatAdamW: gradients must match their parameters (float32, same shape)")
            g = g.contiguous()
            self._keep.append(g)
            ptrs.append(g.data_ptr())
        k = len(ptrs)
        return ((ctypes.c_void_p * k)(*ptrs), (ctypes.c_int64 * k)(*self.offsets),
                (ctypes.c_int64 * k)(*[p.numel() for p in self.params]), k)

    @torch.no_grad()
    def gather(self, grads: Optional[Sequence[Optional[torch.Tensor]]] = None):
        """Copy the step's gradients (default: each parameter's ``.grad``; None = zero) into the flat
        gradient buffer ``self.grad`` (one launch)."""
        self._keep = []
        ptrs, offs, sizes, k = self._table(grads)
        check(lib().pgf_gather_multi(self.grad.data_ptr(), self.n, ptrs, offs, sizes, k, _stream()),
              "pgf_gather_multi")
        self._keep = []

    @torch.no_grad()
    def gather_subset(self, params: Sequence[torch.nn.Parameter], grads: Sequence[torch.Tensor]):
        """Copy the gradients of some parameters into their slots of ``self.grad`` (one launch)."""
        idx = {id(p): k for k, p in enumerate(self.params)}
        ks = [idx[id(p)] for p in params]
        keep = [g.contiguous() for g in grads]
        for k, g in zip(ks, keep):
            p = self.params[k]
            if g.dtype != torch.float32 or g.shape != p.shape or g.device != p.device:
                raise ValueError("FlatAdamW: gradients must match their parameters (float32, same shape)")
        n = len(ks)
        ptrs = (ctypes.c_void_p * n)(*[g.data_ptr() for g in keep])
        offs = (ctypes.c_int64 * n)(*[self.offsets[k] for k in ks])
        sizes = (ctypes.c_int64 * n)(*[self.params[k].numel() for k in ks])
        check(lib().pgf_gather_multi(self.grad.data_ptr(), self.n, ptrs, offs, sizes, n, _stream()),
              "pgf_gather_multi")

    def slice_of(self, params: Sequence[torch.nn.Parameter]) -> torch.Tensor:
        """The range of ``self.grad`` covering the slots of these parameters (adjacent in the buffer)."""
        idx = {id(p): k for k, p in enumerate(self.params)}
        ks = sorted(idx[id(p)] for p in params)
        if ks != list(range(ks[0], ks[-1] + 1)):
            raise ValueError("FlatAdamW.slice_of: the parameters are not adjacent in the flat buffer")
        a = self.offsets[ks[0]]
        b = self.offsets[ks[-1]] + (self.params[ks[-1]].numel() + 3) // 4 * 4
        return self.grad[a:b]

    @torch.no_grad()
    def step(self, grads: Optional[Sequence[Optional[torch.Tensor]]] = None, gather: bool = True):
        """One AdamW step.  Without clipping, the update reads each gradient where it lies (no flat
        copy); with clipping the gradients are gathered first.  gather=False uses the flat gradient
        buffer as it stands (a caller that gathered and, e.g., all-reduced it in place)."""
        s = _stream()
        L = lib()
        b1, b2 = self.betas
        hyper = (float(self.lr), float(b1), float(b2), float(self.eps), float(self.weight_decay))
        if gather and self.max_grad_norm is None:
            self._keep = []
            ptrs, offs, sizes, k = self._table(grads)
            check(L.pgf_adamw_step_multi(self.flat.data_ptr(), self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(),
                                         self.n, ptrs, offs, sizes, k, *hyper, self.step_count.data_ptr(), None, s),
                  "pgf_adamw_step_multi")
            self._keep = []
            return
        if gather:
            self.gather(grads)
        clip_ptr = None
        if self.max_grad_norm is not None:
            check(L.pgf_grad_norm(self.grad.data_ptr(), self.n, self.grad_norm.data_ptr(), float(self.max_grad_norm),
                                  self.clip.data_ptr(), self._norm_ws.data_ptr(), self._norm_ws.numel(), s),
                  "pgf_grad_norm")
            clip_ptr = self.clip.data_ptr()
        check(L.pgf_adamw_step(self.flat.data_ptr(), self.grad.data_ptr(), self.exp_avg.data_ptr(),
                               self.exp_avg_sq.data_ptr(), self.n, *hyper, self.step_count.data_ptr(), clip_ptr, s),
              "pgf_adamw_step")


class OverlappedGradReduce:
    """All-reduce of the step's gradients across ranks, layer by layer while the backward goes on.

    PGF's backward finishes the gradients of layer i as soon as that layer's pgf_backward returns
    (pgf_mamba_block.py:238), so each layer's gradients are copied into their (adjacent) slots of the
    flat optimizer's gradient buffer and all-reduced there on a side stream, overlapping the
    backward of the layers below; ``finish`` reduces the rest (embedding, LM head, final norm) and
    joins the side stream.  Works inside CUDA-graph capture (every rank issues the same collectives
    in the same order).  op: ReduceOp.AVG for data parallelism (replicas), SUM for sequence sharding
    (partial sums)."""

    def __init__(self, model, op):
        import torch.distributed as dist
        self.dist = dist
        self.model = model
        self.opt = model.optimizer
        self.op = op
        self.stream = torch.cuda.Stream(device=self.opt.flat.device)

    def _reduce(self, params, grads):
        self.opt.gather_subset(params, grads)
        sl = self.opt.slice_of(params)
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            self.dist.all_reduce(sl, op=self.op)

    def layer(self, i: int, grads) -> None:
        named = list(self.model.backbone.layers[i].named_parameters())
        self._reduce([p for _, p in named], [grads[n] for n, _ in named])

    def finish(self, grads, extra: Optional[torch.Tensor] = None) -> None:
        """Reduce the non-layer gradients (and `extra`, e.g. a loss sum, in place), then wait for all."""
        m = self.model
        ps, gs = [m.emb_weight], [grads["emb"]]
        if not m.tied:
            ps.append(m.lm_head_weight)
            gs.append(grads["lm_head"])
        if m.final_norm is not None:
            ps.append(m.final_norm.weight)
            gs.append(grads["final_norm"])
        self.opt.gather_subset(ps, gs)
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            for p in ps:
                self.dist.all_reduce(self.opt.slice_of([p]), op=self.op)
            if extra is not None:
                self.dist.all_reduce(extra, op=self.op)
        torch.cuda.current_stream().wait_stream(self.stream)


def grad_norm(grad: torch.Tensor, max_norm: Optional[float] = None):
    """Global L2 norm of a flat float32 gradient (and the clip factor when max_norm is given)."""
    if grad.dtype != torch.float32 or not grad.is_cuda or not grad.is_contiguous():
        raise ValueError("grad_norm: contiguous float32 CUDA tensor expected")
    n = grad.numel()
    norm = torch.empty(1, device=grad.device)
    clip = torch.empty(1, device=grad.device) if max_norm is not None else None
    ws = torch.empty(max(lib().pgf_grad_norm_workspace(n), 8), device=grad.device, dtype=torch.uint8)
    check(lib().pgf_grad_norm(grad.data_ptr(), n, norm.data_ptr(), float(max_norm or 0.0),
                              clip.data_ptr() if clip is not None else None, ws.data_ptr(), ws.numel(), _stream()),
          "pgf_grad_norm")
    return (norm, clip) if max_norm is not None else norm
