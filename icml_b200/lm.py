"""PGF language-model training step (the reference's ExternalPGFLanguageModel,
train_wikitext_rebuttal.py:58-149) on libpgf.so.

Differences from the reference's step, none of which changes the mathematics:
* the LM head and cross entropy are fused and tiled over tokens and vocabulary, so the (T, V)
  logits are never materialised (the reference builds them and their softmax in full);
* activations between operators may be bfloat16 (``act_dtype``), parameters, gradients and the
  optimizer state stay float32;
* ``step()`` returns the loss as a device tensor, so a training loop need not synchronise.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.nn as nn

from . import ops
from .pgf_mamba_block import PGFMambaBlock, PGFMambaSequential
from .pgf_rmsnorm import RMSNorm


class LayerStash:
    """Where the step keeps each layer's input between its forward and its backward (the
    ``layer_inputs`` list of train_wikitext_rebuttal.py:105-108, popped at :133).

    policy "device": on the GPU (what the reference does; bf16 when the activations are bf16).
    policy "host": each input except the last layer's is copied to pinned host memory on a copy
    stream as soon as it is produced (its device memory is released when the copy has run), and the
    backward brings input i-1 back while layer i runs its backward, so at most two stashed inputs
    occupy device memory instead of one per layer.  The copies are ordered against the compute
    stream with stream waits only, so the step stays capturable in a CUDA graph (the pinned buffers
    are allocated at the first step and reused).
    policy "scan": as "device", and each layer's forward also keeps what its backward would
    recompute before the scan backward (the scan's 8-token checkpoints and the residual sum), so the
    backward runs no forward scan.  More device memory (about 10.5 bytes per token and channel per
    layer in bf16) for less recompute.
    """

    def __init__(self, policy: str = "device"):
        if policy not in ("device", "host", "scan"):
            raise ValueError(f"stash policy: {policy!r}")
        self.policy = policy
        self._host: Dict[int, torch.Tensor] = {}
        self._stream: Optional[torch.cuda.Stream] = None
        self.items: List = []

    def begin(self, n: int):
        self.items = [None] * n
        self._where = ["device"] * n

    def _copy_stream(self, dev) -> torch.cuda.Stream:
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=dev)
        return self._stream

    def put(self, i: int, x: torch.Tensor):
        n = len(self.items)
        if self.policy != "host" or i == n - 1 or not x.is_cuda:
            self.items[i] = x
            return
        h = self._host.get(i)
        if h is None or h.shape != x.shape or h.dtype != x.dtype:
            h = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
            self._host[i] = h
        cur = torch.cuda.current_stream(x.device)
        cs = self._copy_stream(x.device)
        cs.wait_stream(cur)
        with torch.cuda.stream(cs):
            h.copy_(x, non_blocking=True)
        x.record_stream(cs)  # x's memory returns to the allocator once the copy has run
        self.items[i] = h
        self._where[i] = "host"

    def prefetch(self, i: int, dev):
        """Start bringing input i back (on the copy stream, after its own download)."""
        if self._where[i] != "host":
            return
        h = self.items[i]
        d = torch.empty(h.shape, dtype=h.dtype, device=dev)  # allocated on the compute stream
        cs = self._copy_stream(dev)
        cs.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(cs):
            d.copy_(h, non_blocking=True)
        d.record_stream(cs)
        self.items[i] = d
        self._where[i] = "inflight"

    def take(self, i: int, dev) -> torch.Tensor:
        if self._where[i] == "host":
            self.prefetch(i, dev)
        if self._where[i] == "inflight":
            torch.cuda.current_stream(dev).wait_stream(self._copy_stream(dev))
            self._where[i] = "device"
        x = self.items[i]
        self.items[i] = None
        return x


class PGFLanguageModel:
    def __init__(self, vocab_size: int, d_model: int, d_state: int, d_ff: int, n_layers: int,
                 block_size: int, device, act_dtype=torch.float32, lr: float = 1e-3,
                 weight_decay: float = 0.01, tie_embeddings: bool = False, init_std: float = 0.02,
                 variant: str = "reference", final_norm: bool = False, expand: int = 2, d_conv: int = 4,
                 dt_rank: Optional[int] = None, optimizer: Optional[str] = None,
                 max_grad_norm: Optional[float] = None, stash: str = "device"):
        """variant "reference": the reference's PGFMambaBlock; "std": the Mamba-standard block
        (pgf_mamba_std.PGFMambaStdBlock).  final_norm adds an RMSNorm before the LM head.
        optimizer "flat" (default on a GPU): AdamW over one flat parameter buffer on libpgf's kernels
        (icml_b200.optim.FlatAdamW); "torch": torch.optim.AdamW (fused on a GPU).  max_grad_norm
        clips the global gradient norm first (flat optimizer only).  stash: where the layer inputs wait
        for the backward, "device" or "host" (pinned host memory; LayerStash)."""
        self.vocab_size = vocab_size
        self.d_model = d_model
        self.block_size = block_size
        self.n_layers = n_layers
        self.device = torch.device(device)
        self.act_dtype = act_dtype
        self.emb_weight = nn.Parameter(torch.randn(vocab_size, d_model, device=device) * init_std)
        self.tied = tie_embeddings
        self.lm_head_weight = (self.emb_weight if tie_embeddings else
                               nn.Parameter(torch.randn(vocab_size, d_model, device=device) * init_std))
        if variant == "reference":
            blocks = [PGFMambaBlock(d_model, d_state, d_ff, block_size) for _ in range(n_layers)]
        elif variant == "std":
            from .pgf_mamba_std import PGFMambaStdBlock
            blocks = [PGFMambaStdBlock(d_model, d_state, d_ff, block_size, expand, d_conv, dt_rank)
                      for _ in range(n_layers)]
        else:
            raise ValueError(variant)
        self.variant = variant
        self.backbone = PGFMambaSequential(blocks).to(device)
        self.final_norm = RMSNorm(d_model).to(device) if final_norm else None
        self.stash = LayerStash(stash)
        from .train_singlemamba_optimized import flat_order
        self.params = [self.emb_weight] + ([] if tie_embeddings else [self.lm_head_weight]) + \
            flat_order(self.backbone.parameters(), self.backbone) + \
            (list(self.final_norm.parameters()) if final_norm else [])
        on_gpu = self.device.type == "cuda"
        self.optimizer_kind = optimizer or ("flat" if on_gpu else "torch")
        if self.optimizer_kind == "flat":
            from .optim import FlatAdamW
            self.optimizer = FlatAdamW(self.params, lr=lr, weight_decay=weight_decay, max_grad_norm=max_grad_norm)
        elif self.optimizer_kind == "torch":
            if max_grad_norm is not None:
                raise ValueError("max_grad_norm needs optimizer='flat'")
            # capturable: the optimizer keeps its step count on the device, so the step can be
            # captured in a CUDA graph (GraphedStep)
            self.optimizer = torch.optim.AdamW(self.params, lr=lr, weight_decay=weight_decay, fused=on_gpu,
                                               capturable=on_gpu)
        else:
            raise ValueError(f"optimizer: {optimizer!r}")

    @torch.no_grad()
    def load_(self, emb: torch.Tensor, lm_head: torch.Tensor, backbone_state: Dict[str, torch.Tensor]):
        self.emb_weight.copy_(emb)
        if not self.tied:
            self.lm_head_weight.copy_(lm_head)
        self.backbone.load_state_dict(backbone_state)

    @torch.no_grad()
    def forward_backward(self, input_ids: torch.Tensor, targets: torch.Tensor, on_layer_grads=None):
        """PGF pass 1 over all layers (stashing each layer's input), fused LM head + CE, pass 2 in
        reverse.  Returns (loss tensor, {param name: grad}).  on_layer_grads(i, {name: grad}) is
        called as soon as layer i's gradients are final (e.g. to start their all-reduce)."""
        B, L = input_ids.shape
        d = self.d_model
        x = ops.embedding_fwd(input_ids, self.emb_weight, dtype=self.act_dtype)
        stash = self.stash
        stash.begin(self.n_layers)
        # every block hands its scan's boundary states to its backward (PGF keeps them per block)
        ssm_states: List[Optional[torch.Tensor]] = [None] * self.n_layers
        keep = stash.policy == "scan"
        for i, layer in enumerate(self.backbone.layers):
            stash.put(i, x)
            x, ssm_states[i] = layer.pgf_forward(x, return_ssm_states=True, keep_scan=keep)
        xf = ops.rmsnorm_fwd(x, self.final_norm.weight, self.final_norm.eps) if self.final_norm is not None else x
        h = xf.reshape(-1, d)
        tg = targets.reshape(-1)
        loss_rows, lse = ops.lm_head_ce_fwd(h, self.lm_head_weight, tg)
        loss = loss_rows.mean()
        gW, gh = ops.lm_head_ce_bwd(h, self.lm_head_weight, tg, lse, 1.0 / h.shape[0])
        grads = {"lm_head": gW}
        g = gh.reshape(B, L, d)
        if self.final_norm is not None:
            gfw, g = ops.rmsnorm_bwd(x, g, self.final_norm.weight, self.final_norm.eps)
            grads["final_norm"] = gfw
        del x, xf, h, gh
        for i in reversed(range(self.n_layers)):
            xi = stash.take(i, g.device)
            if i > 0:
                stash.prefetch(i - 1, g.device)  # overlaps this layer's backward
            res = self.backbone.layers[i].pgf_backward(xi, g, ssm_states=ssm_states[i])
            ssm_states[i] = None
            del xi
            for k, v in res["grads"].items():
                grads[f"layers.{i}.{k}"] = v
            if on_layer_grads is not None:
                on_layer_grads(i, res["grads"])
            g = res["grad_input"]
            del res
        grads["emb"] = ops.embedding_bwd(input_ids, g, self.vocab_size)
        if self.tied:
            grads["emb"] = grads["emb"] + grads.pop("lm_head")
        return loss, grads

    def _assign(self, grads):
        self.emb_weight.grad = grads["emb"]
        if not self.tied:
            self.lm_head_weight.grad = grads["lm_head"]
        if self.final_norm is not None:
            self.final_norm.weight.grad = grads["final_norm"]
        for i, layer in enumerate(self.backbone.layers):
            for name, p in layer.named_parameters():
                p.grad = grads[f"layers.{i}.{name}"]

    def step(self, input_ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One training step (forward, backward, AdamW); returns the loss without syncing."""
        self.optimizer.zero_grad(set_to_none=True)
        loss, grads = self.forward_backward(input_ids, targets)
        self._assign(grads)
        self.optimizer.step()
        return loss

    def train_step_pgf(self, input_ids: torch.Tensor, targets: torch.Tensor) -> float:
        """train_wikitext_rebuttal.py:98-149."""
        return self.step(input_ids, targets).item()


class GraphedStep:
    """One whole training step (embedding, PGF forward/backward of every layer, LM head + CE, AdamW,
    and, on several GPUs, the step's NCCL collectives) captured once as a CUDA graph and replayed.

    The step launches about a thousand kernels; replaying them as one graph removes the host's
    per-launch work (Python, ctypes, the launch API), which otherwise sets the pace whenever the
    host must wait for a step's loss.  Inputs live in static device buffers: ``run(x, y)`` copies
    the step's ids and targets into them (from pinned host memory or the device), replays the
    graph and returns the loss tensor, whose storage is reused by the next replay.  Construction
    runs ``warmup`` eager steps (real training steps) on a side stream first, as capture requires
    the optimizer state, the collectives' communicators and every workspace size to be settled.

    ``step`` is ``model`` (its ``step(x, y)``) or any callable ``(x, y) -> loss`` (e.g. a sequence-
    sharded or data-parallel step; every rank must capture the same collectives in the same order).
    Delete the object (``release()``) before destroying a process group whose collectives it holds.
    """

    def __init__(self, step, input_ids: torch.Tensor, targets: torch.Tensor, warmup: int = 2):
        from ._lib import lib
        fn = step.step if isinstance(step, PGFLanguageModel) else step
        dev = input_ids.device if input_ids.is_cuda else torch.device("cuda", torch.cuda.current_device())
        self.x = torch.empty_like(input_ids, device=dev)
        self.y = torch.empty_like(targets, device=dev)
        self.x.copy_(input_ids)
        self.y.copy_(targets)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn(self.x, self.y)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        n0 = lib().pgf_launch_count()
        with torch.cuda.graph(self.graph):
            self.loss = fn(self.x, self.y)
        self.launches = int(lib().pgf_launch_count() - n0)  # libpgf kernels per replay

    def run(self, input_ids: Optional[torch.Tensor] = None, targets: Optional[torch.Tensor] = None) -> torch.Tensor:
        if input_ids is not None:
            self.x.copy_(input_ids, non_blocking=True)
        if targets is not None:
            self.y.copy_(targets, non_blocking=True)
        self.graph.replay()
        return self.loss

    def release(self) -> None:
        self.graph.reset()
        self.loss = None


__all__ = ["PGFLanguageModel", "GraphedStep", "LayerStash"]
