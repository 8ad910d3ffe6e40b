"""The drop-in modules driven exactly as the reference's own scripts drive them, on the GPU.

* test_multi_layer_grads.py:10-126: the reference's gradient-exactness check, with the drop-in
  directory first on sys.path so that ``from pgf_embedding import ...`` etc. resolve to this
  repository's modules: ``pgf_embedding_forward`` / ``pgf_embedding_grad``,
  ``PGFMambaBlock.pgf_forward`` / ``pgf_backward`` per layer, ``pgf_lm_head_forward`` and
  ``pgf_lm_head_grad`` on the full ``g_logits`` built by the reference's ``ce_loss_and_grad``.
  Inputs, weights and expected gradients are the reference's own run of that script at its
  configuration (seed 1, B=2, L=512, d_model 64, d_ff 128, block 128, vocab 1000, 2 layers;
  tests/golden/multilayer.pt).
* PGFMambaSequential.pgf_train_step (pgf_mamba_block.py:290-322) and
  SingleLayerMambaPGF.pgf_train_step (train_singlemamba_optimized.py:474-561) against the
  reference's outputs for the same inputs (tests/golden/train_step.pt).

Bound everywhere: max-abs error <= 1e-5 + 1e-4 * max|reference| per tensor.  ``mamba.scale`` is
compared twice: with ``reference_scale_grad`` set against the reference's PGF value (a scalar
broadcast into every channel, train_singlemamba_optimized.py:400), and by default against autograd
of the reference forward (the per-channel gradient).
"""
import importlib
import os
import sys

import pytest
import torch
import torch.nn.functional as F

from tests.conftest import ROOT, golden
from tests.parity import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
DROPIN = os.path.join(ROOT, "icml_b200", "dropin")


@pytest.fixture(scope="module")
def ref_modules():
    """The reference's module names, resolved to the drop-in directory."""
    sys.path.insert(0, DROPIN)
    try:
        mods = {n: importlib.import_module(n) for n in
                ("pgf_embedding", "pgf_mamba_block", "pgf_lm_head", "train_singlemamba_optimized")}
    finally:
        sys.path.remove(DROPIN)
    assert mods["pgf_mamba_block"].PGFMambaBlock.__module__ == "icml_b200.pgf_mamba_block"
    return mods


def _multilayer_flow(M, G, scale_reference):
    """test_multi_layer_grads.py:43-126 with the golden's weights (the reference's own calls)."""
    ids, targets = G["ids"].to(DEV), G["targets"].to(DEV)
    V, d = G["emb"].shape
    B, L = ids.shape
    bs, nl = G["block_size"], G["n_layers"]
    emb_weight_pgf = G["emb"].to(DEV).requires_grad_(True)
    lm_head_weight_pgf = G["lm_head"].to(DEV).requires_grad_(True)
    blocks = [M["pgf_mamba_block"].PGFMambaBlock(d, 16, G["d_ff"], bs).to(DEV) for _ in range(nl)]
    backbone = M["pgf_mamba_block"].PGFMambaSequential(blocks).to(DEV)
    backbone.load_state_dict({k: v.to(DEV) for k, v in G["params"].items()})
    for blk in backbone.layers:
        blk.reference_scale_grad = scale_reference

    def ce_loss_and_grad(logits, targets_inner):  # :74-86
        logits_flat = logits.view(-1, V)
        targets_flat = targets_inner.view(-1)
        loss_val = F.cross_entropy(logits_flat, targets_flat)
        probs = F.softmax(logits_flat, dim=-1)
        g = probs.clone()
        g[torch.arange(g.size(0)), targets_flat] -= 1.0
        g /= logits_flat.size(0)
        return loss_val, g.view(logits.shape)

    hidden = M["pgf_embedding"].pgf_embedding_forward(ids, emb_weight_pgf, bs)
    layer_inputs = []
    cur = hidden
    for layer in backbone.layers:
        layer_inputs.append(cur.detach().clone())
        cur = layer.pgf_forward(cur)
    logits = M["pgf_lm_head"].pgf_lm_head_forward(cur.view(-1, d), lm_head_weight_pgf, bs).view(B, L, -1)
    loss, g_logits = ce_loss_and_grad(logits, targets)
    lm_res = M["pgf_lm_head"].pgf_lm_head_grad(cur.view(-1, d), g_logits.view(-1, V), lm_head_weight_pgf, bs,
                                               compute_input_grads=True)
    g = lm_res["grad_hidden"].view(B, L, -1)
    for i in reversed(range(nl)):
        layer = backbone.layers[i]
        res = layer.pgf_backward(layer_inputs.pop(), g)
        for name, param in layer.named_parameters():
            if name in res["grads"]:
                if param.grad is None:
                    param.grad = res["grads"][name].clone()
                else:
                    param.grad += res["grads"][name]
        g = res["grad_input"]
    emb_weight_pgf.grad = M["pgf_embedding"].pgf_embedding_grad(ids, g, emb_weight_pgf, bs)["grad_weight"]
    lm_head_weight_pgf.grad = lm_res["grad_W_lm_head"]
    grads = {"emb": emb_weight_pgf.grad, "lm_head": lm_head_weight_pgf.grad}
    for k, p in backbone.named_parameters():
        grads[k] = p.grad
    return loss, grads


def test_multi_layer_grads_flow_matches_reference_pgf(ref_modules):
    G = golden("multilayer.pt")
    loss, grads = _multilayer_flow(ref_modules, G, scale_reference=True)
    assert_close(loss, G["loss"], name="loss")
    assert set(grads) == set(G["grads"])
    for k, v in G["grads"].items():
        assert_close(grads[k], v, name=k)


def test_multi_layer_grads_flow_matches_reference_autograd(ref_modules):
    G = golden("multilayer.pt")
    loss, grads = _multilayer_flow(ref_modules, G, scale_reference=False)
    assert_close(loss, G["autograd"]["loss"], name="loss")
    for k, v in G["autograd"]["grads"].items():
        assert_close(grads[k], v, name="autograd " + k)


@pytest.mark.parametrize("scale_reference", [True, False])
def test_sequential_pgf_train_step_golden(ref_modules, scale_reference):
    G = golden("train_step.pt")["sequential"]
    M = ref_modules["pgf_mamba_block"]
    d = G["x"].shape[-1]
    seq = M.PGFMambaSequential([M.PGFMambaBlock(d, 16, G["d_ff"], G["block_size"]) for _ in range(G["n_layers"])])
    seq.load_state_dict(G["params"])
    seq = seq.to(DEV)
    for blk in seq.layers:
        blk.reference_scale_grad = scale_reference

    def mse(o, tg):
        diff = o - tg
        return (diff * diff).mean(), 2.0 * diff / diff.numel()

    r = seq.pgf_train_step(G["x"].to(DEV), G["target"].to(DEV), mse)
    assert_close(r["loss"], G["loss"], name="loss")
    want = G["grads"] if scale_reference else G["autograd"]["grads"]
    assert set(r["grads"]) == set(want)
    for k, v in want.items():
        assert_close(r["grads"][k], v, name=k)


@pytest.mark.parametrize("scale_reference", [True, False])
def test_single_layer_pgf_train_step_golden(ref_modules, scale_reference):
    G = golden("train_step.pt")["single"]
    T = ref_modules["train_singlemamba_optimized"]
    d = G["u"].shape[-1]
    m = T.SingleLayerMambaPGF(d, 16)
    m.load_state_dict(G["params"])
    m = m.to(DEV)
    m.reference_scale_grad = scale_reference
    opt = torch.optim.SGD(m.parameters(), lr=G["lr"])
    loss = m.pgf_train_step(G["u"].to(DEV), G["target"].to(DEV), opt, G["block_size"])
    assert isinstance(loss, float)
    assert abs(loss - G["loss"]) <= 1e-5 + 1e-4 * abs(G["loss"])
    want = G["grads"] if scale_reference else G["autograd"]["grads"]
    for k, p in m.named_parameters():
        assert_close(p.grad, want[k], name="grad " + k)
    if scale_reference:
        # the optimizer stepped with those gradients (SGD: p - lr g)
        for k, v in G["params_after"].items():
            assert_close(m.state_dict()[k], v, name="after step " + k)
