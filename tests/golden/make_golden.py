"""Generate the golden fixtures in this folder from the reference implementation itself.

Run where a checkout of the reference (zhry915/icml, pure Python) is readable; its directory is
a required argument:

    python tests/golden/make_golden.py REF_DIR          # every fixture
    python tests/golden/make_golden.py REF_DIR jvp      # jvp.pt only
    python tests/golden/make_golden.py REF_DIR hvp      # hvp.pt only

The reference is imported as-is with two adjustments, both applied from the outside:
* ``TORCHDYNAMO_DISABLE=1`` so ``pgf_lm_head``'s ``torch.compile`` wrapper runs eagerly on the CPU;
* ``pgf_ffn._process_single_block_grad`` is replaced by the same computation with the missing
  ``grad_W1 = grad_z^T @ x`` line (pgf_ffn.py:101-117 returns an undefined name as shipped).

Everything else (SSM scan, PGF block forward/backward, RMSNorm, embedding, LM head, the CE
gradient of test_multi_layer_grads.py:74-86) is the reference's own code.  Outputs are small
float32 tensors saved with ``torch.save``; the tests never read the reference at run time.
"""
from __future__ import annotations

import os
import sys

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(path):
    sys.path.insert(0, path)
    import pgf_ffn  # noqa: F401
    import pgf_rmsnorm  # noqa: F401
    import pgf_embedding  # noqa: F401
    import pgf_lm_head  # noqa: F401
    import train_singlemamba_optimized as tso  # noqa: F401
    import pgf_mamba_block  # noqa: F401
    import pgf_mamba  # noqa: F401

    def fixed_block_grad(x_block, g_out_block, W1, b1, W2, b2, activation="gelu", comp_dtype=None):
        if comp_dtype is not None:
            x_block, g_out_block = x_block.to(comp_dtype), g_out_block.to(comp_dtype)
            W1, W2, b1 = W1.to(comp_dtype), W2.to(comp_dtype), b1.to(comp_dtype)
        z = torch.matmul(x_block, W1.t()) + b1
        if activation == "gelu":
            h, hp = pgf_ffn._gelu_jit(z), pgf_ffn._gelu_prime_jit(z)
        elif activation == "relu":
            h, hp = F.relu(z), pgf_ffn._relu_prime_jit(z)
        else:
            raise ValueError(activation)
        gW2 = torch.matmul(g_out_block.t(), h)
        gb2 = g_out_block.sum(dim=0)
        gz = torch.matmul(g_out_block, W2) * hp
        gW1 = torch.matmul(gz.t(), x_block)
        gb1 = gz.sum(dim=0)
        gx = torch.matmul(gz, W1)
        return gW1, gb1, gW2, gb2, gx

    pgf_ffn._process_single_block_grad = fixed_block_grad
    return {
        "ffn": pgf_ffn, "rms": pgf_rmsnorm, "emb": pgf_embedding, "lm": pgf_lm_head,
        "tso": tso, "blk": pgf_mamba_block, "mamba": pgf_mamba,
    }


def _sd(module):
    return {k: v.detach().clone() for k, v in module.state_dict().items()}


def gen_ssm_block(R):
    """One call of SingleLayerMambaPGF._pass2_block_direct_grad (train_singlemamba_optimized.py:350-472)."""
    torch.manual_seed(11)
    B, L, d, N = 2, 48, 32, 16
    m = R["tso"].SingleLayerMambaPGF(d, N)
    u = torch.randn(B, L, d)
    g = torch.randn(B, L, d)
    h0 = torch.randn(B, d, N) * 0.5
    dh_next = torch.randn(B, d, N) * 0.3
    dA_next = torch.rand(B, d, N) * 0.5 + 0.5
    with torch.no_grad():
        out = m._pass2_block_direct_grad(u, g, h0, dh_next, dA_next)
    names = ["A_log", "D", "scale_ref", "dt_w", "dt_b", "B_w", "B_b", "C_w", "C_b",
             "delta_h0", "dA0", "grad_u"]
    return {"params": _sd(m), "u": u, "g": g, "h0": h0, "delta_h_next": dh_next, "dA_next": dA_next,
            "out": {k: v.detach().clone() for k, v in zip(names, out)}}


def gen_ssm_autograd(R, act=None):
    """forward_standard + autograd (train_singlemamba_optimized.py:731-765): truth for mamba.scale."""
    torch.manual_seed(12)
    B, L, d, N = 2, 40, 24, 16
    m = R["tso"].SingleLayerMambaPGF(d, N, output_activation=act)
    with torch.no_grad():
        m.scale.mul_(torch.rand(d) + 0.5)
        m.D.mul_(torch.rand(d) + 0.5)
    u = torch.randn(B, L, d, requires_grad=True)
    g = torch.randn(B, L, d)
    y = m.forward_standard(u)
    y.backward(g)
    return {"params": {k: v.detach().clone() for k, v in _sd(m).items()}, "u": u.detach().clone(),
            "g": g, "act": act, "y": y.detach().clone(), "grad_u": u.grad.detach().clone(),
            "grads": {k: p.grad.detach().clone() for k, p in m.named_parameters()}}


def gen_block(R, act=None, seed=21):
    """PGFMambaBlock.pgf_forward / pgf_backward (pgf_mamba_block.py:70-249) and its autograd twin."""
    torch.manual_seed(seed)
    B, L, d, N, dff, bs = 2, 80, 32, 16, 64, 32
    blk = R["blk"].PGFMambaBlock(d, N, dff, bs, output_activation=act)
    with torch.no_grad():
        blk.norm1.weight.mul_(1 + 0.1 * torch.randn(d))
        blk.norm2.weight.mul_(1 + 0.1 * torch.randn(d))
        blk.b1.normal_(0, 0.05)
        blk.b2.normal_(0, 0.05)
    x = torch.randn(B, L, d)
    g = torch.randn(B, L, d)
    y = blk.pgf_forward(x)
    res = blk.pgf_backward(x, g)
    xa = x.clone().requires_grad_(True)
    ya = blk.forward(xa)
    ya.backward(g)
    return {"params": _sd(blk), "x": x, "g": g, "act": act, "block_size": bs, "d_ff": dff,
            "y": y, "grads": {k: v.clone() for k, v in res["grads"].items()},
            "grad_input": res["grad_input"].clone(),
            "autograd": {"y": ya.detach().clone(), "grad_input": xa.grad.detach().clone(),
                         "grads": {k: p.grad.detach().clone() for k, p in blk.named_parameters()}}}


def gen_lm(R):
    """The reference's PGF LM step (test_multi_layer_grads.py:88-126) and autograd (:57-68)."""
    torch.manual_seed(1)
    B, L, d, N, dff, bs, V, nl = 2, 96, 32, 16, 64, 32, 128, 2
    ids = torch.randint(0, V, (B, L))
    tg = torch.randint(0, V, (B, L))
    emb = torch.randn(V, d)
    lmw = torch.randn(V, d) * 0.2
    blocks = [R["blk"].PGFMambaBlock(d, N, dff, bs) for _ in range(nl)]
    seq = R["blk"].PGFMambaSequential(blocks)
    params = {k: v.detach().clone() for k, v in seq.state_dict().items()}
    # PGF path
    h = R["emb"].pgf_embedding_forward(ids, emb, bs)
    inputs, cur = [], h
    for layer in seq.layers:
        inputs.append(cur.detach().clone())
        cur = layer.pgf_forward(cur)
    logits = R["lm"].pgf_lm_head_forward(cur.view(-1, d), lmw, bs)
    lf = logits.view(-1, V)
    loss = F.cross_entropy(lf, tg.view(-1))
    probs = F.softmax(lf, dim=-1)
    gl = probs.clone()
    gl[torch.arange(gl.size(0)), tg.view(-1)] -= 1.0
    gl /= lf.size(0)
    lres = R["lm"].pgf_lm_head_grad(cur.view(-1, d), gl, lmw, bs, compute_input_grads=True)
    g = lres["grad_hidden"].view(B, L, d)
    grads = {"lm_head": lres["grad_W_lm_head"].clone()}
    for i in reversed(range(nl)):
        r = seq.layers[i].pgf_backward(inputs[i], g)
        for k, v in r["grads"].items():
            grads[f"layers.{i}.{k}"] = v.clone()
        g = r["grad_input"]
    grads["emb"] = R["emb"].pgf_embedding_grad(ids, g, emb, bs)["grad_weight"].clone()
    # autograd path
    emb_a = emb.clone().requires_grad_(True)
    lm_a = lmw.clone().requires_grad_(True)
    x = F.embedding(ids, emb_a)
    for layer in seq.layers:
        x = layer.forward(x)
    la = F.cross_entropy((x @ lm_a.t()).view(-1, V), tg.view(-1))
    la.backward()
    ag = {"emb": emb_a.grad.clone(), "lm_head": lm_a.grad.clone()}
    for k, p in seq.named_parameters():
        ag[k] = p.grad.clone()
    return {"ids": ids, "targets": tg, "emb": emb, "lm_head": lmw, "params": params, "n_layers": nl,
            "block_size": bs, "d_ff": dff, "loss": loss.detach(), "grads": grads,
            "autograd": {"loss": la.detach(), "grads": ag}}


def gen_components(R):
    torch.manual_seed(31)
    out = {}
    # RMSNorm (pgf_rmsnorm.py:75-214), ragged token blocks
    for eps in (1e-6, 1e-5):
        n = R["rms"].RMSNorm(48, eps=eps)
        with torch.no_grad():
            n.weight.copy_(1 + 0.02 * torch.randn(48))
        x = torch.randn(3, 40, 48)
        g = torch.randn(3, 40, 48)
        y = n.pgf_forward(x, block_size=37)
        r = n.pgf_grad(x, g, block_size=37, compute_input_grads=True)
        out[f"rmsnorm_{eps:g}"] = {"x": x, "g": g, "w": n.weight.detach().clone(), "eps": eps, "y": y,
                                   "grad_weight": r["grad_weight"], "grad_x": r["grad_x"]}
    # FFN (pgf_ffn.py:183-307)
    for act in ("gelu", "relu"):
        x = torch.randn(70, 24)
        g = torch.randn(70, 24)
        W1 = torch.randn(64, 24) * 0.2
        b1 = torch.randn(64) * 0.1
        W2 = torch.randn(24, 64) * 0.2
        b2 = torch.randn(24) * 0.1
        y = R["ffn"].pgf_ffn_forward(x, W1, b1, W2, b2, block_size=32, activation=act)
        r = R["ffn"].pgf_ffn_grad(x, g, W1, b1, W2, b2, block_size=32, activation=act,
                                  compute_input_grads=True)
        out[f"ffn_{act}"] = {"x": x, "g": g, "W1": W1, "b1": b1, "W2": W2, "b2": b2, "y": y,
                             **{k: v.clone() for k, v in r.items()}}
    # Embedding (pgf_embedding.py), with repeated ids
    ids = torch.randint(0, 30, (2, 50))
    W = torch.randn(30, 24)
    g = torch.randn(2, 50, 24)
    out["embedding"] = {"ids": ids, "W": W, "g": g,
                        "y": R["emb"].pgf_embedding_forward(ids, W, block_size=16),
                        "grad_weight": R["emb"].pgf_embedding_grad(ids, g, W, block_size=16)["grad_weight"]}
    # LM head (pgf_lm_head.py)
    h = torch.randn(50, 24)
    W = torch.randn(40, 24) * 0.3
    gl = torch.randn(50, 40) * 0.1
    r = R["lm"].pgf_lm_head_grad(h, gl, W, block_size=16, compute_input_grads=True)
    out["lm_head"] = {"h": h, "W": W, "g_logits": gl,
                      "logits": R["lm"].pgf_lm_head_forward(h, W, block_size=16),
                      "grad_W_lm_head": r["grad_W_lm_head"], "grad_hidden": r["grad_hidden"]}
    return out


def gen_init(R):
    """Freshly constructed modules under fixed seeds: the initial weights a drop-in must reproduce
    (pgf_mamba_block.py:21-49, train_singlemamba_optimized.py:89-101, pgf_rmsnorm.py:77-81)."""
    out = {}
    torch.manual_seed(5)
    out["block"] = _sd(R["blk"].PGFMambaBlock(32, 16, 64, 32))
    torch.manual_seed(6)
    out["ssm"] = _sd(R["tso"].SingleLayerMambaPGF(24, 16))
    return out


def gen_jvp(R):
    """The forward-mode operators: RMSNorm.pgf_jvp (pgf_rmsnorm.py:119-155), pgf_ffn_jvp
    (pgf_ffn.py:146-180) and FrechetMambaOperator.pgf_forward (pgf_mamba.py:69-139), blocked and
    streamed as the reference runs them."""
    out = {}
    g = torch.Generator().manual_seed(31)
    x = torch.randn(3, 40, 48, generator=g)
    xd = torch.randn(3, 40, 48, generator=g)
    wd = 0.1 * torch.randn(48, generator=g)
    torch.manual_seed(32)
    norm = R["rms"].RMSNorm(48)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.05 * torch.randn(48, generator=g))
    y, yd = norm.pgf_jvp(x, xd, wd, block_size=16)
    out["rmsnorm"] = {"x": x, "x_dot": xd, "w": norm.weight.detach().clone(), "w_dot": wd, "eps": norm.eps,
                      "y": y, "y_dot": yd}
    for act in ("gelu", "relu"):
        t = {k: torch.randn(*s, generator=g) * sc for k, s, sc in (
            ("x", (100, 24), 1.0), ("x_dot", (100, 24), 1.0), ("W1", (64, 24), 0.2), ("W1_dot", (64, 24), 0.05),
            ("b1", (64,), 0.1), ("b1_dot", (64,), 0.05), ("W2", (24, 64), 0.2), ("W2_dot", (24, 64), 0.05),
            ("b2", (24,), 0.1), ("b2_dot", (24,), 0.05))}
        y, yd = R["ffn"].pgf_ffn_jvp(t["x"], t["x_dot"], t["W1"], t["W1_dot"], t["b1"], t["b1_dot"], t["W2"],
                                     t["W2_dot"], t["b2"], t["b2_dot"], block_size=32, activation=act)
        out[f"ffn_{act}"] = dict(t, y=y, y_dot=yd)
    for name, L, D in (("frechet", 150, 32), ("frechet_short", 2, 16)):
        torch.manual_seed(33)
        m = R["mamba"].FrechetMambaOperator(d_model=D, d_state=16)
        u = 0.5 * torch.randn(L, D, generator=g)
        du = torch.randn(L, D, generator=g)
        y, yd = m.pgf_forward(u, du, block_size=64)
        blocks = []
        m.pgf_forward(u, du, block_size=64, streaming=True,
                      callback=lambda a, b, s, e: blocks.append((s, e, float(a.sum()), float(b.sum()))))
        out[name] = {"params": _sd(m), "u": u, "du": du, "y": y, "y_dot": yd, "stream": blocks,
                     "y_standard": m.forward(u).detach()}
    return out


def gen_hvp(R):
    """SingleLayerMambaPGF.compute_state_hvp (train_singlemamba_optimized.py:563-685), blocked as the
    reference runs it, with no output activation and with tanh and relu."""
    out = {}
    for act, seed in ((None, 41), ("tanh", 42), ("relu", 43)):
        torch.manual_seed(seed)
        B, L, d, N = 2, 100, 16, 16
        m = R["tso"].SingleLayerMambaPGF(d, N, output_activation=act)
        with torch.no_grad():
            m.scale.mul_(torch.rand(d) + 0.5)
            m.D.mul_(torch.rand(d) + 0.5)
        u = torch.randn(B, L, d)
        target = torch.randn(B, L, d)
        v_h = torch.randn(B, d, N)
        hvp = m.compute_state_hvp(u, target, v_h, block_size=32)
        out[str(act)] = {"params": {k: v.detach().clone() for k, v in _sd(m).items()}, "u": u, "target": target,
                         "v_h": v_h, "act": act, "block_size": 32, "hvp": hvp.detach().clone()}
    return out


def gen_multilayer(R, n_layers=2):
    """test_multi_layer_grads.py:10-126 as the reference runs it (seed 1, B=2, L=512, d_model=64,
    d_state=16, d_ff=128, block_size=128, vocab 1000), at its smallest layer count, on the CPU: the
    weights, the PGF gradients of every parameter and the autograd gradients."""
    torch.manual_seed(1)
    B, L, d, N, dff, bs, V = 2, 512, 64, 16, 128, 128, 1000
    ids = torch.randint(0, V, (B, L))
    tg = torch.randint(0, V, (B, L))
    emb = torch.randn(V, d)
    lmw = torch.randn(V, d)
    seq = R["blk"].PGFMambaSequential([R["blk"].PGFMambaBlock(d, N, dff, bs) for _ in range(n_layers)])
    params = _sd(seq)
    # PGF path (:89-126)
    h = R["emb"].pgf_embedding_forward(ids, emb, bs)
    inputs, cur = [], h
    for layer in seq.layers:
        inputs.append(cur.detach().clone())
        cur = layer.pgf_forward(cur)
    lf = R["lm"].pgf_lm_head_forward(cur.view(-1, d), lmw, bs).view(-1, V)
    loss = F.cross_entropy(lf, tg.view(-1))
    gl = F.softmax(lf, dim=-1).clone()
    gl[torch.arange(gl.size(0)), tg.view(-1)] -= 1.0
    gl /= lf.size(0)
    lres = R["lm"].pgf_lm_head_grad(cur.view(-1, d), gl, lmw, bs, compute_input_grads=True)
    g = lres["grad_hidden"].view(B, L, d)
    grads = {"lm_head": lres["grad_W_lm_head"].clone()}
    for i in reversed(range(n_layers)):
        r = seq.layers[i].pgf_backward(inputs[i], g)
        for k, v in r["grads"].items():
            grads[f"layers.{i}.{k}"] = v.clone()
        g = r["grad_input"]
    grads["emb"] = R["emb"].pgf_embedding_grad(ids, g, emb, bs)["grad_weight"].clone()
    # autograd path (:57-68)
    emb_a = emb.clone().requires_grad_(True)
    lm_a = lmw.clone().requires_grad_(True)
    x = F.embedding(ids, emb_a)
    for layer in seq.layers:
        x = layer.forward(x)
    la = F.cross_entropy((x @ lm_a.t()).view(-1, V), tg.view(-1))
    la.backward()
    ag = {"emb": emb_a.grad.clone(), "lm_head": lm_a.grad.clone()}
    for k, p in seq.named_parameters():
        ag[k] = p.grad.clone()
    return {"ids": ids, "targets": tg, "emb": emb, "lm_head": lmw, "params": params, "n_layers": n_layers,
            "d_ff": dff, "block_size": bs, "loss": loss.detach(), "grads": grads,
            "autograd": {"loss": la.detach(), "grads": ag}}


def gen_train_steps(R):
    """SingleLayerMambaPGF.pgf_train_step (train_singlemamba_optimized.py:474-561: MSE target, two
    block passes, writes .grad, steps the optimizer) and PGFMambaSequential.pgf_train_step
    (pgf_mamba_block.py:290-322) with an MSE loss_fn, plus autograd of the same losses."""
    out = {}
    torch.manual_seed(51)
    B, L, d, N, bs, lr = 2, 72, 24, 16, 32, 0.05
    m = R["tso"].SingleLayerMambaPGF(d, N)
    with torch.no_grad():
        m.scale.mul_(torch.rand(d) + 0.5)
        m.D.mul_(torch.rand(d) + 0.5)
    u = torch.randn(B, L, d)
    target = torch.randn(B, L, d)
    p0 = _sd(m)
    # autograd of the same MSE loss through forward_standard (the truth for the per-channel scale)
    ua = u.clone()
    ya = m.forward_standard(ua)
    la = ((ya - target) ** 2).mean()
    la.backward()
    ag = {k: p.grad.detach().clone() for k, p in m.named_parameters()}
    m.zero_grad(set_to_none=True)
    opt = torch.optim.SGD(m.parameters(), lr=lr)
    loss = m.pgf_train_step(u, target, opt, bs)
    out["single"] = {"params": p0, "u": u, "target": target, "block_size": bs, "lr": lr, "loss": loss,
                     "grads": {k: p.grad.detach().clone() for k, p in m.named_parameters()},
                     "params_after": _sd(m), "autograd": {"loss": la.detach(), "grads": ag}}
    torch.manual_seed(52)
    B, L, d, N, dff, bs, nl = 2, 80, 32, 16, 64, 32, 3
    seq = R["blk"].PGFMambaSequential([R["blk"].PGFMambaBlock(d, N, dff, bs) for _ in range(nl)])
    x = torch.randn(B, L, d)
    target = torch.randn(B, L, d)

    def mse(o, tg):
        diff = o - tg
        return (diff * diff).mean(), 2.0 * diff / diff.numel()

    p0 = _sd(seq)
    r = seq.pgf_train_step(x, target, mse)
    xa = x.clone().requires_grad_(True)
    la = ((seq(xa) - target) ** 2).mean()
    la.backward()
    out["sequential"] = {"params": p0, "x": x, "target": target, "n_layers": nl, "d_ff": dff, "block_size": bs,
                         "loss": r["loss"].detach().clone(),
                         "grads": {k: v.detach().clone() for k, v in r["grads"].items()},
                         "autograd": {"loss": la.detach(),
                                      "grads": {k: p.grad.detach().clone() for k, p in seq.named_parameters()}}}
    return out


def main(ref_path, only=None):
    R = _import_reference(ref_path)
    torch.set_num_threads(1)
    if only == "jvp":
        torch.save(gen_jvp(R), os.path.join(HERE, "jvp.pt"))
        print("golden fixture jvp.pt written to", HERE)
        return
    if only == "hvp":
        torch.save(gen_hvp(R), os.path.join(HERE, "hvp.pt"))
        print("golden fixture hvp.pt written to", HERE)
        return
    if only == "train_step":
        torch.save(gen_train_steps(R), os.path.join(HERE, "train_step.pt"))
        torch.save(gen_multilayer(R), os.path.join(HERE, "multilayer.pt"))
        print("golden fixtures train_step.pt and multilayer.pt written to", HERE)
        return
    torch.save(gen_ssm_block(R), os.path.join(HERE, "ssm_block.pt"))
    torch.save({"none": gen_ssm_autograd(R, None), "tanh": gen_ssm_autograd(R, "tanh")},
               os.path.join(HERE, "ssm_autograd.pt"))
    torch.save({"none": gen_block(R, None), "tanh": gen_block(R, "tanh", seed=22)},
               os.path.join(HERE, "block.pt"))
    torch.save(gen_lm(R), os.path.join(HERE, "lm.pt"))
    torch.save(gen_components(R), os.path.join(HERE, "components.pt"))
    torch.save(gen_init(R), os.path.join(HERE, "init.pt"))
    torch.save(gen_jvp(R), os.path.join(HERE, "jvp.pt"))
    torch.save(gen_hvp(R), os.path.join(HERE, "hvp.pt"))
    torch.save(gen_train_steps(R), os.path.join(HERE, "train_step.pt"))
    torch.save(gen_multilayer(R), os.path.join(HERE, "multilayer.pt"))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py REF_DIR [jvp|hvp|train_step]")
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else None)
