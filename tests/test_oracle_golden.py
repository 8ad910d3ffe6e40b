"""Pin the CPU oracle against golden outputs of the reference implementation (CPU only)."""
import pytest
import torch

from oracle import pgf_oracle as O
from tests.conftest import golden

TOL = dict(rtol=1e-5, atol=2e-6)


def _close(a, b, atol=2e-6, rtol=1e-5):
    assert a.shape == b.shape, (a.shape, b.shape)
    err = (a - b).abs().max().item() if a.numel() else 0.0
    lim = atol + rtol * b.abs().max().item() if b.numel() else atol
    assert err <= lim, f"max abs err {err:.3e} > {lim:.3e}"


def _ssm_params(sd, prefix=""):
    m = {"A_log": "A_log", "D": "D", "scale": "scale", "dt_w": "dt_proj.weight",
         "dt_b": "dt_proj.bias", "B_w": "B_proj.weight", "B_b": "B_proj.bias",
         "C_w": "C_proj.weight", "C_b": "C_proj.bias"}
    return {k: sd[prefix + v] for k, v in m.items()}


def test_ssm_block_grad_matches_reference():
    G = golden("ssm_block.pt")
    p = _ssm_params(G["params"])
    r = O.ssm_block_grad(p, G["u"], G["g"], G["h0"], G["delta_h_next"], G["dA_next"])
    for k, v in G["out"].items():
        _close(r[k], v, atol=5e-6)


@pytest.mark.parametrize("act", ["none", "tanh"])
def test_ssm_pgf_matches_autograd_except_reference_scale(act):
    """The oracle's PGF backward equals autograd of the reference forward on every tensor;
    the reference's own scalar scale gradient is reproduced under scale_grad='reference'."""
    G = golden("ssm_autograd.pt")[act]
    p = _ssm_params(G["params"])
    a = G["act"]
    y = O.ssm_forward_standard(p, G["u"], act=a)
    _close(y, G["y"])
    grads, gu = O.ssm_backward(p, G["u"], G["g"], block_size=16, act=a)
    _close(gu, G["grad_u"], atol=1e-5)
    names = {"A_log": "A_log", "D": "D", "scale": "scale", "dt_w": "dt_proj.weight",
             "dt_b": "dt_proj.bias", "B_w": "B_proj.weight", "B_b": "B_proj.bias",
             "C_w": "C_proj.weight", "C_b": "C_proj.bias"}
    for k, n in names.items():
        _close(grads[k], G["grads"][n], atol=2e-5, rtol=1e-4)
    gref, _ = O.ssm_backward(p, G["u"], G["g"], block_size=16, act=a, scale_grad="reference")
    assert torch.allclose(gref["scale"], gref["scale"][0].expand_as(gref["scale"]))
    _close(gref["scale"][0], grads["scale"].sum(), atol=1e-4)


@pytest.mark.parametrize("act", ["none", "tanh"])
def test_block_matches_reference_pgf(act):
    G = golden("block.pt")[act]
    bp = G["params"]
    a = G["act"]
    y = O.block_pgf_forward(bp, G["x"], G["block_size"], act=a)
    _close(y, G["y"])
    r = O.block_pgf_backward(bp, G["x"], G["g"], G["block_size"], act=a, scale_grad="reference")
    _close(r["grad_input"], G["grad_input"], atol=1e-5)
    for k, v in G["grads"].items():
        _close(r["grads"][k], v, atol=2e-5, rtol=1e-4)
    # autograd truth, incl. the per-channel scale gradient
    ra = O.block_pgf_backward(bp, G["x"], G["g"], G["block_size"], act=a)
    for k, v in G["autograd"]["grads"].items():
        _close(ra["grads"][k], v, atol=5e-5, rtol=1e-4)


def test_lm_step_matches_reference_pgf_and_autograd():
    G = golden("lm.pt")
    nl = G["n_layers"]
    blocks = [{k.split(".", 2)[2]: v for k, v in G["params"].items() if k.startswith(f"layers.{i}.")}
              for i in range(nl)]
    loss, grads = O.lm_pgf_step(G["emb"], G["lm_head"], blocks, G["ids"], G["targets"],
                                G["block_size"], scale_grad="reference")
    assert abs(loss.item() - G["loss"].item()) < 1e-5
    for k, v in G["grads"].items():
        _close(grads[k], v, atol=2e-5, rtol=1e-4)
    loss2, grads2 = O.lm_pgf_step(G["emb"], G["lm_head"], blocks, G["ids"], G["targets"],
                                  G["block_size"])
    for k, v in G["autograd"]["grads"].items():
        kk = k if k in ("emb", "lm_head") else k
        _close(grads2[kk], v, atol=5e-5, rtol=1e-4)


def test_components_match_reference():
    G = golden("components.pt")
    for eps in ("1e-06", "1e-05"):
        c = G[f"rmsnorm_{eps}"]
        _close(O.rmsnorm_forward(c["x"], c["w"], c["eps"]), c["y"])
        gw, gx = O.rmsnorm_grad(c["x"], c["g"], c["w"], c["eps"])
        _close(gw, c["grad_weight"], atol=1e-5)
        _close(gx, c["grad_x"])
    for act in ("gelu", "relu"):
        c = G[f"ffn_{act}"]
        _close(O.ffn_forward(c["x"], c["W1"], c["b1"], c["W2"], c["b2"], act), c["y"])
        r = O.ffn_grad(c["x"], c["g"], c["W1"], c["b1"], c["W2"], c["b2"], act)
        for k in ("grad_W1", "grad_b1", "grad_W2", "grad_b2", "grad_x"):
            _close(r[k], c[k], atol=1e-5)
    c = G["embedding"]
    _close(O.embedding_forward(c["ids"], c["W"]), c["y"])
    _close(O.embedding_grad(c["ids"], c["g"], c["W"]), c["grad_weight"])
    c = G["lm_head"]
    _close(O.lm_head_forward(c["h"], c["W"]), c["logits"])
    gW, gh = O.lm_head_grad(c["h"], c["g_logits"], c["W"])
    _close(gW, c["grad_W_lm_head"])
    _close(gh, c["grad_hidden"])


def test_float64_oracle_agrees_with_float32_reference():
    """The float64 run of the oracle is the high-precision truth the GPU kernels are held to;
    the reference's float32 PGF path sits within 1e-5 of it."""
    G = golden("block.pt")["none"]
    bp = {k: v.double() for k, v in G["params"].items()}
    r = O.block_pgf_backward(bp, G["x"].double(), G["g"].double(), G["block_size"], scale_grad="reference")
    for k, v in G["grads"].items():
        _close(r["grads"][k].float(), v, atol=2e-5, rtol=1e-4)


# ----------------------------------------------------------------------------- forward-mode operators
def frechet_params(sd):
    """FrechetMambaOperator state dict (pgf_mamba.py:33-49) -> the oracle's parameter dict."""
    return {"A_log": sd["A_log"], "dt_w": sd["dt_proj.weight"], "dt_b": sd["dt_proj.bias"],
            "B_w": sd["B_proj.weight"], "B_b": sd["B_proj.bias"], "C_w": sd["C_proj.weight"],
            "C_b": sd["C_proj.bias"], "D_w": sd["D"], "scale": sd["redshift_scale"],
            "init_w": sd["init_estimator.weight"], "init_b": sd["init_estimator.bias"],
            "init_window": torch.tensor(sd["init_estimator.weight"].shape[1] // sd["D"].shape[0])}


def _jclose(a, b, name=""):
    """float64 oracle vs the reference's float32 outputs: 1e-5 absolute + 1e-4 relative to max|ref|."""
    _close(a.to(b.dtype) if a.dtype != b.dtype else a, b, atol=1e-5, rtol=1e-4)


def test_jvp_oracle_matches_reference():
    from oracle import jvp_oracle as J
    G = golden("jvp.pt")
    r = G["rmsnorm"]
    y, yd = J.rmsnorm_jvp(r["x"].double(), r["x_dot"].double(), r["w"].double(), r["w_dot"].double(), r["eps"])
    _jclose(y, r["y"], name="rmsnorm y")
    _jclose(yd, r["y_dot"], name="rmsnorm y_dot")
    for act in ("gelu", "relu"):
        f = {k: v.double() if torch.is_tensor(v) else v for k, v in G[f"ffn_{act}"].items()}
        y, yd = J.ffn_jvp(f["x"], f["x_dot"], f["W1"], f["W1_dot"], f["b1"], f["b1_dot"], f["W2"], f["W2_dot"],
                          f["b2"], f["b2_dot"], act)
        _jclose(y, G[f"ffn_{act}"]["y"], name=f"ffn {act} y")
        _jclose(yd, G[f"ffn_{act}"]["y_dot"], name=f"ffn {act} y_dot")
    for name in ("frechet", "frechet_short"):
        c = G[name]
        p = {k: v.double() for k, v in frechet_params(c["params"]).items()}
        y, yd, _, _ = J.frechet_jvp(p, c["u"].double(), c["du"].double())
        _jclose(y, c["y"], name=f"{name} y")
        _jclose(yd, c["y_dot"], name=f"{name} y_dot")
        _jclose(y, c["y_standard"], name=f"{name} y vs forward()")
        for s, e, ys, yds in c["stream"]:   # the streamed blocks carry the same values
            assert abs(float(y[s:e].sum()) - ys) <= 1e-5 * max(1.0, abs(ys))
            assert abs(float(yd[s:e].sum()) - yds) <= 1e-4 * max(1.0, abs(yds))


def test_state_hvp_oracle_matches_reference():
    G = golden("hvp.pt")
    for act, c in G.items():
        p = {k: v.double() for k, v in _ssm_params(c["params"]).items()}
        z = O.ssm_state_hvp(p, c["u"].double(), c["target"].double(), c["v_h"].double(), c["act"])
        _close(z.to(c["hvp"].dtype), c["hvp"], atol=1e-7, rtol=1e-4)
