"""Forward-mode operators and the state HVP on the GPU: RMSNorm.pgf_jvp, pgf_ffn_jvp, the Frechet
operator's pgf_forward and SingleLayerMambaPGF.compute_state_hvp against the reference's own outputs
(tests/golden/jvp.pt, hvp.pt) and the float64 oracle."""
import pytest
import torch

from oracle import jvp_oracle as J
from tests.conftest import golden
from tests.parity import BF16_RTOL, assert_close, rel_err
from tests.test_oracle_golden import frechet_params

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _gen(seed):
    return torch.Generator().manual_seed(seed)


# ----------------------------------------------------------------------------- RMSNorm
def test_rmsnorm_jvp_golden():
    from icml_b200.pgf_rmsnorm import RMSNorm
    r = golden("jvp.pt")["rmsnorm"]
    norm = RMSNorm(48, eps=r["eps"]).to(DEV)
    with torch.no_grad():
        norm.weight.copy_(r["w"])
    y, yd = norm.pgf_jvp(r["x"].to(DEV), r["x_dot"].to(DEV), r["w_dot"].to(DEV), block_size=16)
    assert_close(y, r["y"], name="y")
    assert_close(yd, r["y_dot"], name="y_dot")


@pytest.mark.parametrize("rows,dim", [(1000, 256), (7, 1024), (33, 100)])
def test_rmsnorm_jvp_f64(rows, dim):
    from icml_b200 import ops
    g = _gen(rows + dim)
    x, xd = torch.randn(rows, dim, generator=g), torch.randn(rows, dim, generator=g)
    w, wd = 1 + 0.1 * torch.randn(dim, generator=g), 0.1 * torch.randn(dim, generator=g)
    y, yd = ops.rmsnorm_jvp(x.to(DEV), xd.to(DEV), w.to(DEV), wd.to(DEV), 1e-6)
    ry, ryd = J.rmsnorm_jvp(x.double(), xd.double(), w.double(), wd.double(), 1e-6)
    assert_close(y, ry, name="y")
    assert_close(yd, ryd, name="y_dot")
    yb, ydb = ops.rmsnorm_jvp(x.bfloat16().to(DEV), xd.bfloat16().to(DEV), w.to(DEV), wd.to(DEV), 1e-6)
    ry, ryd = J.rmsnorm_jvp(x.bfloat16().double(), xd.bfloat16().double(), w.double(), wd.double(), 1e-6)
    assert rel_err(yb, ry) < BF16_RTOL and rel_err(ydb, ryd) < BF16_RTOL


# ----------------------------------------------------------------------------- FFN
@pytest.mark.parametrize("act", ["gelu", "relu"])
def test_ffn_jvp_golden(act):
    from icml_b200.pgf_ffn import pgf_ffn_jvp
    f = golden("jvp.pt")[f"ffn_{act}"]
    t = {k: v.to(DEV) for k, v in f.items() if k not in ("y", "y_dot")}
    y, yd = pgf_ffn_jvp(t["x"], t["x_dot"], t["W1"], t["W1_dot"], t["b1"], t["b1_dot"], t["W2"], t["W2_dot"],
                        t["b2"], t["b2_dot"], block_size=32, activation=act)
    assert_close(y, f["y"], name="y")
    assert_close(yd, f["y_dot"], name="y_dot")


@pytest.mark.parametrize("rows,d_in,d_h", [(4096, 256, 1024), (300, 64, 256), (50, 24, 40)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_ffn_jvp_f64(rows, d_in, d_h, dtype):
    """Tensor-core path (bf16, widths that suit it), SIMT path (float32, and narrow widths)."""
    from icml_b200 import ops
    g = _gen(rows + d_h)
    sh = {"x": (rows, d_in), "x_dot": (rows, d_in), "W1": (d_h, d_in), "W1_dot": (d_h, d_in), "b1": (d_h,),
          "b1_dot": (d_h,), "W2": (d_in, d_h), "W2_dot": (d_in, d_h), "b2": (d_in,), "b2_dot": (d_in,)}
    t = {k: torch.randn(*v, generator=g) * (1.0 if k.startswith("x") else 0.1) for k, v in sh.items()}
    xs = {k: (t[k].to(dtype) if k.startswith("x") else t[k]) for k in t}
    y, yd = ops.ffn_jvp(*(xs[k].to(DEV) for k in sh))
    ref = {k: xs[k].double() if k.startswith("x") else
           (t[k].bfloat16().double() if dtype == torch.bfloat16 else t[k].double()) for k in t}
    ry, ryd = J.ffn_jvp(*(ref[k] for k in sh))
    if dtype == torch.float32:
        assert_close(y, ry, name="y")
        assert_close(yd, ryd, name="y_dot")
    else:
        assert rel_err(y, ry) < BF16_RTOL, rel_err(y, ry)
        assert rel_err(yd, ryd) < BF16_RTOL, rel_err(yd, ryd)


# ----------------------------------------------------------------------------- Frechet operator
def _operator(name):
    from icml_b200.pgf_mamba import FrechetMambaOperator
    c = golden("jvp.pt")[name]
    D = c["params"]["D"].shape[0]
    m = FrechetMambaOperator(d_model=D, d_state=16)
    m.load_state_dict(c["params"])
    return m.to(DEV), c


@pytest.mark.parametrize("name", ["frechet", "frechet_short"])
def test_frechet_jvp_golden(name):
    m, c = _operator(name)
    u, du = c["u"].to(DEV), c["du"].to(DEV)
    y, yd = m.pgf_forward(u, du, block_size=64)
    assert_close(y, c["y"], name="y")
    assert_close(yd, c["y_dot"], name="y_dot")
    assert_close(m.forward(u), c["y_standard"], name="forward")
    blocks = []
    assert m.pgf_forward(u, du, block_size=64, streaming=True,
                         callback=lambda a, b, s, e: blocks.append((s, e, float(a.sum()), float(b.sum())))) is None
    assert [(s, e) for s, e, _, _ in blocks] == [(s, e) for s, e, _, _ in c["stream"]]
    for (_, _, ys, yds), (_, _, rs, rds) in zip(blocks, c["stream"]):
        assert abs(ys - rs) <= 1e-5 * max(1.0, abs(rs)) and abs(yds - rds) <= 1e-4 * max(1.0, abs(rds))


@pytest.mark.parametrize("L,D", [(5000, 64), (1537, 256), (3, 32)])
def test_frechet_jvp_f64(L, D):
    """Many chunks (the chunk pass, compose and output pass), a ragged last chunk, and L at the
    estimator window, against the float64 token-by-token oracle."""
    from icml_b200.pgf_mamba import FrechetMambaOperator
    torch.manual_seed(L)
    m = FrechetMambaOperator(d_model=D, d_state=16)
    g = _gen(D)
    u = 0.3 * torch.randn(L, D, generator=g)
    du = torch.randn(L, D, generator=g)
    y, yd = m.to(DEV).pgf_forward(u.to(DEV), du.to(DEV))
    p = {k: v.double() for k, v in frechet_params({k: v.detach().cpu() for k, v in m.state_dict().items()}).items()}
    ry, ryd, _, _ = J.frechet_jvp(p, u.double(), du.double())
    assert_close(y, ry, name="y")
    assert_close(yd, ryd, name="y_dot")


def test_frechet_jvp_end_state_and_linearity():
    """The returned end pair matches the oracle's, and y_dot is linear in the direction."""
    from icml_b200 import ops
    from icml_b200.pgf_mamba import FrechetMambaOperator
    torch.manual_seed(4)
    m = FrechetMambaOperator(d_model=64, d_state=16).to(DEV)
    g = _gen(5)
    u = (0.3 * torch.randn(700, 64, generator=g)).to(DEV)
    d1, d2 = torch.randn(700, 64, generator=g).to(DEV), torch.randn(700, 64, generator=g).to(DEV)
    W, b = m._cat()
    h0 = (0.1 * torch.randn(64, 16, generator=g)).to(DEV)
    hd = (0.1 * torch.randn(64, 16, generator=g)).to(DEV)
    y, yd, he, hde = ops.frechet_jvp(u, d1, W, b, m.A_log, m.D, m.redshift_scale, h0, hd, want_state=True)
    p = {k: v.double() for k, v in frechet_params({k: v.detach().cpu() for k, v in m.state_dict().items()}).items()}
    ry, ryd, rh, rhd = J.frechet_jvp(p, u.cpu().double(), d1.cpu().double(), h0.cpu().double(), hd.cpu().double())
    assert_close(he, rh, name="h_end")
    assert_close(hde, rhd, name="h_end_dot")
    _, ya = ops.frechet_jvp(u, d1, W, b, m.A_log, m.D, m.redshift_scale)
    _, yb = ops.frechet_jvp(u, d2, W, b, m.A_log, m.D, m.redshift_scale)
    _, yab = ops.frechet_jvp(u, 2 * d1 - 3 * d2, W, b, m.A_log, m.D, m.redshift_scale)
    assert_close(yab, 2 * ya - 3 * yb, atol=1e-4, name="linearity")


# ----------------------------------------------------------------------------- state HVP
def _ssm_layer(c):
    from icml_b200.train_singlemamba_optimized import SingleLayerMambaPGF
    d = c["params"]["D"].shape[0]
    m = SingleLayerMambaPGF(d, 16, output_activation=c["act"])
    m.load_state_dict(c["params"])
    return m.to(DEV)


@pytest.mark.parametrize("act", ["None", "tanh", "relu"])
def test_state_hvp_golden(act):
    c = golden("hvp.pt")[act]
    m = _ssm_layer(c)
    z = m.compute_state_hvp(c["u"].to(DEV), c["target"].to(DEV), c["v_h"].to(DEV), c["block_size"])
    assert z.shape == c["hvp"].shape
    assert_close(z, c["hvp"], atol=1e-7, name="hvp")


@pytest.mark.parametrize("act", [None, "tanh"])
@pytest.mark.parametrize("B,L,d", [(2, 1000, 64), (1, 4099, 32), (3, 7, 16)])
def test_state_hvp_f64(act, B, L, d):
    """Many chunks (prefix of dt over chunks, reverse compose) and ragged / single-chunk lengths."""
    from oracle import pgf_oracle as O
    from icml_b200.train_singlemamba_optimized import SingleLayerMambaPGF
    torch.manual_seed(L + d)
    m = SingleLayerMambaPGF(d, 16, output_activation=act)
    g = _gen(L)
    with torch.no_grad():
        m.scale.mul_(0.5 + torch.rand(d, generator=g))
    u = torch.randn(B, L, d, generator=g)
    tg = torch.randn(B, L, d, generator=g)
    v = torch.randn(B, d, 16, generator=g)
    z = m.to(DEV).compute_state_hvp(u.to(DEV), tg.to(DEV), v.to(DEV), 64)
    p = {k: getattr(m, k).detach().cpu().double() for k in ("A_log", "D", "scale")}
    p.update({"dt_w": m.dt_proj.weight, "dt_b": m.dt_proj.bias, "B_w": m.B_proj.weight, "B_b": m.B_proj.bias,
              "C_w": m.C_proj.weight, "C_b": m.C_proj.bias})
    p = {k: v_.detach().cpu().double() for k, v_ in p.items()}
    ref = O.ssm_state_hvp(p, u.double(), tg.double(), v.double(), act)
    assert_close(z, ref, atol=1e-9, rtol=1e-4, name="hvp")
