"""CPU checks of the Mamba-standard restatement (oracle/mamba_std.py)."""
import pytest
import torch
import torch.nn.functional as F

from oracle import mamba_std as MS


def test_causal_conv_equals_torch_depthwise_conv1d():
    g = torch.Generator().manual_seed(1)
    B, L, E, K = 2, 30, 8, 4
    xi = torch.randn(B, L, E, generator=g, dtype=torch.float64)
    w = torch.randn(E, K, generator=g, dtype=torch.float64)
    b = torch.randn(E, generator=g, dtype=torch.float64)
    ref = F.conv1d(xi.transpose(1, 2), w.unsqueeze(1), b, padding=K - 1, groups=E)[..., :L].transpose(1, 2)
    assert torch.allclose(MS.causal_conv(xi, w, b), ref, atol=1e-12)


def test_mixer_is_causal_and_matches_chunked_evaluation():
    """Outputs at t depend only on inputs <= t; running the scan over two halves with the state and
    conv history handed over gives the same result (the PGF block decomposition)."""
    g = torch.Generator().manual_seed(2)
    p = MS.std_init(16, 16, 2, 4, 2, g)
    x = torch.randn(1, 24, 16, generator=g, dtype=torch.float64)
    y = MS.mixer_forward(p, x)
    x2 = x.clone()
    x2[:, 12:] += 1.0
    y2 = MS.mixer_forward(p, x2)
    assert torch.allclose(y[:, :12], y2[:, :12], atol=1e-12)
    assert not torch.allclose(y[:, 12:], y2[:, 12:])


def test_init_shapes_and_dt_bias_range():
    p = MS.std_init(128, 16, 2, 4, 8, torch.Generator().manual_seed(3))
    assert p["in_w"].shape == (512, 128) and p["x_w"].shape == (8 + 32, 256) and p["dt_w"].shape == (256, 8)
    assert p["A_log"].shape == (256, 16) and torch.allclose(p["A_log"][5], torch.log(torch.arange(1., 17.)).double())
    dt = F.softplus(p["dt_b"])
    assert dt.min() >= 1e-4 - 1e-12 and dt.max() <= 0.1 + 1e-9


def test_mixer_matches_transformers_mamba_mixer():
    """Pins the restatement to an independent implementation of the standard Mamba mixer: the
    pure-PyTorch path of transformers' MambaMixer (`slow_forward`, sequential scan), with the same
    weights, at the single-block configuration (B=2, L=512, d_model 128, d_inner 256, d_state 16,
    d_conv 4, dt_rank 8).  transformers evaluates the scan in float32, so both run in float32 and
    outputs and every gradient must agree within 1e-4 of the largest magnitude."""
    mm = pytest.importorskip("transformers.models.mamba.modeling_mamba")
    from transformers import MambaConfig
    torch.manual_seed(0)
    g = torch.Generator().manual_seed(7)
    d, N, E, K, R = 128, 16, 256, 4, 8
    p = {k: v.float() for k, v in MS.std_init(d, N, 2, K, R, g).items()}
    cfg = MambaConfig(hidden_size=d, state_size=N, expand=2, conv_kernel=K, time_step_rank=R, use_bias=False,
                      use_conv_bias=True, hidden_act="silu", use_mambapy=False)
    mix = mm.MambaMixer(cfg, layer_idx=0).float()
    with torch.no_grad():
        mix.in_proj.weight.copy_(p["in_w"])
        mix.conv1d.weight.copy_(p["conv_w"].unsqueeze(1))
        mix.conv1d.bias.copy_(p["conv_b"])
        mix.x_proj.weight.copy_(p["x_w"])
        mix.dt_proj.weight.copy_(p["dt_w"])
        mix.dt_proj.bias.copy_(p["dt_b"])
        mix.A_log.copy_(p["A_log"])
        mix.D.copy_(p["D"])
        mix.out_proj.weight.copy_(p["out_w"])
    x = torch.randn(2, 512, d, generator=g)
    gy = torch.randn(2, 512, d, generator=g)

    xa = x.clone().requires_grad_(True)
    ya = mix.slow_forward(xa)
    (ya * gy).sum().backward()
    theirs = {"x": xa.grad, "in_w": mix.in_proj.weight.grad, "conv_w": mix.conv1d.weight.grad[:, 0],
              "conv_b": mix.conv1d.bias.grad, "x_w": mix.x_proj.weight.grad, "dt_w": mix.dt_proj.weight.grad,
              "dt_b": mix.dt_proj.bias.grad, "A_log": mix.A_log.grad, "D": mix.D.grad,
              "out_w": mix.out_proj.weight.grad}

    q = {k: v.clone().requires_grad_(True) for k, v in p.items()}
    xb = x.clone().requires_grad_(True)
    yb = MS.mixer_forward(q, xb)
    (yb * gy).sum().backward()
    ours = dict({k: v.grad for k, v in q.items()}, x=xb.grad)

    def close(a, b, name):
        err = (a - b).abs().max().item()
        assert err <= 1e-6 + 1e-4 * b.abs().max().item(), (name, err, b.abs().max().item())

    close(yb.detach(), ya.detach(), "out")
    for k, v in theirs.items():
        close(ours[k], v, k)
