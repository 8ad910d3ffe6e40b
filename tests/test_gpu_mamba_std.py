"""Mamba-standard variant on the GPU against autograd of the float64 oracle, at the small test
shapes (B=2, L=512, d_model 128, d_inner 256, d_state 16) and ragged ones.

The reference has no code for this variant, so the truth is autograd of the CPU restatement in
oracle/mamba_std.py: every parameter and input gradient of the PGF path against plain autograd.
"""
import pytest
import torch

from oracle import mamba_std as MS
from tests.parity import BF16_RTOL, assert_close, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"
NAMES = {"in_w": "mixer.in_proj.weight", "conv_w": "mixer.conv1d.weight", "conv_b": "mixer.conv1d.bias",
         "x_w": "mixer.x_proj.weight", "dt_w": "mixer.dt_proj.weight", "dt_b": "mixer.dt_proj.bias",
         "A_log": "mixer.A_log", "D": "mixer.D", "out_w": "mixer.out_proj.weight"}


def _block_module(bp, d, d_ff, expand, K, R):
    from icml_b200.pgf_mamba_std import PGFMambaStdBlock
    blk = PGFMambaStdBlock(d, 16, d_ff, 128, expand, K, R)
    sd = {}
    for k, v in bp.items():
        if k.startswith("mixer."):
            name = NAMES[k[6:]]
            sd[name] = v.float().reshape(blk.state_dict()[name].shape)
        else:
            sd[k] = v.float()
    blk.load_state_dict(sd)
    return blk.to(DEV)


def _case(seed, B, L, d, E, R, K=4, d_ff=None):
    g = torch.Generator().manual_seed(seed)
    bp = MS.block_init(d, 16, d_ff or 2 * d, E // d, K, R, g)
    bp["norm1.weight"] = 1 + 0.05 * torch.randn(d, generator=g, dtype=torch.float64)
    bp["mixer.D"] = 1 + 0.2 * torch.randn(E, generator=g, dtype=torch.float64)
    x = torch.randn(B, L, d, generator=g, dtype=torch.float64)
    gy = torch.randn(B, L, d, generator=g, dtype=torch.float64)
    return bp, x, gy


@pytest.mark.parametrize("B,L,d,E,R", [(2, 512, 128, 256, 8), (1, 100, 64, 128, 4), (3, 37, 32, 64, 2)])
def test_std_block_pgf_backward_matches_autograd(B, L, d, E, R):
    bp, x, gy = _case(60 + L, B, L, d, E, R)
    blk = _block_module(bp, d, 2 * d, E // d, 4, R)
    y_ref, g_ref, gx_ref = MS.block_grads(bp, x, gy)
    y = blk.pgf_forward(x.float().to(DEV))
    assert_close(y, y_ref, name="pgf_forward")
    r = blk.pgf_backward(x.float().to(DEV), gy.float().to(DEV))
    assert_close(r["grad_input"], gx_ref, name="grad_input")
    for k, v in g_ref.items():
        name = NAMES[k[6:]] if k.startswith("mixer.") else k
        got = r["grads"][name].reshape(v.shape)
        assert_close(got, v, name=name)


def test_std_block_autograd_forward():
    bp, x, gy = _case(70, 2, 64, 32, 64, 2)
    blk = _block_module(bp, 32, 64, 2, 4, 2)
    xx = x.float().to(DEV).requires_grad_(True)
    y = blk(xx)
    y.backward(gy.float().to(DEV))
    y_ref, g_ref, gx_ref = MS.block_grads(bp, x, gy)
    assert_close(y, y_ref)
    assert_close(xx.grad, gx_ref)
    named = dict(blk.named_parameters())
    for k, v in g_ref.items():
        name = NAMES[k[6:]] if k.startswith("mixer.") else k
        assert_close(named[name].grad.reshape(v.shape), v, name=name)


def test_std_block_bf16_activations():
    bp, x, gy = _case(71, 1, 2048, 256, 512, 16, d_ff=1024)
    blk = _block_module(bp, 256, 1024, 2, 4, 16)
    xb, gb = x.bfloat16(), gy.bfloat16()
    r = blk.pgf_backward(xb.to(DEV), gb.to(DEV))
    _, g_ref, gx_ref = MS.block_grads(bp, xb.double(), gb.double())
    assert rel_err(r["grad_input"], gx_ref) < BF16_RTOL
    for k in ("mixer.in_w", "mixer.x_w", "mixer.A_log", "mixer.conv_w", "W1"):
        name = NAMES[k[6:]] if k.startswith("mixer.") else k
        assert rel_err(r["grads"][name].reshape(g_ref[k].shape), g_ref[k]) < BF16_RTOL, name


def test_std_lm_step_matches_autograd():
    """8-layer shape family at small size: tied embedding / LM head and a final RMSNorm."""
    from icml_b200.lm import PGFLanguageModel
    g = torch.Generator().manual_seed(72)
    V, d, E, R, nl, B, L = 97, 32, 64, 2, 2, 2, 40
    blocks = [MS.block_init(d, 16, 4 * d, 2, 4, R, g) for _ in range(nl)]
    emb = 0.5 * torch.randn(V, d, generator=g, dtype=torch.float64)
    fnw = 1 + 0.1 * torch.randn(d, generator=g, dtype=torch.float64)
    ids = torch.randint(0, V, (B, L), generator=g)
    tg = torch.randint(0, V, (B, L), generator=g)
    lm = PGFLanguageModel(V, d, 16, 4 * d, nl, 16, DEV, variant="std", tie_embeddings=True, final_norm=True,
                          expand=2, d_conv=4, dt_rank=R)
    with torch.no_grad():
        lm.emb_weight.copy_(emb.float())
        lm.final_norm.weight.copy_(fnw.float())
        for i, layer in enumerate(lm.backbone.layers):
            sd = {}
            for k, v in blocks[i].items():
                name = NAMES[k[6:]] if k.startswith("mixer.") else k
                sd[name] = v.float().reshape(layer.state_dict()[name].shape)
            layer.load_state_dict(sd)
    loss, grads = lm.forward_backward(ids.to(DEV), tg.to(DEV))
    rloss, rgrads = MS.lm_grads(emb, None, fnw, blocks, ids, tg)
    assert abs(loss.item() - rloss.item()) < 1e-5
    assert_close(grads["emb"], rgrads["emb"], name="emb (tied)")
    assert_close(grads["final_norm"], rgrads["final_norm"], name="final_norm")
    for i in range(nl):
        for k, v in rgrads.items():
            if not k.startswith(f"layers.{i}."):
                continue
            kk = k.split(".", 2)[2]
            name = NAMES[kk[6:]] if kk.startswith("mixer.") else kk
            assert_close(grads[f"layers.{i}.{name}"].reshape(v.shape), v, name=f"{i}.{name}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mixer_saved_forward_equals_recompute(dtype):
    """bwd_saved over fwd_save's intermediates gives bitwise the gradients of the re-running bwd."""
    from icml_b200 import ops
    g = torch.Generator().manual_seed(80)
    p = {k: v.float().to(DEV) for k, v in MS.std_init(64, 16, 2, 4, 4, g).items()}
    x = torch.randn(2, 300, 64, generator=g).to(DEV, dtype)
    gy = torch.randn(2, 300, 64, generator=g).to(DEV, dtype)
    out_s, saved = ops.mamba_mixer_fwd_save(x, p)
    out = ops.mamba_mixer_fwd(x, p)
    assert torch.equal(out_s, out)
    g1, gx1 = ops.mamba_mixer_bwd(x, gy, p)
    g2, gx2 = ops.mamba_mixer_bwd(x, gy, p, saved=saved)
    assert torch.equal(gx1, gx2)
    for k in ops.MIXER_KEYS:
        assert torch.equal(g1[k], g2[k]), k


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mixer_save_from_boundary_states_is_bitwise(dtype):
    """fwd_save given the boundary states of fwd(want_states=True) skips the scan's chunk pass and
    compose; the output and the backward over its saved buffer are the same bits (the buffer's
    forward-only chunk summaries are left unwritten)."""
    from icml_b200 import ops
    g = torch.Generator().manual_seed(81)
    p = {k: v.float().to(DEV) for k, v in MS.std_init(64, 16, 2, 4, 4, g).items()}
    x = torch.randn(2, 700, 64, generator=g).to(DEV, dtype)
    gy = torch.randn(2, 700, 64, generator=g).to(DEV, dtype)
    out0, st = ops.mamba_mixer_fwd(x, p, want_states=True)
    assert torch.equal(out0, ops.mamba_mixer_fwd(x, p))
    o1, s1 = ops.mamba_mixer_fwd_save(x, p)
    o2, s2 = ops.mamba_mixer_fwd_save(x, p, states=st)
    assert torch.equal(o1, o2)
    g1, gx1 = ops.mamba_mixer_bwd(x, gy, p, saved=s1)
    g2, gx2 = ops.mamba_mixer_bwd(x, gy, p, saved=s2)
    assert torch.equal(gx1, gx2)
    for k in ops.MIXER_KEYS:
        assert torch.equal(g1[k], g2[k]), k


@pytest.mark.parametrize("mode", ["recompute", "states", "scan"])
@pytest.mark.parametrize("K", [4, 2])
def test_std_block_segments_match_autograd(mode, K):
    """The Mamba-standard block over several segments (scan state and the conv's K-1-token context
    carried forward; adjoint, decay and the context rows' gradient carried backward; parameter
    gradients added up) against autograd of the float64 oracle over the whole sequence."""
    B, L, d, E, R = 2, 300, 32, 64, 2
    bp, x, gy = _case(80 + K, B, L, d, E, R, K=K)
    blk = _block_module(bp, d, 2 * d, E // d, K, R)
    blk.block_size = 64
    blk.segment_tokens = 2 * 64  # B=2: 64 tokens per segment, five segments of L=300
    assert len(blk._segments(B, L)) == 5
    y_ref, g_ref, gx_ref = MS.block_grads(bp, x, gy)
    xd, gd = x.float().to(DEV), gy.float().to(DEV)
    if mode == "recompute":
        y = blk.pgf_forward(xd)
        r = blk.pgf_backward(xd, gd)
    else:
        y, st = blk.pgf_forward(xd, return_ssm_states=True, keep_scan=mode == "scan")
        assert isinstance(st, list) and len(st) == 5
        r = blk.pgf_backward(xd, gd, ssm_states=st)
    assert_close(y, y_ref, name="pgf_forward")
    assert_close(r["grad_input"], gx_ref, name="grad_input")
    for k, v in g_ref.items():
        name = NAMES[k[6:]] if k.startswith("mixer.") else k
        assert_close(r["grads"][name].reshape(v.shape), v, name=name)


def test_std_mixer_staged_calls_equal_segment_call():
    """fwd_begin + fwd_finish and bwd_begin + bwd_finish with the carries equal the one-call segment
    forms (the pieces sequence sharding runs on each rank)."""
    from icml_b200 import ops
    B, L, d, E, R, K = 1, 200, 32, 64, 2, 4
    bp, x, gy = _case(90, B, L, d, E, R, K=K)
    blk = _block_module(bp, d, 2 * d, E // d, K, R)
    p = blk.mixer.params()
    g = torch.Generator().manual_seed(91)
    xn = x.float().to(DEV)
    halo = torch.randn(B, K - 1, d, generator=g).to(DEV)
    h0 = (0.3 * torch.randn(B, E, 16, generator=g)).to(DEV)
    dh = (0.3 * torch.randn(B, E, 16, generator=g)).to(DEV)
    dA = (0.5 + 0.5 * torch.rand(B, E, 16, generator=g)).to(DEV)
    out1, hf1, st1, saved = ops.mamba_mixer_fwd_seg(xn, p, x_halo=halo, h_init=h0, want_h_final=True,
                                                    want_states=False, save=True)
    hs, sdt, state = ops.mamba_mixer_fwd_begin(xn, p, x_halo=halo)
    out2, st2 = ops.mamba_mixer_fwd_finish(state, h0, want_states=True)
    assert_close(out2, out1, name="out")
    assert_close(ops.mamba_mixer_end_state(st2, B, L, d, E, R, 16, K), hf1, name="h_final")
    g1, gx1, gh1, dh0_1, dA0_1 = ops.mamba_mixer_bwd_seg(xn, gy.float().to(DEV), p, saved, x_halo=halo, dh_end=dh,
                                                        dA_end=dA, want_carry=True, want_g_halo=True)
    d0, a0, sx, bst = ops.mamba_mixer_bwd_begin(xn, gy.float().to(DEV), p, saved, x_halo=halo)
    g2, gx2, gh2 = ops.mamba_mixer_bwd_finish(bst, dh_end=dh, dA_end=dA, want_g_halo=True)
    assert_close(gx2, gx1, name="grad_x")
    assert_close(gh2, gh1, name="grad_x_halo")
    for k in g1:
        assert_close(g2[k], g1[k], name=k)
