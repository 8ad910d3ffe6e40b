"""Parity of the drop-in modules (PGFMambaBlock, SingleLayerMambaPGF, the LM step) against the
reference's own golden outputs and the float64 oracle."""
import pytest
import torch

from oracle import pgf_oracle as O
from tests.conftest import golden
from tests.parity import BF16_RTOL, assert_close, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _block_from(sd, d, dff, bs, act=None):
    from icml_b200.pgf_mamba_block import PGFMambaBlock
    blk = PGFMambaBlock(d, 16, dff, bs, output_activation=act)
    blk.load_state_dict(sd)
    return blk.to(DEV)


@pytest.mark.parametrize("act", ["none", "tanh"])
def test_block_matches_reference_golden(act):
    G = golden("block.pt")[act]
    d = G["x"].shape[-1]
    blk = _block_from(G["params"], d, G["d_ff"], G["block_size"], G["act"])
    x, g = G["x"].to(DEV), G["g"].to(DEV)
    assert_close(blk.pgf_forward(x), G["y"], name="pgf_forward")
    blk.reference_scale_grad = True
    r = blk.pgf_backward(x, g)
    assert_close(r["grad_input"], G["grad_input"], name="grad_input")
    for k, v in G["grads"].items():
        assert_close(r["grads"][k], v, name=k)
    # default: per-channel scale gradient = autograd of the reference forward
    blk.reference_scale_grad = False
    r = blk.pgf_backward(x, g)
    for k, v in G["autograd"]["grads"].items():
        assert_close(r["grads"][k], v, atol=2e-5, name="autograd " + k)
    assert_close(r["grad_input"], G["autograd"]["grad_input"], atol=2e-5, name="autograd grad_input")


def test_block_autograd_forward_matches_reference_autograd():
    G = golden("block.pt")["none"]
    d = G["x"].shape[-1]
    blk = _block_from(G["params"], d, G["d_ff"], G["block_size"])
    x = G["x"].to(DEV).requires_grad_(True)
    y = blk(x)
    y.backward(G["g"].to(DEV))
    assert_close(y, G["autograd"]["y"], name="y")
    assert_close(x.grad, G["autograd"]["grad_input"], atol=2e-5, name="grad_input")
    for k, p in blk.named_parameters():
        assert_close(p.grad, G["autograd"]["grads"][k], atol=2e-5, name=k)


def test_single_layer_pass2_block_golden():
    from icml_b200.train_singlemamba_optimized import SingleLayerMambaPGF
    G = golden("ssm_block.pt")
    m = SingleLayerMambaPGF(G["u"].shape[-1], 16)
    m.load_state_dict(G["params"])
    m = m.to(DEV)
    m.reference_scale_grad = True
    out = m._pass2_block_direct_grad(G["u"].to(DEV), G["g"].to(DEV), G["h0"].to(DEV),
                                     G["delta_h_next"].to(DEV), G["dA_next"].to(DEV))
    names = ["A_log", "D", "scale_ref", "dt_w", "dt_b", "B_w", "B_b", "C_w", "C_b", "delta_h0", "dA0", "grad_u"]
    for n, v in zip(names, out):
        assert_close(v, G["out"][n], name=n)


def _lm_from_golden(G, act_dtype=torch.float32):
    from icml_b200.lm import PGFLanguageModel
    V, d = G["emb"].shape
    lm = PGFLanguageModel(V, d, 16, G["d_ff"], G["n_layers"], G["block_size"], DEV, act_dtype=act_dtype)
    lm.load_(G["emb"].to(DEV), G["lm_head"].to(DEV), {k: v.to(DEV) for k, v in G["params"].items()})
    return lm


def test_lm_step_matches_reference_golden():
    G = golden("lm.pt")
    lm = _lm_from_golden(G)
    for layer in lm.backbone.layers:
        layer.reference_scale_grad = True
    loss, grads = lm.forward_backward(G["ids"].to(DEV), G["targets"].to(DEV))
    assert abs(loss.item() - G["loss"].item()) < 1e-5
    for k, v in G["grads"].items():
        assert_close(grads[k], v, atol=2e-5, name=k)


def test_lm_step_matches_autograd_golden():
    G = golden("lm.pt")
    lm = _lm_from_golden(G)
    loss, grads = lm.forward_backward(G["ids"].to(DEV), G["targets"].to(DEV))
    assert abs(loss.item() - G["autograd"]["loss"].item()) < 1e-5
    for k, v in G["autograd"]["grads"].items():
        assert_close(grads[k], v, atol=5e-5, name=k)


def _oracle_lm_f64(G):
    n = G["n_layers"]
    blocks = [{k[len(f"layers.{i}."):]: v.double() for k, v in G["params"].items() if k.startswith(f"layers.{i}.")}
              for i in range(n)]
    return O.lm_pgf_step(G["emb"].double(), G["lm_head"].double(), blocks, G["ids"], G["targets"], G["block_size"])


def test_lm_step_f32_within_f32_bound_of_f64_oracle():
    """The whole float32 PGF LM step (embedding, 2 layers, LM head + CE) against the float64 oracle at
    the float32 bound: max-abs error <= 1e-5 + 1e-4 max|ref| for every gradient, loss within 1e-5."""
    G = golden("lm.pt")
    lm = _lm_from_golden(G)
    loss, grads = lm.forward_backward(G["ids"].to(DEV), G["targets"].to(DEV))
    rloss, ref = _oracle_lm_f64(G)
    assert abs(loss.item() - rloss.item()) < 1e-5
    assert set(grads) == set(ref)
    for k, v in ref.items():
        assert_close(grads[k], v, name=k)


def test_lm_step_bf16_every_gradient_close_to_f64_oracle():
    """bf16 activations (float32 weights and gradients): every gradient within 5e-2 relative L2 of the
    float64 oracle, the loss within 2e-2 relative."""
    G = golden("lm.pt")
    lm = _lm_from_golden(G, act_dtype=torch.bfloat16)
    loss, grads = lm.forward_backward(G["ids"].to(DEV), G["targets"].to(DEV))
    rloss, ref = _oracle_lm_f64(G)
    assert abs(loss.item() - rloss.item()) < 2e-2 * abs(rloss.item())
    errs = {k: rel_err(grads[k], v) for k, v in ref.items()}
    bad = {k: e for k, e in errs.items() if not e < 5e-2}
    assert not bad, bad


def test_block_config1_reference_variant_f64_oracle():
    """Config-1 shapes on the reference variant (d=128, N=16, B=2, L=512), bs=128, float64 truth."""
    g = torch.Generator().manual_seed(40)
    d, dff, bs = 128, 512, 128
    bp = O.block_init(d, 16, dff, g)
    bp["norm1.weight"] = 1 + 0.02 * torch.randn(d, generator=g)
    x = torch.randn(2, 512, d, generator=g)
    gy = torch.randn(2, 512, d, generator=g)
    blk = _block_from(bp, d, dff, bs)
    r = blk.pgf_backward(x.to(DEV), gy.to(DEV))
    bpd = {k: v.double() for k, v in bp.items()}
    ref = O.block_pgf_backward(bpd, x.double(), gy.double(), bs)
    assert_close(r["grad_input"], ref["grad_input"], name="grad_input")
    for k, v in ref["grads"].items():
        assert_close(r["grads"][k], v, name=k)


def test_lm_step_bf16_activations_close_to_f32_oracle():
    G = golden("lm.pt")
    lm = _lm_from_golden(G, act_dtype=torch.bfloat16)
    loss, grads = lm.forward_backward(G["ids"].to(DEV), G["targets"].to(DEV))
    assert abs(loss.item() - G["autograd"]["loss"].item()) < 2e-2 * abs(G["autograd"]["loss"].item())
    for k in ("emb", "lm_head", "layers.0.W1", "layers.1.mamba.A_log", "layers.0.mamba.dt_proj.weight"):
        assert rel_err(grads[k], G["autograd"]["grads"][k]) < 5e-2, k


def test_lm_training_step_updates_and_loss_decreases():
    torch.manual_seed(0)
    from icml_b200.lm import PGFLanguageModel
    lm = PGFLanguageModel(256, 64, 16, 128, 2, 64, DEV)
    ids = torch.randint(0, 256, (2, 256), device=DEV)
    tg = torch.roll(ids, -1, 1)
    losses = [lm.step(ids, tg).item() for _ in range(30)]
    assert losses[-1] < losses[0] - 0.5, losses


@pytest.mark.parametrize("mode", ["recompute", "states", "scan"])
@pytest.mark.parametrize("act", ["none", "tanh"])
def test_block_segments_match_reference_golden(mode, act):
    """A block whose sequence runs in several segments (state carried forward, adjoint and decay
    carried backward, parameter gradients added up) matches the reference's block-wise PGF."""
    G = golden("block.pt")[act]
    d = G["x"].shape[-1]
    blk = _block_from(G["params"], d, G["d_ff"], G["block_size"], G["act"])
    blk.segment_tokens = 2 * G["block_size"]  # B=2: one PGF block per segment, three segments of L=80
    B, L, _ = G["x"].shape
    assert len(blk._segments(B, L)) == 3
    x, g = G["x"].to(DEV), G["g"].to(DEV)
    blk.reference_scale_grad = True
    if mode == "recompute":
        y = blk.pgf_forward(x)
        r = blk.pgf_backward(x, g)
    else:
        y, st = blk.pgf_forward(x, return_ssm_states=True, keep_scan=mode == "scan")
        assert isinstance(st, list) and len(st) == 3
        r = blk.pgf_backward(x, g, ssm_states=st)
    assert_close(y, G["y"], name="pgf_forward")
    assert_close(r["grad_input"], G["grad_input"], name="grad_input")
    for k, v in G["grads"].items():
        assert_close(r["grads"][k], v, name=k)


def test_lm_step_segmented_matches_reference_golden():
    G = golden("lm.pt")
    lm = _lm_from_golden(G)
    for layer in lm.backbone.layers:
        layer.reference_scale_grad = True
        layer.segment_tokens = 2 * G["block_size"]
    loss, grads = lm.forward_backward(G["ids"].to(DEV), G["targets"].to(DEV))
    assert abs(loss.item() - G["loss"].item()) < 1e-5
    for k, v in G["grads"].items():
        assert_close(grads[k], v, atol=2e-5, name=k)


def _step_peak(L, stash="device"):
    from icml_b200.lm import PGFLanguageModel
    torch.manual_seed(0)
    lm = PGFLanguageModel(50257, 256, 16, 1024, 8, 4096, DEV, act_dtype=torch.bfloat16, stash=stash)
    ids = torch.randint(0, 50257, (1, L + 1), device=DEV)
    lm.step(ids[:, :-1], ids[:, 1:])  # settles the optimizer state
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    loss, grads = lm.forward_backward(ids[:, :-1], ids[:, 1:])
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    del loss, grads, lm
    torch.cuda.empty_cache()
    return peak


@pytest.mark.parametrize("stash", ["device", "host"])
def test_step_memory_grows_only_by_the_per_token_buffers(stash):
    """Peak memory of the 8-layer step (d_model 256, bf16) at 262144 tokens minus that at 65536 stays
    within what must grow with L: the stashed layer inputs (8 per token-channel, or 2 with the host
    stash), the scan's boundary states (16 floats per channel per 128-token chunk and layer), the
    step's activation, gradient and output buffers (6 per token-channel) and the per-token vectors of
    the embedding and the cross entropy (64 bytes).  Scan, FFN and LM-head workspaces run in segments
    and tiles of fixed size, so they do not grow."""
    d, layers = 256, 8
    L1, L2 = 65536, 262144
    p1, p2 = _step_peak(L1, stash), _step_peak(L2, stash)
    stashed = layers if stash == "device" else 2
    per_token = (stashed + 6) * d * 2 + layers * d * 16 * 4 / 128 + 64
    assert p2 - p1 <= (L2 - L1) * per_token, (p1 / 1e9, p2 / 1e9, (L2 - L1) * per_token / 1e9)
