"""Flat-buffer AdamW and global gradient norm (pgf_adamw_step, pgf_grad_norm) against torch.

The reference's optimizer is torch.optim.AdamW(lr=1e-3, weight_decay=0.01) (train_wikitext_rebuttal.py:77),
so torch's own AdamW (the single-tensor float32 implementation) is the truth here; clipping is
torch.nn.utils.clip_grad_norm_.
"""
import pytest
import torch

from tests.parity import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
SHAPES = [(257, 33), (1024,), (3,), (64, 64), (5, 7, 9), (1,)]


def _params(seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(*s, generator=g) for s in SHAPES]


def _grads(seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return [scale * torch.randn(*s, generator=g) for s in SHAPES]


@pytest.mark.parametrize("max_norm", [None, 0.5, 1e6])
def test_flat_adamw_matches_torch_adamw(max_norm):
    from icml_b200.optim import FlatAdamW
    p0 = _params(1)
    ours = [torch.nn.Parameter(p.clone().to(DEV)) for p in p0]
    ref = [torch.nn.Parameter(p.clone().to(DEV)) for p in p0]
    opt = FlatAdamW(ours, lr=1e-2, weight_decay=0.01, max_grad_norm=max_norm)
    topt = torch.optim.AdamW(ref, lr=1e-2, weight_decay=0.01, foreach=False, fused=False)
    for it in range(6):
        gs = _grads(100 + it, scale=0.3 * (it + 1))
        for p, q, g in zip(ours, ref, gs):
            p.grad = g.to(DEV)
            q.grad = g.to(DEV)
        if max_norm is not None:
            torch.nn.utils.clip_grad_norm_(ref, max_norm)
        opt.step()
        topt.step()
    for p, q in zip(ours, ref):
        assert_close(p, q, atol=2e-6, rtol=1e-5)
    # the parameters are views into the flat buffer
    assert all(p.data_ptr() >= opt.flat.data_ptr() for p in ours)
    assert opt.step_count.item() == 6.0


def test_flat_adamw_none_grad_is_zero_grad():
    from icml_b200.optim import FlatAdamW
    p0 = _params(2)
    ours = [torch.nn.Parameter(p.clone().to(DEV)) for p in p0]
    ref = [torch.nn.Parameter(p.clone().to(DEV)) for p in p0]
    opt = FlatAdamW(ours, lr=1e-3)
    topt = torch.optim.AdamW(ref, lr=1e-3, foreach=False, fused=False)
    gs = _grads(7)
    for i, (p, q, g) in enumerate(zip(ours, ref, gs)):
        p.grad = None if i == 1 else g.to(DEV)
        q.grad = torch.zeros_like(q) if i == 1 else g.to(DEV)
    opt.step()
    topt.step()
    for p, q in zip(ours, ref):
        assert_close(p, q, atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("n", [1, 5, 4096, 3_000_001])
def test_grad_norm_deterministic_and_exact(n):
    from icml_b200.optim import grad_norm
    g = torch.Generator().manual_seed(n)
    x = torch.randn(n, generator=g).to(DEV)
    norm, clip = grad_norm(x, max_norm=1.0)
    norm2, _ = grad_norm(x, max_norm=1.0)
    assert torch.equal(norm, norm2)
    ref = torch.linalg.vector_norm(x.double()).item()
    assert abs(norm.item() - ref) <= 2e-6 * ref
    assert abs(clip.item() - min(1.0, 1.0 / (ref + 1e-6))) <= 2e-6


def test_lm_flat_optimizer_matches_torch_optimizer():
    """Two training steps of the LM with the flat optimizer and with torch's AdamW from one init."""
    from icml_b200.lm import PGFLanguageModel
    torch.manual_seed(3)
    a = PGFLanguageModel(301, 64, 16, 128, 2, 64, DEV, optimizer="flat")
    b = PGFLanguageModel(301, 64, 16, 128, 2, 64, DEV, optimizer="torch")
    b.load_(a.emb_weight.detach(), a.lm_head_weight.detach(), a.backbone.state_dict())
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, 301, (2, 200), generator=g).to(DEV)
    tg = torch.randint(0, 301, (2, 200), generator=g).to(DEV)
    for _ in range(2):
        la = a.step(ids, tg)
        lb = b.step(ids, tg)
        assert abs(la.item() - lb.item()) < 1e-5
    for (n1, p1), (n2, p2) in zip(a.backbone.named_parameters(), b.backbone.named_parameters()):
        assert_close(p1, p2, atol=1e-5, rtol=1e-4, name=n1)
    assert_close(a.emb_weight, b.emb_weight, atol=1e-5, rtol=1e-4)


def test_adamw_rejects_misaligned_buffers():
    from icml_b200._lib import lib
    buf = torch.zeros(64, device=DEV)
    step = torch.zeros(1, device=DEV)
    rc = lib().pgf_adamw_step(buf[1:].data_ptr(), buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), 8, 1e-3, 0.9,
                              0.999, 1e-8, 0.0, step.data_ptr(), None, None)
    assert rc != 0


def test_multi_tensor_path_equals_flat_path_across_launches():
    """The multi-tensor update (gradients in place, chunk tables over several launches for a tensor
    of more than 1000 chunks) gives bitwise the flat-gradient update."""
    from icml_b200.optim import FlatAdamW
    g = torch.Generator().manual_seed(9)
    shapes = [(33_000_001,), (5,), (129, 3)]
    p0 = [torch.randn(*s, generator=g) for s in shapes]
    gr = [torch.randn(*s, generator=g) for s in shapes]
    a = [torch.nn.Parameter(p.to(DEV)) for p in p0]
    b = [torch.nn.Parameter(p.to(DEV)) for p in p0]
    oa, ob = FlatAdamW(a, lr=1e-2), FlatAdamW(b, lr=1e-2)
    for it in range(2):
        for p, q, x in zip(a, b, gr):
            p.grad = (x * (it + 1)).to(DEV)
            q.grad = (x * (it + 1)).to(DEV)
        oa.step()                   # multi-tensor, no flat gradient
        ob.gather()
        ob.step(gather=False)       # flat gradient
    assert torch.equal(oa.flat, ob.flat)
    assert torch.equal(oa.exp_avg_sq, ob.exp_avg_sq)
    ob.gather()
    assert torch.equal(ob.grad[:33_000_001], gr[0].to(DEV) * 2)
