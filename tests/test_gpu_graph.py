"""The CUDA-graph captured training step replays exactly the eager step."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _pair(variant, stash="device"):
    from icml_b200.lm import PGFLanguageModel
    kw = dict(act_dtype=torch.bfloat16, variant=variant, stash=stash)
    if variant == "std":
        kw.update(tie_embeddings=True, final_norm=True, expand=2, d_conv=4, dt_rank=4)
    torch.manual_seed(5)
    m1 = PGFLanguageModel(301, 64, 16, 128, 2, 64, DEV, **kw)
    m2 = PGFLanguageModel(301, 64, 16, 128, 2, 64, DEV, **kw)
    with torch.no_grad():
        for p1, p2 in zip(m1.params, m2.params):
            p2.copy_(p1)
    return m1, m2


@pytest.mark.parametrize("variant,stash", [("reference", "device"), ("std", "device"), ("reference", "host"),
                                           ("reference", "scan"), ("std", "scan")])
def test_graphed_step_equals_eager(variant, stash):
    from icml_b200.lm import GraphedStep
    m1, m2 = _pair(variant, stash)
    g = torch.Generator().manual_seed(9)
    batches = [(torch.randint(0, 301, (2, 200), generator=g), torch.randint(0, 301, (2, 200), generator=g))
               for _ in range(3)]
    x0, y0 = batches[0][0].to(DEV), batches[0][1].to(DEV)
    # eager: one step on batch 0 (the graph's warm-up step), then batches 1, 2
    m1.step(x0, y0)
    eager_losses = [m1.step(x.to(DEV), y.to(DEV)).item() for x, y in batches[1:]]
    gs = GraphedStep(m2, x0, y0, warmup=1)
    assert gs.launches > 0
    graph_losses = []
    for x, y in batches[1:]:
        graph_losses.append(gs.run(x.pin_memory(), y.pin_memory()).item())
    assert graph_losses == eager_losses
    for p1, p2 in zip(m1.params, m2.params):
        assert torch.equal(p1, p2)


def test_host_stash_equals_device_stash():
    """Layer inputs parked in pinned host memory between the passes give bitwise the same step."""
    from icml_b200.lm import PGFLanguageModel
    torch.manual_seed(6)
    kw = dict(act_dtype=torch.bfloat16)
    m1 = PGFLanguageModel(301, 64, 16, 128, 3, 64, DEV, stash="device", **kw)
    m2 = PGFLanguageModel(301, 64, 16, 128, 3, 64, DEV, stash="host", **kw)
    with torch.no_grad():
        for p1, p2 in zip(m1.params, m2.params):
            p2.copy_(p1)
    g = torch.Generator().manual_seed(10)
    x = torch.randint(0, 301, (2, 300), generator=g).to(DEV)
    y = torch.randint(0, 301, (2, 300), generator=g).to(DEV)
    l1, g1 = m1.forward_backward(x, y)
    l2, g2 = m2.forward_backward(x, y)
    assert torch.equal(l1, l2)
    for k in g1:
        assert torch.equal(g1[k], g2[k]), k
    assert len(m2.stash._host) == 2  # every layer input but the last went through host memory


@pytest.mark.parametrize("variant", ["reference", "std"])
def test_scan_stash_matches_recompute(variant):
    """Keeping the scan's saved states from the forward gives the step that recomputes them in the
    backward: the same loss bits, gradients within float32 rounding (float32 activations)."""
    from icml_b200.lm import PGFLanguageModel
    from tests.parity import assert_close
    kw = dict(act_dtype=torch.float32, variant=variant)
    if variant == "std":
        kw.update(tie_embeddings=True, final_norm=True, expand=2, d_conv=4, dt_rank=4)
    torch.manual_seed(7)
    m1 = PGFLanguageModel(301, 64, 16, 128, 3, 64, DEV, stash="device", **kw)
    m2 = PGFLanguageModel(301, 64, 16, 128, 3, 64, DEV, stash="scan", **kw)
    with torch.no_grad():
        for p1, p2 in zip(m1.params, m2.params):
            p2.copy_(p1)
    g = torch.Generator().manual_seed(11)
    x = torch.randint(0, 301, (2, 700), generator=g).to(DEV)
    y = torch.randint(0, 301, (2, 700), generator=g).to(DEV)
    l1, g1 = m1.forward_backward(x, y)
    l2, g2 = m2.forward_backward(x, y)
    assert torch.equal(l1, l2)
    assert g1.keys() == g2.keys()
    for k in g1:
        assert_close(g2[k], g1[k], name=k)
