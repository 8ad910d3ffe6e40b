"""CPU checks of the drop-in surface: module names, signatures, parameter names and seeded init."""
import inspect
import os
import subprocess
import sys

import torch

from tests.conftest import ROOT, golden


def test_dropin_modules_import_under_reference_names():
    code = ("import pgf_mamba_block, pgf_rmsnorm, pgf_ffn, pgf_embedding, pgf_lm_head, pgf_mamba, "
            "train_singlemamba_optimized as t;"
            "assert hasattr(pgf_mamba, 'FrechetMambaOperator');"
            "assert hasattr(pgf_mamba_block, 'PGFMambaSequential');"
            "assert hasattr(t, 'SingleLayerMambaPGF');"
            "print(pgf_mamba_block.PGFMambaBlock.__module__)")
    env = dict(os.environ, PYTHONPATH=os.path.join(ROOT, "icml_b200", "dropin"))
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, cwd="/")
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "icml_b200.pgf_mamba_block"


def test_signatures_match_reference():
    from icml_b200 import pgf_embedding, pgf_ffn, pgf_lm_head
    from icml_b200.pgf_mamba_block import PGFMambaBlock
    from icml_b200.pgf_rmsnorm import RMSNorm
    from icml_b200.train_singlemamba_optimized import SingleLayerMambaPGF

    def params(f):
        return list(inspect.signature(f).parameters)

    assert params(pgf_ffn.pgf_ffn_grad) == ["x", "g_out", "W1", "b1", "W2", "b2", "block_size", "activation",
                                             "compute_input_grads", "fp32_accum"]
    assert params(pgf_ffn.pgf_ffn_forward) == ["x", "W1", "b1", "W2", "b2", "block_size", "activation",
                                                "streaming", "callback"]
    assert params(pgf_lm_head.pgf_lm_head_grad) == ["hidden", "g_logits", "W_lm_head", "block_size",
                                                     "compute_input_grads", "fp32_accum"]
    assert params(pgf_embedding.pgf_embedding_grad) == ["input_ids", "g_out", "weight", "block_size",
                                                         "compute_input_grads", "fp32_accum"]
    assert params(RMSNorm.pgf_grad) == ["self", "x", "g_out", "block_size", "fp32_accum",
                                        "compute_input_grads"]
    assert params(PGFMambaBlock.__init__) == ["self", "d_model", "d_state", "d_ff", "block_size",
                                              "output_activation", "ffn_activation"]
    assert params(SingleLayerMambaPGF._pass2_block_direct_grad) == [
        "self", "u_block", "g_out_block", "h0_block", "delta_h_next", "dA_next", "fp32_accum"]
    # forward-mode operators (pgf_ffn.py:146-158, pgf_rmsnorm.py:120-126, pgf_mamba.py:36,69)
    from icml_b200.pgf_mamba import FrechetMambaOperator
    assert params(pgf_ffn.pgf_ffn_jvp) == ["x", "x_dot", "W1", "W1_dot", "b1", "b1_dot", "W2", "W2_dot", "b2",
                                            "b2_dot", "block_size", "activation"]
    assert params(RMSNorm.pgf_jvp) == ["self", "x", "x_dot", "weight_dot", "block_size"]
    assert params(FrechetMambaOperator.__init__) == ["self", "d_model", "d_state", "init_window"]
    assert params(FrechetMambaOperator.pgf_forward) == ["self", "u_seq", "du_seq", "block_size", "streaming",
                                                        "callback"]


def test_seeded_init_matches_reference():
    from icml_b200.pgf_mamba_block import PGFMambaBlock
    from icml_b200.train_singlemamba_optimized import SingleLayerMambaPGF
    G = golden("init.pt")
    torch.manual_seed(5)
    sd = PGFMambaBlock(32, 16, 64, 32).state_dict()
    assert sorted(sd) == sorted(G["block"])
    for k, v in G["block"].items():
        assert torch.equal(sd[k], v), k
    torch.manual_seed(6)
    sd = SingleLayerMambaPGF(24, 16).state_dict()
    for k, v in G["ssm"].items():
        assert torch.equal(sd[k], v), k


def test_frechet_operator_seeded_init_matches_reference():
    """FrechetMambaOperator keeps the reference's parameter names and construction order
    (pgf_mamba.py:33-49): a seeded construction gives the reference's initial weights."""
    from icml_b200.pgf_mamba import FrechetMambaOperator
    G = golden("jvp.pt")
    for name, D in (("frechet", 32), ("frechet_short", 16)):
        torch.manual_seed(33)
        sd = FrechetMambaOperator(d_model=D, d_state=16).state_dict()
        assert set(sd) == set(G[name]["params"])
        for k, v in G[name]["params"].items():
            assert torch.equal(sd[k], v), k


def test_projection_weights_adjacent_view():
    """With a layer's projections laid out back to back in one flat buffer (the order flat_order
    gives), _cat_weights returns views of that buffer equal to the concatenation; otherwise copies."""
    from icml_b200.train_singlemamba_optimized import SingleLayerMambaPGF, _cat_weights, flat_order
    torch.manual_seed(3)
    m = SingleLayerMambaPGF(24, 16)
    ref_W = torch.cat([m.dt_proj.weight, m.B_proj.weight, m.C_proj.weight]).detach().clone()
    ref_b = torch.cat([m.dt_proj.bias, m.B_proj.bias, m.C_proj.bias]).detach().clone()
    W, b = _cat_weights(m)                       # separate parameters: copies
    assert torch.equal(W, ref_W) and torch.equal(b, ref_b)
    order = flat_order(m.parameters(), m)
    at = [id(p) for p in order].index(id(m.dt_proj.weight))
    assert [id(p) for p in order[at:at + 6]] == [
        id(p) for p in (m.dt_proj.weight, m.B_proj.weight, m.C_proj.weight, m.dt_proj.bias, m.B_proj.bias,
                        m.C_proj.bias)]
    assert sorted(map(id, order)) == sorted(map(id, m.parameters()))
    flat = torch.zeros(sum(p.numel() for p in order))
    o = 0
    with torch.no_grad():
        for p in order:
            v = flat[o:o + p.numel()].view_as(p)
            v.copy_(p)
            p.data = v
            o += p.numel()
    W, b = _cat_weights(m)
    assert torch.equal(W, ref_W) and torch.equal(b, ref_b)
    assert W.untyped_storage().data_ptr() == flat.untyped_storage().data_ptr()
    assert b.untyped_storage().data_ptr() == flat.untyped_storage().data_ptr()


def test_layer_stash_policies():
    """The stash policies the LM accepts; tensors that stay on their device come back as they were
    put, and each slot is released when taken."""
    import pytest
    from icml_b200.lm import LayerStash
    for bad in ("gpu", "", "Host"):
        with pytest.raises(ValueError):
            LayerStash(bad)
    for policy in ("device", "host", "scan"):
        st = LayerStash(policy)
        st.begin(3)
        xs = [torch.randn(2, 5) for _ in range(3)]  # CPU tensors never go through the copy stream
        for i, x in enumerate(xs):
            st.put(i, x)
        for i in reversed(range(3)):
            if i > 0:
                st.prefetch(i - 1, "cpu")
            assert st.take(i, "cpu") is xs[i]
            assert st.items[i] is None


def test_operators_refuse_cpu_tensors():
    """No CPU path: every operator checks its tensors before any work and raises on host tensors,
    rather than computing something on the CPU."""
    import pytest
    from icml_b200 import ops
    x = torch.randn(4, 8)
    w = torch.ones(8)
    calls = [
        lambda: ops.rmsnorm_fwd(x, w, 1e-6),
        lambda: ops.embedding_fwd(torch.zeros(4, dtype=torch.long), torch.randn(10, 8)),
        lambda: ops.ffn_fwd(x, torch.randn(16, 8), torch.zeros(16), torch.randn(8, 16), torch.zeros(8)),
        lambda: ops.lm_head_ce_fwd(x, torch.randn(10, 8), torch.zeros(4, dtype=torch.long)),
        lambda: ops.ssm_fwd(x.view(1, 4, 8), torch.randn(8 + 32, 8), torch.zeros(8 + 32), torch.zeros(8, 16),
                            torch.ones(8), 1.0),
    ]
    for call in calls:
        with pytest.raises(RuntimeError, match="CUDA tensors only"):
            call()
