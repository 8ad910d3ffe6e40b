"""Sequence sharding of the PGF step across ranks: host logic on gloo CPU ranks against the oracle.

Two (and three) CPU processes each hold a contiguous segment of the same sequences; the segment
summaries are all-gathered and composed, gradients all-reduced.  The result must equal the
single-process oracle step on the whole sequences.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import pgf_oracle as O
from tests.conftest import ROOT

V, D_MODEL, D_FF, N_LAYERS, B, L = 64, 16, 32, 2, 2, 48


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(variant="reference"):
    from icml_b200.lm import PGFLanguageModel
    torch.manual_seed(3)
    if variant == "std":
        m = PGFLanguageModel(V, D_MODEL, 16, D_FF, N_LAYERS, 16, "cpu", variant="std", tie_embeddings=True,
                             final_norm=True, expand=2, d_conv=4, dt_rank=2)
    else:
        m = PGFLanguageModel(V, D_MODEL, 16, D_FF, N_LAYERS, 16, "cpu")
    with torch.no_grad():
        m.emb_weight.normal_(0, 0.5)
        m.lm_head_weight.normal_(0, 0.3)
    return m


def _data():
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, V, (B, L), generator=g)
    return ids, torch.randint(0, V, (B, L), generator=g)


def _worker(rank, world, port, out_path, variant="reference"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, ROOT)
        from icml_b200 import seqpar
        from tests import cpu_ops
        m = _model(variant)
        ids, tg = _data()
        seg = L // world
        sl = slice(rank * seg, (rank + 1) * seg)
        sp = seqpar.SeqGroup.from_default()
        loss, grads = seqpar.lm_forward_backward(m, ids[:, sl].contiguous(), tg[:, sl].contiguous(), sp,
                                                 ops=cpu_ops)
        if rank == 0:
            torch.save({"loss": loss, "grads": grads}, out_path)
    finally:
        dist.destroy_process_group()


def _reference():
    m = _model()
    ids, tg = _data()
    blocks = [{k: v.detach() for k, v in layer.state_dict().items()} for layer in m.backbone.layers]
    return O.lm_pgf_step(m.emb_weight.detach(), m.lm_head_weight.detach(), blocks, ids, tg, 16)


def _std_reference():
    from oracle import mamba_std as MS
    m = _model("std")
    ids, tg = _data()
    blocks = []
    for layer in m.backbone.layers:
        sd = {k: v.detach().double() for k, v in layer.state_dict().items()}
        bp = {k: v for k, v in sd.items() if not k.startswith("mixer.")}
        for k, name in (("in_w", "in_proj.weight"), ("conv_b", "conv1d.bias"), ("x_w", "x_proj.weight"),
                        ("dt_w", "dt_proj.weight"), ("dt_b", "dt_proj.bias"), ("A_log", "A_log"), ("D", "D"),
                        ("out_w", "out_proj.weight")):
            bp["mixer." + k] = sd["mixer." + name]
        bp["mixer.conv_w"] = sd["mixer.conv1d.weight"].reshape(sd["mixer.conv1d.weight"].shape[0], -1)
        blocks.append(bp)
    loss, g = MS.lm_grads(m.emb_weight.detach().double(), None, m.final_norm.weight.detach().double(), blocks, ids, tg)
    names = {"in_w": "in_proj.weight", "conv_w": "conv1d.weight", "conv_b": "conv1d.bias", "x_w": "x_proj.weight",
             "dt_w": "dt_proj.weight", "dt_b": "dt_proj.bias", "A_log": "A_log", "D": "D", "out_w": "out_proj.weight"}
    out = {}
    for k, v in g.items():
        parts = k.split(".")
        if len(parts) > 3 and parts[2] == "mixer":
            k = ".".join(parts[:3] + [names[parts[3]]])
        out[k] = v
    return loss, out


@pytest.mark.parametrize("world", [2, 3])
def test_std_sequence_sharded_step_matches_oracle_autograd(world, tmp_path):
    """The Mamba-standard model (final RMSNorm, tied head) sharded over gloo ranks: conv context rows
    from the previous rank, per-channel-A state and adjoint composition, context-row gradients back."""
    out = str(tmp_path / "r0.pt")
    mp.start_processes(_worker, args=(world, _free_port(), out, "std"), nprocs=world, start_method="spawn")
    got = torch.load(out, weights_only=False)
    rloss, rgrads = _std_reference()
    assert abs(got["loss"].item() - rloss.item()) < 1e-5
    for k, v in rgrads.items():
        gv = got["grads"][k].reshape(v.shape).double()
        err = (gv - v).abs().max().item()
        assert err <= 1e-5 + 1e-4 * v.abs().max().item(), (k, err)


@pytest.mark.parametrize("world", [2, 3])
def test_sequence_sharded_step_matches_single_process_oracle(world, tmp_path):
    out = str(tmp_path / "r0.pt")
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
    got = torch.load(out, weights_only=False)
    rloss, rgrads = _reference()
    assert abs(got["loss"].item() - rloss.item()) < 1e-5
    for k, v in rgrads.items():
        err = (got["grads"][k] - v).abs().max().item()
        assert err <= 1e-5 + 1e-4 * v.abs().max().item(), (k, err)


def _gathered(rows):
    return torch.stack([torch.cat([t.reshape(-1) for t in r]) for r in rows])


def test_compose_functions_equal_sequential_scan():
    """The rank composition (forward state, backward carry) against one long oracle scan."""
    from tests import cpu_ops
    g = torch.Generator().manual_seed(8)
    d, N, Lt, P = 12, 16, 60, 4
    p = O.ssm_init(d, N, g, dtype=torch.float64)
    W = torch.cat([p["dt_w"], p["B_w"], p["C_w"]]).double()
    bb = torch.cat([p["dt_b"], p["B_b"], p["C_b"]]).double()
    u = torch.randn(1, Lt, d, generator=g, dtype=torch.float64)
    gy = torch.randn(1, Lt, d, generator=g, dtype=torch.float64)
    segs = [slice(i * Lt // P, (i + 1) * Lt // P) for i in range(P)]
    fwd = _gathered([cpu_ops.ssm_summary(u[:, s], W, bb, p["A_log"]) for s in segs])
    _, h0s, _ = O.ssm_forward(p, u, Lt // P)
    for r in range(P):
        assert torch.allclose(cpu_ops.ssm_compose_ranks_fwd(fwd, r, p["A_log"], 1, d, N), h0s[r], atol=1e-10)
    # backward carries: the whole-sequence block chain of the oracle is the truth
    bwd = _gathered([cpu_ops.ssm_bwd_summary(u[:, s], gy[:, s], W, bb, p["A_log"], p["scale"]) for s in segs])
    dh = torch.zeros(1, d, N, dtype=torch.float64)
    dA = torch.ones(1, d, N, dtype=torch.float64)
    for r in reversed(range(P)):
        G, aE = cpu_ops.ssm_compose_ranks_bwd(bwd, r, p["A_log"], 1, d, N)
        assert torch.allclose(G, dh, atol=1e-10) and torch.allclose(aE, dA, atol=1e-12)
        res = O.ssm_block_grad(p, u[:, segs[r]], gy[:, segs[r]], h0s[r], dh, dA)
        dh, dA = res["delta_h0"], res["dA0"]
