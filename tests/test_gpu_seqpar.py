"""Sequence sharding over NCCL on 2 GPUs against the single-GPU step on the whole sequence.

Runs only where two GPUs are visible (skipped otherwise).  The ranks are child processes with a
short process-group timeout; NVLS is off.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import ROOT

pytestmark = pytest.mark.gpu
V, D_MODEL, D_FF, N_LAYERS, B, L = 512, 64, 128, 2, 1, 4096


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(dev):
    from icml_b200.lm import PGFLanguageModel
    torch.manual_seed(5)
    m = PGFLanguageModel(V, D_MODEL, 16, D_FF, N_LAYERS, 256, "cpu")
    with torch.no_grad():
        m.emb_weight.normal_(0, 0.5)
        m.lm_head_weight.normal_(0, 0.3)
    m.emb_weight.data = m.emb_weight.data.to(dev)
    m.lm_head_weight.data = m.lm_head_weight.data.to(dev)
    m.backbone.to(dev)
    return m


def _data():
    g = torch.Generator().manual_seed(6)
    return torch.randint(0, V, (B, L), generator=g), torch.randint(0, V, (B, L), generator=g)


def _worker(rank, world, port, out_path):
    import datetime
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from icml_b200 import seqpar
        dev = torch.device("cuda", rank)
        m = _model(dev)
        ids, tg = _data()
        seg = L // world
        sl = slice(rank * seg, (rank + 1) * seg)
        loss, grads = seqpar.lm_forward_backward(m, ids[:, sl].contiguous().to(dev), tg[:, sl].contiguous().to(dev),
                                                 seqpar.SeqGroup.from_default())
        torch.cuda.synchronize()
        if rank == 0:
            torch.save({"loss": loss.cpu(), "grads": {k: v.cpu() for k, v in grads.items()}}, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_sequence_sharding_matches_one_gpu(tmp_path):
    out = str(tmp_path / "r0.pt")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    got = torch.load(out, weights_only=False)
    m = _model(torch.device("cuda", 0))
    ids, tg = _data()
    loss, ref = m.forward_backward(ids.cuda(), tg.cuda())
    assert abs(got["loss"].item() - loss.item()) < 1e-5
    for k, v in ref.items():
        v = v.cpu()
        err = (got["grads"][k] - v).abs().max().item()
        assert err <= 1e-5 + 1e-4 * v.abs().max().item(), (k, err)


def _flat_model(dev, variant="reference"):
    from icml_b200.lm import PGFLanguageModel
    torch.manual_seed(5)
    if variant == "std":
        m = PGFLanguageModel(V, D_MODEL, 16, D_FF, N_LAYERS, 256, dev, variant="std", tie_embeddings=True,
                             final_norm=True, expand=2, d_conv=4, dt_rank=4)
    else:
        m = PGFLanguageModel(V, D_MODEL, 16, D_FF, N_LAYERS, 256, dev)  # flat AdamW on the GPU
    with torch.no_grad():
        m.emb_weight.normal_(0, 0.5)
        m.lm_head_weight.normal_(0, 0.3)
    return m


def _named_params(m):
    out = {"emb": m.emb_weight}
    if not m.tied:
        out["lm_head"] = m.lm_head_weight
    if m.final_norm is not None:
        out["final_norm"] = m.final_norm.weight
    for i, layer in enumerate(m.backbone.layers):
        for n, p in layer.named_parameters():
            out[f"layers.{i}.{n}"] = p
    return out


def _reducer_worker(rank, world, port, out_path, mode):
    import datetime
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from icml_b200 import seqpar
        from icml_b200.optim import OverlappedGradReduce
        dev = torch.device("cuda", rank)
        m = _flat_model(dev, "std" if mode == "sp_std" else "reference")
        ids, tg = _data()
        if mode in ("sp", "sp_std"):
            seg = L // world
            sl = slice(rank * seg, (rank + 1) * seg)
            red = OverlappedGradReduce(m, dist.ReduceOp.SUM)
            loss, _ = seqpar.lm_forward_backward(m, ids[:, sl].contiguous().to(dev), tg[:, sl].contiguous().to(dev),
                                                 seqpar.SeqGroup.from_default(), reducer=red)
        else:
            # data parallel: every rank the whole batch of its own copy of the data (identical replicas
            # and data, so the average equals the one-GPU gradient)
            red = OverlappedGradReduce(m, dist.ReduceOp.AVG)
            loss, grads = m.forward_backward(ids.to(dev), tg.to(dev), on_layer_grads=red.layer)
            red.finish(grads)
        torch.cuda.synchronize()
        opt = m.optimizer
        slot = {id(q): o for q, o in zip(opt.params, opt.offsets)}
        got = {k: opt.grad[slot[id(p)]:slot[id(p)] + p.numel()].view_as(p).cpu() for k, p in _named_params(m).items()}
        if rank == 0:
            torch.save({"loss": loss.cpu(), "grads": got}, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["sp", "dp", "sp_std"])
def test_two_gpu_overlapped_reduce_matches_one_gpu(tmp_path, mode):
    """Layer-by-layer gradient all-reduce into the flat optimizer buffer (side stream), for sequence
    sharding (sum of partial gradients) and data parallelism (average of replicas)."""
    out = str(tmp_path / "r0.pt")
    mp.start_processes(_reducer_worker, args=(2, _free_port(), out, mode), nprocs=2, start_method="spawn")
    got = torch.load(out, weights_only=False)
    m = _flat_model(torch.device("cuda", 0), "std" if mode == "sp_std" else "reference")
    ids, tg = _data()
    loss, ref = m.forward_backward(ids.cuda(), tg.cuda())
    assert abs(got["loss"].item() - loss.item()) < 1e-5
    for k, v in ref.items():
        v = v.cpu()
        err = (got["grads"][k] - v).abs().max().item()
        assert err <= 1e-5 + 1e-4 * v.abs().max().item(), (k, err)


@pytest.mark.parametrize("per_channel", [False, True])
@pytest.mark.parametrize("P", [1, 2, 3, 8])
def test_compose_ranks_kernels_equal_host_fold(P, per_channel):
    """The rank-composition kernels against the host statement of the same fold (tests/cpu_ops.py)."""
    from icml_b200 import ops
    from tests import cpu_ops
    g = torch.Generator().manual_seed(30 + P)
    Bsz, D, N = 2, 40, 16
    A_log = torch.log(torch.rand(D, N, generator=g) + 0.1) if per_channel else torch.log(torch.rand(N, generator=g) + 0.1)
    n = Bsz * D * N
    fwd = torch.cat([torch.randn(P, n, generator=g), torch.rand(P, Bsz * D, generator=g) * 3], 1)
    bwd = torch.cat([torch.randn(P, n, generator=g), torch.rand(P, n, generator=g), torch.rand(P, Bsz * D, generator=g) * 3], 1)
    for r in range(P):
        h = ops.ssm_compose_ranks_fwd(fwd.cuda(), r, A_log.cuda(), Bsz, D, N)
        assert torch.allclose(h.cpu(), cpu_ops.ssm_compose_ranks_fwd(fwd.double(), r, A_log.double(), Bsz, D, N).float(),
                              atol=1e-5, rtol=1e-5)
        dh, dA = ops.ssm_compose_ranks_bwd(bwd.cuda(), r, A_log.cuda(), Bsz, D, N)
        rdh, rdA = cpu_ops.ssm_compose_ranks_bwd(bwd.double(), r, A_log.double(), Bsz, D, N)
        assert torch.allclose(dh.cpu(), rdh.float(), atol=1e-5, rtol=1e-5)
        assert torch.equal(dA.cpu(), rdA.float())
