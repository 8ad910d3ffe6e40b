"""pgf_rmsnorm_bwd_noalloc: the RMSNorm backward for callers that cannot allocate device memory.

Such callers (an engine that owns every byte of device memory and forbids its operators to
allocate, or a loop that must never enter the allocator) get the same results as the workspace
variant, with the scratch held in a 4 MiB static array inside the library.  This file is collected
last so that a run stopping at the first failure has already run every other test.
"""
import pytest
import torch

from tests.parity import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _call_noalloc(L, x, g, w, eps, gw, gx, accumulate=0):
    from icml_b200.ops import _dt, _stream
    return L.pgf_rmsnorm_bwd_noalloc(x.data_ptr(), g.data_ptr(), w.data_ptr(), gx.data_ptr() if gx is not None else None,
                                     gw.data_ptr(), accumulate, x.numel() // x.shape[-1], x.shape[-1], eps, _dt(x),
                                     _stream())


def _inputs(gen, rows, dim, dtype):
    x = torch.randn(rows, dim, generator=gen).to(DEV, dtype)
    g = torch.randn(rows, dim, generator=gen).to(DEV, dtype)
    w = (1 + 0.02 * torch.randn(dim, generator=gen)).to(DEV)
    return x, g, w


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shapes", [((300, 256), (4096, 1024)), ((4096, 1024), (300, 256))],
                         ids=["small_then_large", "large_then_small"])
def test_noalloc_matches_workspace_entry_on_two_calls(dtype, shapes):
    """Two calls in a row on the one static array; large-then-small makes the second call run over
    partial slots that the first call left behind."""
    from icml_b200 import _lib, ops
    L = _lib.lib()
    gen = torch.Generator().manual_seed(77)
    for rows, dim in shapes:
        x, g, w = _inputs(gen, rows, dim, dtype)
        gw_ref, gx_ref = ops.rmsnorm_bwd(x, g, w, 1e-5)
        gw = torch.full((dim,), float("nan"), device=DEV)
        gx = torch.empty_like(x)
        rc = _call_noalloc(L, x, g, w, 1e-5, gw, gx)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert_close(gw, gw_ref, name="grad_weight")
        assert_close(gx.float(), gx_ref.float(), name="grad_x")


def test_noalloc_accumulate_and_no_grad_x():
    """accumulate=1 adds into grad_weight like the workspace entry point; grad_x may be NULL."""
    from icml_b200 import _lib, ops
    L = _lib.lib()
    gen = torch.Generator().manual_seed(78)
    x, g, w = _inputs(gen, 1000, 512, torch.float32)
    base = torch.randn(512, generator=gen).to(DEV)
    gw_ref, _ = ops.rmsnorm_bwd(x, g, w, 1e-6)
    gw = base.clone()
    rc = _call_noalloc(L, x, g, w, 1e-6, gw, None, accumulate=1)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert_close(gw, base + gw_ref, name="grad_weight accumulated")


def test_noalloc_zero_rows_zeroes_grad_weight():
    from icml_b200 import _lib
    from icml_b200.ops import _stream
    L = _lib.lib()
    w = torch.ones(256, device=DEV)
    gw = torch.full((256,), 3.0, device=DEV)
    assert L.pgf_rmsnorm_bwd_noalloc(None, None, w.data_ptr(), None, gw.data_ptr(), 0, 0, 256, 1e-5, 0,
                                     _stream()) == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert torch.count_nonzero(gw).item() == 0
    gw.fill_(3.0)
    assert L.pgf_rmsnorm_bwd_noalloc(None, None, w.data_ptr(), None, gw.data_ptr(), 1, 0, 256, 1e-5, 0,
                                     _stream()) == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert torch.all(gw == 3.0).item()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from icml_b200 import _lib
    L = _lib.lib()
    # ceil(rows/32) * dim = 2048 * 1024 > 2**20 floats: rejected before any GPU work
    rc = L.pgf_rmsnorm_bwd_noalloc(None, None, 1, None, 1, 0, 65536, 1024, 1e-5, 0, None)
    assert rc != 0
    assert "static scratch" in _lib.last_error()
    rc = L.pgf_rmsnorm_bwd_noalloc(None, None, 1, None, 1, 0, 32, 8192, 1e-5, 0, None)
    assert rc != 0
