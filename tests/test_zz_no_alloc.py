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


def _call_noalloc(L, x, g, w, eps, gw, gx):
    from icml_b200.ops import _dt, _stream
    return L.pgf_rmsnorm_bwd_noalloc(x.data_ptr(), g.data_ptr(), w.data_ptr(), gx.data_ptr(), gw.data_ptr(),
                                     0, x.numel() // x.shape[-1], x.shape[-1], eps, _dt(x), _stream())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_workspace_entry_on_two_calls(dtype):
    from icml_b200 import _lib, ops
    L = _lib.lib()
    gen = torch.Generator().manual_seed(77)
    for rows, dim in ((300, 256), (4096, 1024)):  # two calls in a row, the second reusing the array
        x = torch.randn(rows, dim, generator=gen).to(DEV, dtype)
        g = torch.randn(rows, dim, generator=gen).to(DEV, dtype)
        w = (1 + 0.02 * torch.randn(dim, generator=gen)).to(DEV)
        gw_ref, gx_ref = ops.rmsnorm_bwd(x, g, w, 1e-5)
        gw = torch.full((dim,), float("nan"), device=DEV)
        gx = torch.empty_like(x)
        rc = _call_noalloc(L, x, g, w, 1e-5, gw, gx)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert_close(gw, gw_ref, name="grad_weight")
        assert_close(gx.float(), gx_ref.float(), name="grad_x")


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from icml_b200 import _lib
    L = _lib.lib()
    # ceil(rows/32) * dim = 2048 * 1024 > 2**20 floats: rejected before any GPU work
    rc = L.pgf_rmsnorm_bwd_noalloc(None, None, 1, None, 1, 0, 65536, 1024, 1e-5, 0, None)
    assert rc != 0
    assert "static scratch" in _lib.last_error()
