"""The tcgen05/TMEM bf16 dense-product engine against a float64 product of the same bf16 inputs."""
import ctypes

import pytest
import torch

from tests.parity import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from icml_b200 import ops as _ops
    return _ops


def _tc_launches(fn):
    from icml_b200 import _lib
    L = _lib.lib()
    L.pgf_profile(1)
    out = fn()
    torch.cuda.synchronize()
    L.pgf_profile(0)
    c, t, w = ctypes.c_longlong(0), ctypes.c_double(0), ctypes.c_double(0)
    L.pgf_profile_read(5, ctypes.byref(c), ctypes.byref(t), ctypes.byref(w))
    assert L.pgf_tc_fault() == 0, "tensor-core kernel reported an expired wait"
    return out, c.value


@pytest.mark.parametrize("at,bt", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 384, 512), (200, 72, 40), (1000, 304, 1024),
                                   (64, 1000, 8), (4096, 1024, 256), (1000, 512, 640), (136, 768, 192),
                                   (520, 256, 1024), (4096, 1024, 512)])
def test_tc_gemm_layouts(ops, at, bt, M, N, K):
    """256-column outputs of two or more 128-row blocks and depth >= 512 run on CTA pairs (one
    256-row MMA per pair, each CTA loading half of B); ragged last blocks included."""
    g = torch.Generator().manual_seed(M + N + K + 7 * at + 3 * bt)
    A = (torch.randn(K, M, generator=g) if at else torch.randn(M, K, generator=g)).bfloat16()
    B = (torch.randn(K, N, generator=g) if bt else torch.randn(N, K, generator=g)).bfloat16()
    ref = (A.double().t() if at else A.double()) @ (B.double() if bt else B.double().t())
    D, n = _tc_launches(lambda: ops.gemm(A.to(DEV), B.to(DEV), a_trans=bool(at), b_trans=bool(bt)))
    assert n == 1, "expected the tcgen05 engine to run"
    assert_close(D, ref, atol=1e-4, rtol=1e-5)


@pytest.mark.parametrize("K", [256, 768])
def test_tc_gemm_epilogue_and_bf16_out(ops, K):
    """Bias + GELU with the pre-activation stored, bf16 output, and accumulation into float32; at
    K = 768 on CTA pairs with a ragged last pair (M = 300) and a ragged column tile (N = 500)."""
    g = torch.Generator().manual_seed(3)
    M, N = 300, 500
    A = torch.randn(M, K, generator=g).bfloat16()
    B = torch.randn(N, K, generator=g).bfloat16()
    bias = torch.randn(N, generator=g)
    z = A.double() @ B.double().t() + bias.double()
    zo = torch.empty(M, N, device=DEV)
    h, n = _tc_launches(lambda: ops.gemm(A.to(DEV), B.to(DEV), bias=bias.to(DEV), epilogue="gelu",
                                         aux_out=zo, out_dtype=torch.bfloat16))
    assert n == 1 and h.dtype == torch.bfloat16
    assert_close(zo, z, atol=1e-4)
    from oracle import pgf_oracle as O
    assert_close(h.float(), O.gelu_tanh(z), atol=2e-2, rtol=1e-2)
    acc = torch.randn(M, N, generator=g)
    out = acc.clone().to(DEV)
    _tc_launches(lambda: ops.gemm(A.to(DEV), B.to(DEV), out=out, accumulate=True))
    assert_close(out, acc.double() + A.double() @ B.double().t(), atol=1e-4)


def test_unaligned_pitch_falls_back_to_simt(ops):
    """A row pitch that is not a multiple of 16 bytes cannot be a TMA operand: the SIMT engine runs."""
    g = torch.Generator().manual_seed(9)
    A = torch.randn(100, 64, generator=g).bfloat16()
    B = torch.randn(64, 300, generator=g).bfloat16()  # stored K x N, pitch 600 B
    ref = A.double() @ B.double()
    D, n = _tc_launches(lambda: ops.gemm(A.to(DEV), B.to(DEV), b_trans=True))
    assert n == 0
    assert_close(D, ref, atol=1e-4, rtol=1e-5)


# ---------------------------------------------------------------------------------------------
# split-K: outputs with few tiles and a deep K (weight gradients) are cut into K slices whose
# float32 partials are summed in slice order by the epilogue pass.
@pytest.mark.parametrize("M,N,K,at,bt", [(1024, 256, 32768, 1, 1), (256, 1024, 8192, 1, 1), (288, 256, 65536, 1, 1),
                                         (300, 40, 5000, 0, 1), (128, 128, 640, 0, 0)])
def test_split_k_bf16_matches_unsplit(ops, M, N, K, at, bt):
    from icml_b200 import _lib
    assert _lib.lib().pgf_gemm_workspace(M, N, K) > 0 or M * N > 128 * 128 * 74
    g = torch.Generator().manual_seed(M + N + K)
    A = (torch.randn(K, M, generator=g) if at else torch.randn(M, K, generator=g)).bfloat16().to(DEV)
    B = (torch.randn(K, N, generator=g) if bt else torch.randn(N, K, generator=g)).bfloat16().to(DEV)
    ref = (A.double().t() if at else A.double()) @ (B.double() if bt else B.double().t())
    acc0 = torch.randn(M, N, generator=g).to(DEV)
    split = ops.gemm(A, B, a_trans=bool(at), b_trans=bool(bt), out=acc0.clone(), accumulate=True)
    plain = ops.gemm(A, B, a_trans=bool(at), b_trans=bool(bt), out=acc0.clone(), accumulate=True, split_k=False)
    assert _lib.lib().pgf_tc_fault() == 0
    # one TMEM accumulator over a very deep K drifts by a few 1e-5 relative (the tensor core's
    # float32 accumulation is not IEEE-exact); the slices, summed in float32, stay closer to exact
    err_split = assert_close(split, ref + acc0.double(), atol=1e-3, rtol=1e-5)
    err_plain = assert_close(plain, ref + acc0.double(), atol=1e-3, rtol=1e-4)
    assert err_split <= err_plain + 1e-3
    again = ops.gemm(A, B, a_trans=bool(at), b_trans=bool(bt), out=acc0.clone(), accumulate=True)
    assert torch.equal(split, again), "split-K must be deterministic"


def test_split_k_epilogues(ops):
    g = torch.Generator().manual_seed(11)
    M, N, K = 256, 200, 8192
    A = torch.randn(M, K, generator=g).bfloat16()
    B = torch.randn(N, K, generator=g).bfloat16()
    bias = torch.randn(N, generator=g)
    z = (A.double() @ B.double().t()) / 64 + bias.double()
    zo = torch.empty(M, N, device=DEV)
    h = ops.gemm(A.to(DEV), B.to(DEV), bias=bias.to(DEV), epilogue="gelu", alpha=1 / 64, aux_out=zo,
                 out_dtype=torch.bfloat16)
    assert_close(zo, z, atol=1e-4)
    from oracle import pgf_oracle as O
    assert_close(h.float(), O.gelu_tanh(z), atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("M,N,K,at,bt", [(512, 16, 65536, 1, 1), (48, 512, 65536, 1, 1), (100, 30, 3000, 0, 0)])
def test_split_k_simt_f32(ops, M, N, K, at, bt):
    """float32 operands (the SIMT engine), split over K, within the float32 parity bound."""
    g = torch.Generator().manual_seed(M * 3 + N + K)
    A = (torch.randn(K, M, generator=g) if at else torch.randn(M, K, generator=g)).to(DEV)
    B = (torch.randn(K, N, generator=g) if bt else torch.randn(N, K, generator=g)).to(DEV)
    ref = (A.double().t() if at else A.double()) @ (B.double() if bt else B.double().t())
    D = ops.gemm(A, B, a_trans=bool(at), b_trans=bool(bt))
    assert_close(D, ref, atol=2e-3, rtol=1e-5)
    assert torch.equal(D, ops.gemm(A, B, a_trans=bool(at), b_trans=bool(bt)))
