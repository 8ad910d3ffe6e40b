"""CPU checks of the C-ABI boundary: the library loads and exports every symbol of include/pgf.h."""
import os
import re

from tests.conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "pgf.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(pgf_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("pgf_ssm_fwd", "pgf_ssm_bwd", "pgf_rmsnorm_fwd", "pgf_rmsnorm_bwd", "pgf_embedding_bwd",
              "pgf_ffn_bwd", "pgf_lm_head_ce_bwd", "pgf_gemm", "pgf_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from icml_b200 import _lib
    L = _lib.lib()
    missing = [n for n in _declared() if not hasattr(L, n)]
    assert not missing, missing
    # the Python binding declares a signature for each of them
    assert set(_declared()) <= set(_lib.SIGNATURES), set(_declared()) - set(_lib.SIGNATURES)


def test_calls_without_gpu_return_errors_not_crashes():
    """Argument validation runs on the host and reports through pgf_last_error."""
    from icml_b200 import _lib
    L = _lib.lib()
    rc = L.pgf_ssm_fwd(None, None, None, None, None, None, None, None, None, 1, 8, 32, 8, 0, 0, None,
                       0, None)
    assert rc != 0
    assert "d_state" in _lib.last_error()
    rc = L.pgf_rmsnorm_fwd(None, None, None, 4, 16, 1e-6, 0, None)  # rows > 0
    assert rc != 0 and "null" in _lib.last_error()
    assert L.pgf_version() >= 100


def test_boundary_rejects_bad_arguments_before_any_cuda_call():
    """Shape and dtype checks run on the host before any CUDA call, with the reason in
    pgf_last_error; an empty input is a no-op that touches nothing."""
    from icml_b200 import _lib
    L = _lib.lib()
    dummy = 256  # never dereferenced: each call below returns before touching memory or the GPU
    assert L.pgf_rmsnorm_fwd(dummy, dummy, dummy, 4, 5000, 1e-6, 0, None) != 0
    assert "bad shape" in _lib.last_error()
    assert L.pgf_rmsnorm_fwd(dummy, dummy, dummy, 4, 256, 1e-6, 7, None) != 0
    assert "dtype" in _lib.last_error()
    assert L.pgf_rmsnorm_fwd(None, None, None, 0, 256, 1e-6, 0, None) == 0
    assert L.pgf_embedding_fwd(None, None, None, 0, 10, 8, 0, None) != 0  # null before the empty check
    assert "null" in _lib.last_error()
    assert L.pgf_embedding_fwd(dummy, dummy, dummy, 0, 10, 8, 0, None) == 0
