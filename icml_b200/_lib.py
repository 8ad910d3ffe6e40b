"""ctypes binding of the in-tree libpgf.so (declarations in include/pgf.h).

There is no fallback: if the library is missing or cannot be loaded, every operator raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p, c_char_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libpgf.so")

_lock = threading.Lock()
_lib = None

P = c_void_p
I64 = c_int64


class Epilogue(ctypes.Structure):
    """pgf_epilogue of include/pgf.h."""
    _fields_ = [
        ("kind", c_int), ("alpha", c_float), ("bias", c_void_p),
        ("aux", c_void_p), ("aux_dtype", c_int), ("ld_aux", c_int64),
        ("aux_out", c_void_p), ("aux_out_dtype", c_int), ("ld_aux_out", c_int64),
        ("addend", c_void_p), ("addend_dtype", c_int), ("ld_addend", c_int64),
        ("accumulate", c_int),
    ]


# name -> (restype, argtypes); mirrors include/pgf.h
SIGNATURES = {
    "pgf_last_error": (c_char_p, []),
    "pgf_version": (c_int, []),
    "pgf_launch_count": (ctypes.c_longlong, []),
    "pgf_profile": (c_int, [c_int]),
    "pgf_tc_fault": (c_int, []),
    "pgf_profile_read": (c_int, [c_int, ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_double),
                                 ctypes.POINTER(ctypes.c_double)]),
    "pgf_rmsnorm_fwd": (c_int, [P, P, P, I64, I64, c_float, c_int, P]),
    "pgf_rmsnorm_fwd_res": (c_int, [P, P, P, P, P, I64, I64, c_float, c_int, P]),
    "pgf_rmsnorm_bwd_add": (c_int, [P, P, P, P, P, P, c_int, I64, I64, c_float, c_int, P, c_size_t, P]),
    "pgf_rmsnorm_bwd_workspace": (c_size_t, [I64, I64]),
    "pgf_rmsnorm_bwd": (c_int, [P, P, P, P, P, c_int, I64, I64, c_float, c_int, P, c_size_t, P]),
    "pgf_rmsnorm_bwd_noalloc": (c_int, [P, P, P, P, P, c_int, I64, I64, c_float, c_int, P]),
    "pgf_embedding_fwd": (c_int, [P, P, P, I64, I64, I64, c_int, P]),
    "pgf_embedding_bwd_workspace": (c_size_t, [I64, I64, I64]),
    "pgf_embedding_bwd": (c_int, [P, P, P, c_int, I64, I64, I64, c_int, P, c_size_t, P]),
    "pgf_gemm": (c_int, [I64, I64, I64, P, c_int, I64, c_int, P, c_int, I64, c_int, P, c_int, I64,
                         ctypes.POINTER(Epilogue), P]),
    "pgf_gemm_workspace": (c_size_t, [I64, I64, I64]),
    "pgf_gemm_ex": (c_int, [I64, I64, I64, P, c_int, I64, c_int, P, c_int, I64, c_int, P, c_int, I64,
                            ctypes.POINTER(Epilogue), P, c_size_t, P]),
    "pgf_colsum_workspace": (c_size_t, [I64, I64]),
    "pgf_colsum": (c_int, [P, c_int, I64, I64, I64, P, c_int, P, c_size_t, P]),
    "pgf_ffn_workspace": (c_size_t, [I64, I64, I64, I64, c_int, c_int]),
    "pgf_ffn_fwd": (c_int, [P, P, P, P, P, P, I64, I64, I64, I64, c_int, c_int, P, c_size_t, P]),
    "pgf_ffn_fwd_res": (c_int, [P, P, P, P, P, P, P, I64, I64, I64, I64, c_int, c_int, P, c_size_t, P]),
    "pgf_ffn_bwd": (c_int, [P, P, P, P, P, P, P, P, P, P, c_int, I64, I64, I64, I64, c_int, c_int,
                            P, c_size_t, P]),
    "pgf_lm_head_workspace": (c_size_t, [I64, I64, I64, c_int]),
    "pgf_lm_head_fwd": (c_int, [P, P, P, I64, I64, I64, c_int, P, c_size_t, P]),
    "pgf_lm_head_bwd": (c_int, [P, P, P, P, P, c_int, I64, I64, I64, c_int, P, c_size_t, P]),
    "pgf_lm_head_ce_workspace": (c_size_t, [I64, I64, I64, c_int]),
    "pgf_lm_head_ce_fwd": (c_int, [P, P, P, P, P, I64, I64, I64, c_int, P, c_size_t, P]),
    "pgf_lm_head_ce_bwd": (c_int, [P, P, P, P, c_float, P, P, c_int, I64, I64, I64, c_int, P,
                                   c_size_t, P]),
    "pgf_ssm_workspace": (c_size_t, [I64, I64, I64, I64, c_int, c_int]),
    "pgf_ssm_fwd": (c_int, [P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, c_int, c_int, P,
                            c_size_t, P]),
    "pgf_ssm_bwd": (c_int, [P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, c_int, I64, I64,
                            I64, I64, c_int, c_int, P, c_size_t, P]),
    "pgf_ssm_saved_size": (c_size_t, [I64, I64, I64, I64]),
    "pgf_ssm_fwd_save": (c_int, [P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, c_int, c_int, P, c_size_t, P]),
    "pgf_ssm_bwd_saved": (c_int, [P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, c_int, I64, I64,
                                  I64, I64, c_int, c_int, P, c_size_t, P]),
    "pgf_ssm_fwd_begin": (c_int, [P] * 6 + [I64] * 4 + [c_int, P, c_size_t, P]),
    "pgf_ssm_fwd_finish": (c_int, [P] * 9 + [I64] * 4 + [c_int, c_int, P, c_size_t, P]),
    "pgf_ssm_fwd_finish_states": (c_int, [P] * 9 + [I64] * 4 + [c_int, c_int, P, c_size_t, P]),
    "pgf_ssm_bwd_begin": (c_int, [P] * 11 + [I64] * 4 + [c_int, c_int, P, c_size_t, P]),
    "pgf_ssm_bwd_finish": (c_int, [P] * 19 + [c_int] + [I64] * 4 + [c_int, c_int, P, c_size_t, P]),
    "pgf_mamba_mixer_workspace": (c_size_t, [I64, I64, I64, I64, I64, I64, I64, c_int, c_int]),
    "pgf_mamba_mixer_fwd": (c_int, [P] * 11 + [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_mamba_mixer_bwd": (c_int, [P] * 21 + [c_int] + [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_mamba_mixer_saved_size": (c_size_t, [I64] * 7 + [c_int]),
    "pgf_mamba_mixer_fwd_save": (c_int, [P] * 12 + [c_size_t] + [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_mamba_mixer_bwd_saved": (c_int, [P] * 21 + [c_int, P, c_size_t] + [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_ssm_summary": (c_int, [P, P, P, P, P, P, P, I64, I64, I64, I64, c_int, P, c_size_t, P]),
    "pgf_ssm_bwd_summary": (c_int, [P, P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, c_int, c_int, P,
                                    c_size_t, P]),
    "pgf_adamw_step": (c_int, [P, P, P, P, I64, c_float, c_float, c_float, c_float, c_float, P, P, P]),
    "pgf_adamw_step_multi": (c_int, [P, P, P, I64, P, P, P, c_int, c_float, c_float, c_float, c_float, c_float,
                                     P, P, P]),
    "pgf_gather_multi": (c_int, [P, I64, P, P, P, c_int, P]),
    "pgf_grad_norm_workspace": (c_size_t, [I64]),
    "pgf_rmsnorm_jvp": (c_int, [P, P, P, P, P, P, I64, I64, c_float, c_int, P]),
    "pgf_ssm_states_size": (c_size_t, [I64] * 4),
    "pgf_mamba_mixer_states_size": (c_size_t, [I64] * 7),
    "pgf_mamba_mixer_fwd_states": (c_int, [P] * 12 + [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_mamba_mixer_fwd_save_states": (c_int, [P] * 13 + [c_size_t] + [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_ssm_fwd_states": (c_int, [P] * 9 + [I64] * 4 + [c_int, c_int, P, c_size_t, P]),
    "pgf_ssm_fwd_save_states": (c_int, [P] * 9 + [I64] * 4 + [c_int, c_int, P, c_size_t, P]),
    "pgf_ffn_jvp_workspace": (c_size_t, [I64, I64, I64, I64, c_int]),
    "pgf_ffn_jvp": (c_int, [P] * 12 + [I64] * 4 + [c_int, c_int, P, c_size_t, P]),
    "pgf_frechet_jvp_workspace": (c_size_t, [I64, I64, I64]),
    "pgf_ssm_state_hvp_workspace": (c_size_t, [I64, I64, I64, I64, c_int]),
    "pgf_ssm_state_hvp": (c_int, [P] * 9 + [I64] * 4 + [c_int, P, c_size_t, P]),
    "pgf_frechet_jvp": (c_int, [P] * 13 + [I64] * 3 + [P, c_size_t, P]),
    "pgf_grad_norm": (c_int, [P, I64, P, c_float, P, P, c_size_t, P]),
    "pgf_mamba_mixer_fwd_seg": (c_int, [P] * 17 + [c_size_t] + [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_mamba_mixer_fwd_begin": (c_int, [P] * 13 + [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_mamba_mixer_fwd_finish": (c_int, [P] * 14 + [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_mamba_mixer_bwd_seg": (c_int, [P] * 13 + [c_size_t] + [P] * 2 + [P] * 9 + [P] * 4 + [c_int] + [I64] * 7 +
                                [c_int, P, c_size_t, P]),
    "pgf_mamba_mixer_bwd_begin": (c_int, [P] * 13 + [c_size_t] + [P] * 3 + [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_mamba_mixer_bwd_finish": (c_int, [P] * 13 + [c_size_t] + [P] * 2 + [P] * 9 + [P] * 2 + [c_int] +
                                   [I64] * 7 + [c_int, P, c_size_t, P]),
    "pgf_ssm_compose_ranks_fwd": (c_int, [P, I64, c_int, c_int, P, c_int, P, I64, I64, I64, P]),
    "pgf_ssm_compose_ranks_bwd": (c_int, [P, I64, c_int, c_int, P, c_int, P, P, I64, I64, I64, P]),
}


def lib():
    """Load libpgf.so once and declare every exported symbol's signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m icml_b200.build`")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    msg = lib().pgf_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed (code {rc}): {last_error()}")
