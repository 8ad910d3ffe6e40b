"""Shared parity helpers for the tests (checker side only)."""
import torch

# float32 bound of the north star: max-abs 1e-5, relative 1e-4 (of the reference's magnitude)
F32_ATOL = 1e-5
F32_RTOL = 1e-4
# bf16 activations against the float32/float64 oracle
BF16_RTOL = 3e-2


def assert_close(got, ref, atol=F32_ATOL, rtol=F32_RTOL, name=""):
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    assert got.shape == ref.shape, f"{name}: shape {tuple(got.shape)} vs {tuple(ref.shape)}"
    if ref.numel() == 0:
        return 0.0
    err = (got - ref).abs().max().item()
    lim = atol + rtol * ref.abs().max().item()
    assert err <= lim, f"{name}: max abs err {err:.3e} > {lim:.3e} (ref max {ref.abs().max().item():.3e})"
    return err


def rel_err(got, ref):
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    return ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
