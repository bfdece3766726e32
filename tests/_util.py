"""Helpers shared by the parity tests."""

import numpy as np

import oracle as O

BF16_MAX_ABS = 2e-2     # bf16 outputs vs the fp32 reference, max-abs
BF16_MEAN_REL = 1e-2    # bf16 outputs vs the fp32 reference, mean relative (L1) error
FP32_MAX_ABS = 1e-4     # fp32 outputs vs the fp32 reference


def randn(rng, shape, bf16=False):
    x = rng.standard_normal(shape, dtype=np.float32)
    return O.bf16_round(x) if bf16 else x


def errors(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    d = np.abs(got - want)
    return float(d.max()) if d.size else 0.0, float(d.sum() / max(np.abs(want).sum(), 1e-30))


def assert_bf16_close(got, want, what=""):
    mx, rel = errors(got, want)
    print(f"[parity] {what}: max-abs {mx:.3e} mean-rel {rel:.3e} max|ref| {float(np.abs(want).max()):.3e}")
    assert mx <= BF16_MAX_ABS and rel <= BF16_MEAN_REL, f"{what}: max-abs {mx:.3e}, mean-rel {rel:.3e}"


# Storing a value in bf16 alone moves it by up to half an ulp, i.e. up to
# 2^-8 of its magnitude (8 significant bits).  Gradients reach |x| ~ 8 in the
# parity tests, where that rounding alone (0.031) exceeds the 2e-2 bar, so
# gradient checks allow the bar plus the storage rounding of each element.
BF16_STORE_REL = 2.0 ** -8


def assert_bf16_grad_close(got, want, what=""):
    """bf16 gradients: |got - want| <= 2e-2 + 2^-8 |want| per element, mean-rel <= 1e-2."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    mx, rel = errors(got, want)
    excess = float(np.max(np.abs(got - want) - BF16_STORE_REL * np.abs(want))) if want.size else 0.0
    print(f"[parity] {what}: max-abs {mx:.3e} mean-rel {rel:.3e} max|ref| {float(np.abs(want).max()):.3e} "
          f"max(|err| - 2^-8|ref|) {excess:.3e}")
    assert excess <= BF16_MAX_ABS and rel <= BF16_MEAN_REL, (
        f"{what}: max(|err| - 2^-8|ref|) {excess:.3e}, mean-rel {rel:.3e}")


def assert_fp32_close(got, want, what="", atol=FP32_MAX_ABS):
    mx, rel = errors(got, want)
    print(f"[parity] {what}: max-abs {mx:.3e} mean-rel {rel:.3e} max|ref| {float(np.abs(want).max()):.3e}")
    assert mx <= atol, f"{what}: max-abs {mx:.3e} > {atol:.1e} (mean-rel {rel:.2e})"
