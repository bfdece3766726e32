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


def assert_bf16_close(got, want, what="", scale_with_max=False):
    mx, rel = errors(got, want)
    lim = BF16_MAX_ABS * (max(1.0, float(np.abs(want).max())) if scale_with_max else 1.0)
    assert mx <= lim and rel <= BF16_MEAN_REL, f"{what}: max-abs {mx:.3e} (lim {lim:.1e}), mean-rel {rel:.3e}"


def assert_fp32_close(got, want, what="", atol=FP32_MAX_ABS):
    mx, rel = errors(got, want)
    assert mx <= atol, f"{what}: max-abs {mx:.3e} > {atol:.1e} (mean-rel {rel:.2e})"
