"""The JAX front-end's pure-Python parts (no jax needed): mask attributes and slopes.

attnax_b200/ffi/jax_binding.py flattens its tagged ScoreMods into the
attributes the XLA FFI handlers (attnax_ffi.cc) pass to the C ABI; the
result must equal what the torch front-end's build_spec puts in attn_mask_t.
"""

import numpy as np
import pytest
import torch

import attnax_b200 as ax
import oracle as O
from attnax_b200._spec import build_spec
from attnax_b200.ffi import jax_binding as J


@pytest.mark.parametrize("chain", ["none", "causal", "window", "window_sym", "alibi", "window_alibi",
                                   "causal_window"])
def test_mask_attributes_match_the_c_abi_mask(chain):
    H = 8

    def make(m):
        return {
            "none": (None,),
            "causal": (m.causal_mod(),),
            "window": (m.sliding_window_mod(70),),
            "window_sym": (m.sliding_window_mod(50, causal=False),),
            "alibi": (m.alibi_mod(H),),
            "window_alibi": (m.sliding_window_mod(90), m.alibi_mod(H)),
            "causal_window": (m.causal_mod(), m.sliding_window_mod(30, causal=False)),
        }[chain]

    attrs = J.mask_attrs(J.compose_score_mods(*make(J)), H)
    spec = build_spec(ax.compose_score_mods(*make(ax)), None, batch=1, heads_q=H, seq_q=4, seq_kv=4, device="cpu")
    m = spec.struct
    assert attrs["has_band"] == m.has_band
    if m.has_band:
        assert (attrs["band_lo"], attrs["band_hi"]) == (m.band_lo, m.band_hi)
    assert attrs["alibi"] == bool(m.alibi_slopes)


def test_untagged_mods_are_rejected():
    with pytest.raises(NotImplementedError):
        J.mask_attrs(lambda s, b, h, q, kv: s, 4)
    with pytest.raises(ValueError):
        J.mask_attrs(J.alibi_mod(4), 8)
    with pytest.raises(ValueError):
        J.sliding_window_mod(0)


@pytest.mark.parametrize("n", [1, 4, 6, 8, 12, 32])
def test_alibi_slopes_match_the_reference_schedule(n):
    np.testing.assert_allclose(np.float32(J.alibi_slopes(n)), O.alibi_slopes(n), rtol=0, atol=0)
    np.testing.assert_array_equal(np.float32(J.alibi_slopes(n)), ax.score_mods.alibi_slopes(n).numpy())
