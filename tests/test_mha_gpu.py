"""MultiHeadAttention's attention core (attnax_b200.mha.attention_core) against the oracle.

The oracle restates attention.py:340-445 (head split, RoPE, KV-cache
concatenation and update, the KV-head repeat, the boolean window mask with
cache-shifted query positions, standard_attention); the product path keeps
K/V at their own head count and applies the window as a band.
"""

import numpy as np
import pytest
import torch

import attnax_b200 as ax
import oracle as O
from attnax_b200.mha import attention_core
from tests._util import assert_bf16_close, randn

pytestmark = pytest.mark.gpu
DEV = "cuda"


def T(x):
    return torch.tensor(x, dtype=torch.bfloat16, device=DEV)


def npy(t):
    return t.detach().float().cpu().numpy()


def bf16_tables(L, D, base=10000.0):
    """The product's bf16 RoPE tables, the ones ``attention_core`` builds."""
    c, s = ax.rope_cos_sin_table(L, D, base, torch.bfloat16, DEV)
    return npy(c), npy(s)


def test_bf16_rope_tables_match_the_reference_recipe():
    """bf16 tables: inverse frequencies within two bf16 ulps (2^-6 relative) of
    the oracle's op-by-op bf16 recipe (libraries round ``pow`` differently in a
    few entries, and the reciprocal can add one more), and given those
    frequencies, positions, products and cos/sin rounded as the oracle rounds
    them (cos/sin within one bf16 ulp at 1)."""
    D, L, base = 128, 512, 10000.0
    inv = npy(ax.rope_inv_freq(D, base, torch.bfloat16, DEV))
    want_inv = O.rope_inv_freq(D, base, "bfloat16")
    assert np.all(np.abs(inv - want_inv) <= 2.0 ** -6 * np.abs(want_inv))
    cos, sin = bf16_tables(L, D, base)
    freqs = O.bf16_round(np.outer(O.bf16_round(np.arange(L, dtype=np.float32)), inv))
    assert np.abs(cos - O.bf16_round(np.cos(freqs))).max() <= 2.0 ** -8
    assert np.abs(sin - O.bf16_round(np.sin(freqs))).max() <= 2.0 ** -8


@pytest.mark.parametrize("window,rope", [(None, False), (64, True), (None, True)])
def test_self_attention_gqa(window, rope):
    rng = np.random.default_rng(50)
    B, S, Hq, Hkv, D = 2, 300, 8, 2, 128
    q, k, v = (randn(rng, (B, S, h * D), True) for h in (Hq, Hkv, Hkv))
    got = attention_core(T(q), T(k), T(v), num_heads=Hq, num_kv_heads=Hkv, use_rope=rope,
                         rope_max_positions=512, attention_window=window)
    # a bf16 layer rotates with bf16 tables and stores bf16 q/k, as the reference does
    want = O.mha_attention_core(q, k, v, num_heads=Hq, num_kv_heads=Hkv, use_rope=rope, rope_max_positions=512,
                                attention_window=window, activation_dtype="bfloat16",
                                rope_tables=bf16_tables(512, D) if rope else None)
    assert_bf16_close(npy(got), want, f"self window={window} rope={rope}")


def test_prefill_then_decode_with_cache_and_window():
    rng = np.random.default_rng(51)
    B, Hq, Hkv, D, L, W = 2, 8, 2, 128, 512, 96
    cache = ax.init_kv_layer_cache(B, Hkv, D, L, torch.bfloat16)
    ocache = O.init_kv_layer_cache(B, Hkv, D, L)
    tables = bf16_tables(L, D)
    for step, n in enumerate([200, 1, 1, 3]):
        q, k, v = (randn(rng, (B, n, h * D), True) for h in (Hq, Hkv, Hkv))
        pos = np.broadcast_to(np.arange(ocache.length, ocache.length + n)[None], (B, n)).astype(np.int32)
        got, cache = attention_core(T(q), T(k), T(v), num_heads=Hq, num_kv_heads=Hkv, use_rope=True,
                                    rope_max_positions=L, position_ids_q=torch.tensor(pos, device=DEV),
                                    position_ids_kv=torch.tensor(pos, device=DEV), kv_cache=cache,
                                    attention_window=W, base_score_mod=ax.alibi_mod(Hq))
        want, ocache = O.mha_attention_core(q, k, v, num_heads=Hq, num_kv_heads=Hkv, use_rope=True,
                                            rope_max_positions=L, position_ids_q=pos, position_ids_kv=pos,
                                            kv_cache=ocache, attention_window=W, base_score_mod=O.alibi_mod(Hq),
                                            activation_dtype="bfloat16", rope_tables=tables)
        assert cache.length == ocache.length
        assert_bf16_close(npy(got), want, f"cache step {step} ({n} tokens)")


def test_cross_attention_has_no_window():
    rng = np.random.default_rng(52)
    B, Sq, Skv, Hq, Hkv, D = 1, 100, 260, 4, 4, 64
    q = randn(rng, (B, Sq, Hq * D), True)
    k, v = (randn(rng, (B, Skv, Hkv * D), True) for _ in range(2))
    got = attention_core(T(q), T(k), T(v), num_heads=Hq, num_kv_heads=Hkv, attention_window=16,
                         self_attention=False)
    want = O.mha_attention_core(q, k, v, num_heads=Hq, num_kv_heads=Hkv, attention_window=16,
                                self_attention=False)
    assert_bf16_close(npy(got), want, "cross")
