"""Decode over the contiguous per-layer KV cache on the GPU, against the oracle."""

import pathlib

import numpy as np
import pytest
import torch

import attnax_b200 as ax
import oracle as O
from tests._util import assert_bf16_close, assert_fp32_close, randn

pytestmark = pytest.mark.gpu
DEV = "cuda"
G = pathlib.Path(__file__).resolve().parent / "golden"


def test_golden_kv_cache_fp32():
    """The reference's own cache contents and decode outputs (head_dim 16,
    fp32: the flash kernel on the [:length] views)."""
    d = dict(np.load(G / "golden_kvcache.npz"))
    B, Hkv, L, D = d["kvc_keys"].shape
    c = ax.init_kv_layer_cache(B, Hkv, D, L, torch.float32)
    for k, v in (("kvc_k1", "kvc_v1"), ("kvc_k2", "kvc_v2")):
        c = ax.update_kv_layer_cache(c, torch.tensor(d[k], device=DEV), torch.tensor(d[v], device=DEV), c.length)
    assert c.length == int(d["kvc_len"])
    np.testing.assert_array_equal(c.keys.cpu().numpy(), d["kvc_keys"])
    for sq in (1, 3):
        got = ax.kv_cache_attention(torch.tensor(d[f"kvc_q{sq}"], device=DEV), c)
        assert_fp32_close(got.cpu().numpy(), d[f"kvc_out{sq}"], f"golden sq={sq}")


def _cache(rng, B, Hkv, L, n, dtype):
    """A cache holding ``n`` positions; the slots past ``n`` hold NaN (never
    written), which must not reach the output."""
    k = randn(rng, (B, Hkv, L, 128), True)
    v = randn(rng, (B, Hkv, L, 128), True)
    c = ax.init_kv_layer_cache(B, Hkv, 128, L, dtype)
    c.keys.fill_(float("nan"))
    c.values.fill_(float("nan"))
    c = ax.update_kv_layer_cache(c, torch.tensor(k[:, :, :n], dtype=dtype, device=DEV),
                                 torch.tensor(v[:, :, :n], dtype=dtype, device=DEV), 0)
    return c, O.KVLayerCache(k, v, n)


@pytest.mark.parametrize("B,Hq,Hkv,L,n,sq,dtype", [
    (3, 32, 8, 4096, 3001, 1, torch.bfloat16),   # 32-token TMA units, GQA 4
    (2, 32, 1, 1040, 1040, 1, torch.bfloat16),   # MQA: 32 rows per kv head (two row groups), full cache
    (2, 8, 2, 528, 17, 2, torch.float16),        # two positions per query (8 rows), fp16, short history
])
def test_decode_kernel_matches_oracle(B, Hq, Hkv, L, n, sq, dtype):
    rng = np.random.default_rng(L + n)
    c, oc = _cache(rng, B, Hkv, L, n, dtype)
    q = randn(rng, (B, Hq, sq, 128), True)
    got = ax.kv_cache_attention(torch.tensor(q, dtype=dtype, device=DEV), c)
    got = got.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert_bf16_close(got, O.kv_cache_attention(q, oc), f"kv decode B{B} Hq{Hq} Hkv{Hkv} L{L} n{n} sq{sq}")


def test_decode_odd_max_len_and_score_mod_take_flash_path():
    rng = np.random.default_rng(77)
    c, oc = _cache(rng, 2, 2, 1000, 999, torch.bfloat16)  # max_len not a multiple of 16
    q = randn(rng, (2, 4, 1, 128), True)
    got = ax.kv_cache_attention(torch.tensor(q, dtype=torch.bfloat16, device=DEV), c)
    assert_bf16_close(got.float().cpu().numpy(), O.kv_cache_attention(q, oc), "odd max_len")
    got = ax.kv_cache_attention(torch.tensor(q, dtype=torch.bfloat16, device=DEV), c, score_mod=ax.alibi_mod(4))
    want = O.kv_cache_attention(q, oc, score_mod=O.alibi_mod(4))
    assert_bf16_close(got.float().cpu().numpy(), want, "alibi")
