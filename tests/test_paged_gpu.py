"""Paged KV cache and paged decode parity on the GPU, against the oracle."""

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


def npy(t):
    return t.detach().float().cpu().numpy()


def test_golden_paged_cache_ops_bit_exact():
    d = dict(np.load(G / "golden_paged.npz"))
    nseq = len(d["paged_lens"])
    cache = ax.init_paged_kv_cache(num_blocks=12, block_size=4, num_kv_heads=2, head_dim=8,
                                   batch_size=nseq, max_blocks_per_seq=4, dtype=torch.float32)
    perm, used = d["paged_perm"], 0
    for s, n in enumerate(d["paged_lens"]):
        cache, got = ax.allocate_blocks(cache, sequence_idx=s, num_new_tokens=int(n),
                                        free_block_ids=torch.tensor(perm[used:]))
        used += got
        if n:
            cache = ax.append_kv(cache, s, torch.tensor(d[f"paged_newk_{s}"], device=DEV),
                                 torch.tensor(d[f"paged_newv_{s}"], device=DEV))
    np.testing.assert_array_equal(cache.block_table.cpu().numpy(), d["paged_block_table"])
    np.testing.assert_array_equal(cache.seq_lengths.cpu().numpy(), d["paged_seq_lengths"])
    np.testing.assert_array_equal(cache.key_pool.cpu().numpy(), d["paged_key_pool"])
    np.testing.assert_array_equal(cache.value_pool.cpu().numpy(), d["paged_value_pool"])
    for s in range(nseq):
        k, v, n = ax.gather_kv(cache, s)
        np.testing.assert_array_equal(k.cpu().numpy(), d[f"paged_gather_k_{s}"])
        np.testing.assert_array_equal(v.cpu().numpy(), d[f"paged_gather_v_{s}"])
        for kind in ("decode", "prefill"):
            q = torch.tensor(d[f"paged_q_{kind}"][s], device=DEV)
            out = ax.paged_attention(q, cache, s)
            assert_fp32_close(npy(out), d[f"paged_out_{kind}_{s}"], f"{kind} seq {s}", atol=2e-5)


def test_append_unallocated_raises():
    cache = ax.init_paged_kv_cache(num_blocks=2, block_size=4, num_kv_heads=2, head_dim=8,
                                   batch_size=1, max_blocks_per_seq=2, dtype=torch.float32)
    with pytest.raises(ValueError, match="unallocated"):
        ax.append_kv(cache, 0, torch.zeros(1, 2, 8, device=DEV), torch.zeros(1, 2, 8, device=DEV))
    with pytest.raises(ValueError):
        ax.allocate_blocks(cache, sequence_idx=0, num_new_tokens=9, free_block_ids=torch.arange(1))


def _random_cache(rng, lens, hkv, D=128, bs=16, extra=5, dtype=torch.bfloat16):
    pages = [(n + bs - 1) // bs for n in lens]
    nb = sum(pages) + extra
    perm = rng.permutation(nb)
    table = np.full((len(lens), max(max(pages), 1)), -1, np.int32)
    o = 0
    for s, n in enumerate(pages):
        table[s, :n] = perm[o:o + n]
        o += n
    kp = randn(rng, (nb, bs, hkv, D), True)
    vp = randn(rng, (nb, bs, hkv, D), True)
    cache = ax.PagedKVCache(torch.tensor(kp, dtype=dtype, device=DEV), torch.tensor(vp, dtype=dtype, device=DEV),
                            torch.tensor(table, device=DEV), torch.tensor(lens, dtype=torch.int32, device=DEV))
    return cache, O.PagedKVCache(kp, vp, table, np.array(lens, np.int32))


@pytest.mark.parametrize("hq,hkv,sq", [(32, 8, 1), (8, 8, 1), (16, 8, 1), (64, 8, 1), (32, 8, 2)])
def test_decode_matches_oracle(hq, hkv, sq):
    rng = np.random.default_rng(hq + sq)
    lens = [0, 1, 15, 16, 17, 2047, 2048, 2049, 5000]
    cache, oc = _random_cache(rng, lens, hkv)
    q = randn(rng, (len(lens), hq, sq, 128), True)
    got = npy(ax.paged_attention_batched(torch.tensor(q, dtype=torch.bfloat16, device=DEV), cache))
    want = O.paged_attention_batched(q, oc)
    assert_bf16_close(got, want, f"decode hq={hq} hkv={hkv} sq={sq}")


@pytest.mark.parametrize("bs,hq,hkv,sq,dtype", [
    (8, 32, 8, 1, torch.bfloat16),     # scalar consumers (block_size not a multiple of 16)
    (32, 32, 8, 1, torch.bfloat16),    # tensor-core consumers, two 16-token groups per page
    (64, 64, 2, 1, torch.bfloat16),    # 32 rows per kv head: two row groups; 32-token TMA units
    (48, 32, 8, 1, torch.bfloat16),    # three 16-token TMA units per page
    (16, 24, 2, 2, torch.float16),     # 24 rows (12 heads x 2 positions), fp16
])
def test_decode_block_sizes_rows_dtypes_nan_slots(bs, hq, hkv, sq, dtype):
    """Unused slots of each sequence's last page hold NaN (a pool that was
    never written there); only tokens < seq_len may reach the output."""
    rng = np.random.default_rng(bs + hq + sq)
    lens = [1, bs - 3, bs + 5, 3 * bs + 1, 2048 + 7, 4099]
    cache, oc = _random_cache(rng, lens, hkv, bs=bs, dtype=dtype)
    kp, vp = cache.key_pool.clone(), cache.value_pool.clone()
    table = oc.block_table
    for s_, n in enumerate(lens):
        if n % bs:
            last = table[s_, (n - 1) // bs]
            kp[last, n % bs:] = float("nan")
            vp[last, n % bs:] = float("nan")
    cache = ax.PagedKVCache(kp, vp, cache.block_table, cache.seq_lengths)
    q = randn(rng, (len(lens), hq, sq, 128), True)
    got = npy(ax.paged_attention_batched(torch.tensor(q, dtype=dtype, device=DEV), cache))
    assert np.isfinite(got).all()
    want = O.paged_attention_batched(q, oc)
    assert_bf16_close(got, want, f"decode bs={bs} hq={hq} hkv={hkv} sq={sq} {dtype}")


def test_decode_single_sequence_api():
    rng = np.random.default_rng(9)
    cache, oc = _random_cache(rng, [700, 33], 8)
    q = randn(rng, (32, 1, 128), True)
    got = npy(ax.paged_attention(torch.tensor(q, dtype=torch.bfloat16, device=DEV), cache, 1))
    assert_bf16_close(got, O.paged_attention(q, oc, 1), "single")


def test_decode_with_score_mod_uses_gather_path():
    rng = np.random.default_rng(10)
    cache, oc = _random_cache(rng, [300], 2, D=64, bs=16)
    q = randn(rng, (4, 3, 64), True)
    got = npy(ax.paged_attention(torch.tensor(q, dtype=torch.bfloat16, device=DEV), cache, 0,
                                 score_mod=ax.alibi_mod(4)))
    assert_bf16_close(got, O.paged_attention(q, oc, 0, score_mod=O.alibi_mod(4)), "alibi")


def test_minus_one_entries_select_the_last_pool_page():
    """A -1 entry inside a sequence's length reads the pool's last page, as
    the reference's pool[block_ids] does (negative ids count from the end)."""
    rng = np.random.default_rng(40)
    cache, oc = _random_cache(rng, [70, 40], 8)
    table = oc.block_table.copy()
    table[0, 2] = -1
    table[1, 0] = -1
    oc = O.PagedKVCache(oc.key_pool, oc.value_pool, table, oc.seq_lengths)
    cache = ax.PagedKVCache(cache.key_pool, cache.value_pool, torch.tensor(table, device=DEV), cache.seq_lengths)
    for s in range(2):
        k, v, _ = ax.gather_kv(cache, s)
        wk, wv, _ = O.gather_kv(oc, s)
        np.testing.assert_array_equal(npy(k), wk)
        np.testing.assert_array_equal(npy(v), wv)
    q = randn(rng, (2, 32, 1, 128), True)
    got = npy(ax.paged_attention_batched(torch.tensor(q, dtype=torch.bfloat16, device=DEV), cache))
    assert_bf16_close(got, O.paged_attention_batched(q, oc), "-1 entries")


def test_max_context_below_a_length_is_reported():
    """max_context is the caller's bound; a longer sequence attends only the
    splits that bound plans (its first 2048 tokens here) and the decode leaves
    a notice in the device status instead of failing silently."""
    from attnax_b200 import _lib
    from attnax_b200.paged import paged_decode_raw

    rng = np.random.default_rng(41)
    lens = [5000, 300]
    cache, oc = _random_cache(rng, lens, 8)
    _lib.device_status()  # clear
    q = randn(rng, (2, 32, 1, 128), True)
    got = npy(paged_decode_raw(torch.tensor(q, dtype=torch.bfloat16, device=DEV), cache, max_context=2048))
    assert _lib.device_status() == _lib.NOTICE_CONTEXT_OVERRUN
    assert _lib.device_status() == 0  # read and cleared
    cut = O.PagedKVCache(oc.key_pool, oc.value_pool, oc.block_table, np.array([2048, 300], np.int32))
    assert_bf16_close(got, O.paged_attention_batched(q, cut), "first splits only")
    with pytest.raises(ValueError):
        ax.paged_attention_batched(torch.tensor(q, dtype=torch.bfloat16, device=DEV),
                                   ax.PagedKVCache(cache.key_pool, cache.value_pool, cache.block_table[:, :100],
                                                   cache.seq_lengths))
