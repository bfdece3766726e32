"""Pins the numpy oracle to the reference.

Two kinds of evidence: the golden vectors produced by running the
reference's own source (``tests/golden/make_golden.py``), and the
known-answer assertions of the reference's test suite
(tests/test_kernels.py, tests/test_advanced_kernels.py), restated here
against the oracle.
"""

import pathlib

import numpy as np
import pytest

import oracle as O

G = pathlib.Path(__file__).resolve().parent / "golden"


def load(name):
    return dict(np.load(G / f"golden_{name}.npz"))


# --------------------------------------------------------------- golden ----

def _mods(d):
    H = d["mods_q"].shape[1]
    ids, pref, bias = d["mods_ids"], d["mods_pref"], d["mods_bias"]
    return {
        "none": None,
        "causal": O.causal_mod(),
        "window4": O.sliding_window_mod(4),
        "window3_sym": O.sliding_window_mod(3, causal=False),
        "alibi": O.alibi_mod(H),
        "prefix": O.prefix_lm_mod(pref),
        "document": O.document_mask_mod(ids),
        "bias": O.additive_bias_mod(bias),
        "window4_alibi": O.compose_score_mods(O.sliding_window_mod(4), O.alibi_mod(H)),
        "document_causal": O.compose_score_mods(O.document_mask_mod(ids), O.causal_mod()),
        "maskmod_causal": O.mask_mod_to_score_mod(lambda b, h, q, kv: kv <= q),
    }


@pytest.mark.parametrize("name", ["none", "causal", "window4", "window3_sym", "alibi", "prefix",
                                  "document", "bias", "window4_alibi", "document_causal",
                                  "maskmod_causal"])
def test_standard_attention_matches_reference_golden(name):
    d = load("mods")
    out = O.standard_attention(d["mods_q"], d["mods_k"], d["mods_v"], score_mod=_mods(d)[name])
    np.testing.assert_allclose(out, d[f"mods_out_{name}"], atol=2e-6, rtol=1e-5)


def test_fully_masked_row_is_mean_of_v():
    d = load("mods")
    out = O.standard_attention(d["mods_q"], d["mods_k"], d["mods_v"], mask=d["mask_fully"])
    np.testing.assert_allclose(out, d["mods_out_mask_fully"], atol=2e-6, rtol=1e-5)
    np.testing.assert_allclose(out[0, :, 3], d["mods_v"][0].mean(axis=1), atol=1e-6)


def test_padding_mask_with_alibi_golden():
    d = load("mods")
    m = O.make_padding_mask(d["mask_pad_ids"])
    out = O.standard_attention(d["mods_q"], d["mods_k"], d["mods_v"], mask=m,
                               score_mod=O.alibi_mod(d["mods_q"].shape[1]))
    np.testing.assert_allclose(out, d["mods_out_mask_pad_alibi"], atol=2e-6, rtol=1e-5)


def test_raw_mods_and_masks_golden():
    d = load("mods")
    H = d["raw_alibi"].shape[1]
    b, h, q, kv = O.position_indices(1, H, 8, 8)
    np.testing.assert_array_equal(
        O.alibi_mod(H)(np.zeros((1, H, 8, 8), np.float32), b, h, q, kv), d["raw_alibi"])
    b, h, q, kv = O.position_indices(1, 1, 6, 6)
    np.testing.assert_array_equal(
        O.prefix_lm_mod([3])(np.zeros((1, 1, 6, 6), np.float32), b, h, q, kv), d["raw_prefix"])
    for n in (1, 4, 6, 8, 12, 16, 32):
        np.testing.assert_array_equal(O.alibi_slopes(n), d[f"alibi_slopes_{n}"])
    np.testing.assert_array_equal(O.make_sliding_window_mask(6, window_size=3), d["mask_window_6_3"])
    np.testing.assert_array_equal(O.make_sliding_window_mask(5, window_size=2, causal=False),
                                  d["mask_window_5_2_sym"])
    np.testing.assert_array_equal(O.make_sliding_window_mask(7, 9, window_size=3),
                                  d["mask_window_7_9_3"])
    np.testing.assert_array_equal(O.make_causal_mask(5), d["mask_causal_5"])
    np.testing.assert_array_equal(O.make_document_mask(d["mods_ids"]), d["mask_document"])
    np.testing.assert_array_equal(
        O.mask_mod_to_boolean_mask(lambda b, h, q, kv: kv <= q, batch=1, num_heads=2,
                                   seq_q=4, seq_kv=4), d["mask_boolean_causal"])


def test_blockwise_golden():
    d = load("blockwise")
    q, k, v = d["me_q"], d["me_k"], d["me_v"]
    np.testing.assert_allclose(O.standard_attention(q, k, v), d["me_std"], atol=2e-6, rtol=1e-5)
    np.testing.assert_allclose(O.memory_efficient_attention(q, k, v, block_size=32), d["me_b32"],
                               atol=2e-6, rtol=1e-5)
    np.testing.assert_allclose(
        O.memory_efficient_attention(q, k, v, score_mod=O.causal_mod(), block_size=32),
        d["me_b32_causal"], atol=2e-6, rtol=1e-5)
    np.testing.assert_allclose(d["flash_cpu_b32_causal"], d["me_b32_causal"], atol=0)
    np.testing.assert_allclose(O.standard_attention(q, k, v), d["pallas_cpu"], atol=1e-5)
    qr, kr, vr = d["me_rag_q"], d["me_rag_k"], d["me_rag_v"]
    np.testing.assert_allclose(
        O.memory_efficient_attention(qr, kr, vr, score_mod=O.alibi_mod(2), block_size=32),
        d["me_rag_b32_alibi"], atol=2e-6, rtol=1e-5)
    np.testing.assert_allclose(
        O.memory_efficient_attention(qr, kr, vr, score_mod=O.sliding_window_mod(20), block_size=32),
        d["me_rag_b32_window"], atol=2e-6, rtol=1e-5)


def test_gqa_bf16_golden():
    d = load("gqa_bf16")
    q, k, v = d["gqa_q"], d["gqa_k"], d["gqa_v"]
    H = q.shape[1]
    out = O.gqa_attention(q, k, v, score_mod=O.compose_score_mods(O.sliding_window_mod(64),
                                                                  O.alibi_mod(H)))
    np.testing.assert_allclose(out, d["gqa_window64_alibi"], atol=3e-6, rtol=1e-5)
    out = O.gqa_attention(q, k, v, score_mod=O.compose_score_mods(
        O.document_mask_mod(d["gqa_docs"]), O.causal_mod()))
    np.testing.assert_allclose(out, d["gqa_document_causal"], atol=3e-6, rtol=1e-5)


def test_paged_golden():
    d = load("paged")
    nseq = len(d["paged_lens"])
    cache = O.init_paged_kv_cache(num_blocks=12, block_size=4, num_kv_heads=2, head_dim=8,
                                  batch_size=nseq, max_blocks_per_seq=4)
    perm, used = d["paged_perm"], 0
    for s, n in enumerate(d["paged_lens"]):
        cache, got = O.allocate_blocks(cache, sequence_idx=s, num_new_tokens=int(n),
                                       free_block_ids=perm[used:])
        used += got
        if n:
            cache = O.append_kv(cache, s, d[f"paged_newk_{s}"], d[f"paged_newv_{s}"])
    np.testing.assert_array_equal(cache.block_table, d["paged_block_table"])
    np.testing.assert_array_equal(cache.seq_lengths, d["paged_seq_lengths"])
    np.testing.assert_array_equal(cache.key_pool, d["paged_key_pool"])
    np.testing.assert_array_equal(cache.value_pool, d["paged_value_pool"])
    for s in range(nseq):
        k, v, n = O.gather_kv(cache, s)
        np.testing.assert_array_equal(k, d[f"paged_gather_k_{s}"])
        np.testing.assert_array_equal(v, d[f"paged_gather_v_{s}"])
        for kind in ("decode", "prefill"):
            out = O.paged_attention(d[f"paged_q_{kind}"][s], cache, s)
            np.testing.assert_allclose(out, d[f"paged_out_{kind}_{s}"], atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("P", [2, 4])
@pytest.mark.parametrize("name", ["none", "causal", "alibi"])
def test_ring_partitioned_matches_bound_axis_golden(P, name):
    d = load("ring")
    q, k, v = d["ring_q"], d["ring_k"], d["ring_v"]
    mod = {"none": None, "causal": O.causal_mod(), "alibi": O.alibi_mod(q.shape[1])}[name]
    out = O.ring_attention_partitioned(q, k, v, P, score_mod=mod)
    np.testing.assert_allclose(out, d[f"ring_P{P}_{name}"], atol=2e-6, rtol=1e-5)
    ref = O.standard_attention(q, k, v, score_mod=mod)
    np.testing.assert_allclose(out, ref, atol=1e-5, rtol=1e-5)


def test_kv_layer_cache_golden():
    """Contiguous KV cache (cache.py): updates bit-exact, overflow raises,
    decode attention over the first ``length`` positions."""
    d = load("kvcache")
    B, Hkv, _, D = d["kvc_k1"].shape
    c = O.init_kv_layer_cache(B, Hkv, D, d["kvc_keys"].shape[2])
    assert c.length == int(d["kvc_init_len"]) == 0
    c = O.update_kv_layer_cache(c, d["kvc_k1"], d["kvc_v1"], 0)
    c = O.update_kv_layer_cache(c, d["kvc_k2"], d["kvc_v2"], c.length)
    assert c.length == int(d["kvc_len"])
    np.testing.assert_array_equal(c.keys, d["kvc_keys"])
    np.testing.assert_array_equal(c.values, d["kvc_values"])
    assert int(d["kvc_overflow_raises"]) == 1
    with pytest.raises(ValueError, match="overflow"):
        O.update_kv_layer_cache(c, np.zeros((B, Hkv, 27, D), np.float32), np.zeros((B, Hkv, 27, D), np.float32),
                                c.length)
    for sq in (1, 3):
        np.testing.assert_allclose(O.kv_cache_attention(d[f"kvc_q{sq}"], c), d[f"kvc_out{sq}"], atol=1e-6)


def test_kv_layer_cache_update_host_logic_golden():
    """The library's update (a device copy into the buffers; here on host
    tensors) reproduces the reference's cache contents bit for bit."""
    import torch

    import attnax_b200 as ax

    d = load("kvcache")
    B, Hkv, _, D = d["kvc_k1"].shape
    c = ax.init_kv_layer_cache(B, Hkv, D, d["kvc_keys"].shape[2], torch.float32, device="cpu")
    c = ax.update_kv_layer_cache(c, torch.from_numpy(d["kvc_k1"]), torch.from_numpy(d["kvc_v1"]), 0)
    c = ax.update_kv_layer_cache(c, torch.from_numpy(d["kvc_k2"]), torch.from_numpy(d["kvc_v2"]), c.length)
    assert c.length == int(d["kvc_len"])
    np.testing.assert_array_equal(c.keys.numpy(), d["kvc_keys"])
    np.testing.assert_array_equal(c.values.numpy(), d["kvc_values"])
    with pytest.raises(ValueError, match="overflow"):
        ax.update_kv_layer_cache(c, torch.zeros(B, Hkv, 27, D), torch.zeros(B, Hkv, 27, D), c.length)
    assert len(ax.init_decoder_kv_caches(num_layers=3, batch_size=1, num_kv_heads=2, head_dim=8, max_len=4,
                                         dtype=torch.float32, device="cpu")) == 3


def test_rope_golden():
    """RoPE (embeddings.py): tables in the output dtype, gather by position,
    split-half rotation -- the oracle bit for bit, and the library's torch table
    construction (here on host tensors) within one ulp of the table dtype."""
    import torch

    import attnax_b200 as ax

    d = load("rope")
    pos = d["rope_pos"]
    for name, dt, tdt, tol in (("f32", np.float32, torch.float32, 1e-6), ("f16", np.float16, torch.float16, 1e-3)):
        c, s = O.rope_cos_sin_table(3000, 16, 10000.0, dt)
        np.testing.assert_array_equal(c, d[f"rope_cos_{name}"])
        np.testing.assert_array_equal(s, d[f"rope_sin_{name}"])
        cp, sp = O.rope_cos_sin_from_positions(pos, 16, 10000.0, 3000, dt)
        np.testing.assert_array_equal(O.apply_rope(d[f"rope_x_{name}"], cp[:, None], sp[:, None]),
                                      d[f"rope_y_{name}"])
        tc, ts = ax.rope_cos_sin_table(3000, 16, 10000.0, tdt, device="cpu")
        np.testing.assert_allclose(tc.float().numpy(), d[f"rope_cos_{name}"].astype(np.float32), atol=tol)
        np.testing.assert_allclose(ts.float().numpy(), d[f"rope_sin_{name}"].astype(np.float32), atol=tol)


def test_ring_unbound_axis_falls_back_golden():
    d = load("ring")
    out = O.standard_attention(d["ring_q"], d["ring_k"], d["ring_v"])
    np.testing.assert_allclose(out, d["ring_unbound"], atol=2e-6, rtol=1e-5)


# ------------------------------------- reference known-answer tests ------

def _qkv(batch=2, heads=4, seq=8, dim=16, seed=0):
    rng = np.random.default_rng(seed)
    return tuple(rng.standard_normal((batch, heads, seq, dim), dtype=np.float32) for _ in range(3))


def test_kat_memory_efficient_equals_standard():
    # tests/test_kernels.py:44-57
    q, k, v = _qkv()
    np.testing.assert_allclose(O.memory_efficient_attention(q, k, v, block_size=64),
                               O.standard_attention(q, k, v), atol=1e-5)
    q, k, v = _qkv(1, 2, 128, 8, 42)
    np.testing.assert_allclose(O.memory_efficient_attention(q, k, v, block_size=32),
                               O.standard_attention(q, k, v), atol=1e-4)


def test_kat_mods_equal_masks():
    # tests/test_kernels.py:60-87, :173-196, :220-231
    q, k, v = _qkv(seq=10)
    np.testing.assert_allclose(O.standard_attention(q, k, v, mask=O.make_causal_mask(10)),
                               O.standard_attention(q, k, v, score_mod=O.causal_mod()), atol=1e-5)
    q, k, v = _qkv(seq=12)
    np.testing.assert_allclose(
        O.standard_attention(q, k, v, mask=O.make_sliding_window_mask(12, window_size=4)),
        O.standard_attention(q, k, v, score_mod=O.sliding_window_mod(4)), atol=1e-5)
    ids = np.array([[0, 0, 0, 1, 1], [0, 0, 1, 1, 2]])
    q, k, v = _qkv(2, 4, 5, 16, 7)
    np.testing.assert_allclose(
        O.standard_attention(q, k, v, mask=O.make_document_mask(ids)),
        O.standard_attention(q, k, v, score_mod=O.document_mask_mod(ids)), atol=1e-5)
    q, k, v = _qkv(seq=8)
    np.testing.assert_allclose(
        O.standard_attention(q, k, v, score_mod=O.compose_score_mods(O.causal_mod(),
                                                                     O.sliding_window_mod(4))),
        O.standard_attention(q, k, v, mask=O.combine_masks(
            O.make_causal_mask(8), O.make_sliding_window_mask(8, window_size=4))), atol=1e-5)
    np.testing.assert_allclose(
        O.standard_attention(q, k, v, mask=O.make_causal_mask(8)),
        O.standard_attention(q, k, v, score_mod=O.mask_mod_to_score_mod(lambda b, h, q_, kv: kv <= q_)),
        atol=1e-5)
    zero = O.additive_bias_mod(np.zeros((1, 1, 1, 1), np.float32))
    np.testing.assert_allclose(O.standard_attention(q, k, v),
                               O.standard_attention(q, k, v, score_mod=zero), atol=1e-6)


def test_kat_patterns():
    # tests/test_kernels.py:90-171
    m = O.make_sliding_window_mask(6, window_size=3)
    assert m.shape == (1, 1, 6, 6)
    assert m[0, 0, 5, 3] and m[0, 0, 5, 4] and m[0, 0, 5, 5] and not m[0, 0, 5, 2]
    s = O.make_sliding_window_mask(5, window_size=2, causal=False)
    assert s[0, 0, 2, 1] and s[0, 0, 2, 3] and not s[0, 0, 2, 4]
    for w in (0, -1):
        with pytest.raises(ValueError):
            O.make_sliding_window_mask(4, window_size=w)
        with pytest.raises(ValueError):
            O.sliding_window_mod(w)
    sl = O.alibi_slopes(8)
    assert sl.shape == (8,) and np.all(sl > 0) and np.all(sl[1:] < sl[:-1])
    assert O.alibi_slopes(6).shape == (6,) and np.all(O.alibi_slopes(6) > 0)
    b, h, q, kv = O.position_indices(1, 4, 8, 8)
    biased = O.alibi_mod(4)(np.zeros((1, 4, 8, 8), np.float32), b, h, q, kv)
    assert np.allclose(np.diagonal(biased[0, 0]), 0.0) and np.all(biased[0, 0] <= 0)
    b, h, q, kv = O.position_indices(1, 1, 6, 6)
    out = O.prefix_lm_mod(np.array([3]))(np.zeros((1, 1, 6, 6), np.float32), b, h, q, kv)
    assert out[0, 0, 1, 2] == 0 and out[0, 0, 3, 4] < 0 and out[0, 0, 4, 3] == 0
    dm = O.make_document_mask(np.array([[0, 0, 0, 1, 1]]))
    assert dm.shape == (1, 1, 5, 5) and not dm[0, 0, 0, 3] and dm[0, 0, 0, 1]
    assert O.compose_score_mods(None, None) is None
    cm = O.causal_mod()
    assert O.compose_score_mods(None, cm) is cm


def test_kat_paged_cache():
    # tests/test_advanced_kernels.py:121-196
    c = O.init_paged_kv_cache(num_blocks=8, block_size=4, num_kv_heads=2, head_dim=16,
                              batch_size=2, max_blocks_per_seq=4)
    assert c.key_pool.shape == (8, 4, 2, 16) and c.block_table.shape == (2, 4)
    assert c.seq_lengths[0] == 0 and c.block_table[0, 0] == -1
    c = O.init_paged_kv_cache(num_blocks=8, block_size=4, num_kv_heads=2, head_dim=8,
                              batch_size=1, max_blocks_per_seq=4)
    c, used = O.allocate_blocks(c, sequence_idx=0, num_new_tokens=10,
                                free_block_ids=np.arange(8, dtype=np.int32))
    assert used == 3 and list(c.block_table[0, :3]) == [0, 1, 2]
    rng = np.random.default_rng(0)
    kn = rng.standard_normal((10, 2, 8), dtype=np.float32)
    vn = rng.standard_normal((10, 2, 8), dtype=np.float32)
    c = O.append_kv(c, 0, kn, vn)
    kb, vb, n = O.gather_kv(c, 0)
    assert n == 10
    np.testing.assert_array_equal(kb, kn)
    np.testing.assert_array_equal(vb, vn)
    c2 = O.init_paged_kv_cache(num_blocks=2, block_size=4, num_kv_heads=2, head_dim=8,
                               batch_size=1, max_blocks_per_seq=2)
    with pytest.raises(ValueError, match="unallocated"):
        O.append_kv(c2, 0, np.zeros((1, 2, 8), np.float32), np.zeros((1, 2, 8), np.float32))
    with pytest.raises(ValueError):
        O.allocate_blocks(c2, sequence_idx=0, num_new_tokens=9, free_block_ids=np.arange(1))


def test_oracle_backward_matches_torch_autograd():
    """The closed-form backward equals autograd of the same forward (fp64)."""
    import torch
    rng = np.random.default_rng(5)
    B, H, Hkv, S, D = 1, 4, 2, 24, 8
    q = rng.standard_normal((B, H, S, D))
    k = rng.standard_normal((B, Hkv, S, D))
    v = rng.standard_normal((B, Hkv, S, D))
    do = rng.standard_normal((B, H, S, D))
    mask = np.ones((B, 1, S, S), bool)
    mask[0, 0, 5, :] = False  # fully masked row: uniform P reaches dV only
    mod = O.compose_score_mods(O.sliding_window_mod(6), O.alibi_mod(H))
    dq, dk, dv = O.gqa_attention_bwd(q, k, v, do, mask=mask, score_mod=mod)

    tq, tk, tv = (torch.tensor(x, requires_grad=True) for x in (q, k, v))
    rep = H // Hkv
    kk, vv = tk.repeat_interleave(rep, 1), tv.repeat_interleave(rep, 1)
    s = torch.einsum("bhqd,bhkd->bhqk", tq, kk) / np.sqrt(D)
    qi = torch.arange(S)[:, None]
    ki = torch.arange(S)[None, :]
    keep = (ki <= qi) & (qi - ki < 6)
    neg = torch.finfo(torch.float64).min
    s = torch.where(keep, s, torch.tensor(neg, dtype=torch.float64))
    slopes = torch.tensor(O.alibi_slopes(H), dtype=torch.float64)[None, :, None, None]
    s = s - slopes * (qi - ki).abs().double()
    s = torch.where(torch.tensor(mask), s, torch.tensor(neg, dtype=torch.float64))
    out = torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, -1), vv)
    out.backward(torch.tensor(do))
    np.testing.assert_allclose(dq, tq.grad.numpy(), atol=1e-10)
    np.testing.assert_allclose(dk, tk.grad.numpy(), atol=1e-10)
    np.testing.assert_allclose(dv, tv.grad.numpy(), atol=1e-10)
