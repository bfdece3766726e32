"""Generates the golden vectors in this folder from the reference's own source.

Run from the repository root, pointing ``--ref`` at a checkout of the attnax
reference (the directory that contains the ``attnax`` package):

    python tests/golden/make_golden.py --ref <attnax checkout>

The reference's hot-path modules (``attnax/kernels/*.py``,
``attnax/paged_cache.py``, ``attnax/masking.py``, ``attnax/cache.py``,
``attnax/embeddings.py``) are imported unmodified on
top of ``jax_standin`` (numpy in place of ``jax.numpy``) and evaluated on
seeded ``numpy.random.default_rng`` inputs.  Inputs and outputs are stored
in ``golden_*.npz``; the tests read only those files.
"""

from __future__ import annotations

import argparse
import pathlib
import sys
import types

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import jax_standin  # noqa: E402


def load_reference(ref_root: pathlib.Path):
    jax_standin.install()
    pkg = types.ModuleType("attnax")
    pkg.__path__ = [str(ref_root / "attnax")]
    sys.modules["attnax"] = pkg
    import attnax.kernels as K  # noqa: E402
    import attnax.masking as M  # noqa: E402
    import attnax.paged_cache as PC  # noqa: E402
    return K, M, PC


def make_rope(ref_root: pathlib.Path):
    """RoPE (``attnax/embeddings.py``): cos/sin tables built in the output dtype
    (float32 and float16), gathered by position ids, applied split-half."""
    import attnax.embeddings as E  # noqa: E402
    out = {}
    rng = np.random.default_rng(7)
    B, H, S, D, table, base = 2, 3, 24, 16, 3000, 10000.0
    pos = rng.integers(0, table, size=(B, S)).astype(np.int32)
    out["rope_pos"] = pos
    for name, dt in (("f32", np.float32), ("f16", np.float16)):
        cos_t, sin_t = E.rope_cos_sin_table(table, D, base, dt)
        cos, sin = E.rope_cos_sin_from_positions(A(pos), D, base, table, dt)
        x = rnd(rng, (B, H, S, D)).astype(dt)
        y = E.apply_rope(A(x), A(np.asarray(cos))[:, None], A(np.asarray(sin))[:, None])
        out.update({f"rope_cos_{name}": np.asarray(cos_t), f"rope_sin_{name}": np.asarray(sin_t),
                    f"rope_x_{name}": x, f"rope_y_{name}": np.asarray(y)})
    np.savez_compressed(HERE / "golden_rope.npz", **out)


def make_kvcache(ref_root: pathlib.Path, K):
    """Contiguous per-layer KV cache (``attnax/cache.py``): a prefill chunk and a
    decode token written with ``update_kv_layer_cache``, the overflow error,
    and attention of the decode queries over ``keys[:, :, :length]`` (what
    ``MultiHeadAttention`` computes from the concatenated history,
    ``attnax/attention.py:386-400``)."""
    import attnax.cache as KC  # noqa: E402
    out = {}
    rng = np.random.default_rng(6)
    B, Hq, Hkv, L, D = 2, 4, 2, 40, 16
    c = KC.init_kv_layer_cache(B, Hkv, D, L, np.float32)
    out["kvc_init_len"] = np.asarray(c.length)
    k1, v1 = rnd(rng, (B, Hkv, 13, D)), rnd(rng, (B, Hkv, 13, D))
    c = KC.update_kv_layer_cache(c, A(k1), A(v1), 0)
    k2, v2 = rnd(rng, (B, Hkv, 1, D)), rnd(rng, (B, Hkv, 1, D))
    c = KC.update_kv_layer_cache(c, A(k2), A(v2), int(c.length))
    out.update(kvc_k1=k1, kvc_v1=v1, kvc_k2=k2, kvc_v2=v2, kvc_keys=np.asarray(c.keys),
               kvc_values=np.asarray(c.values), kvc_len=np.asarray(c.length))
    try:
        KC.update_kv_layer_cache(c, A(rnd(rng, (B, Hkv, 27, D))), A(rnd(rng, (B, Hkv, 27, D))), int(c.length))
        out["kvc_overflow_raises"] = np.array(0)
    except ValueError:
        out["kvc_overflow_raises"] = np.array(1)
    n = int(c.length)
    for sq in (1, 3):
        q = rnd(rng, (B, Hq, sq, D))
        out[f"kvc_q{sq}"] = q
        # the MHA repeats kv heads before attention (_repeat_kv_heads, attnax/attention.py:32-39)
        kr = A(np.repeat(np.asarray(c.keys[:, :, :n, :]), Hq // Hkv, axis=1))
        vr = A(np.repeat(np.asarray(c.values[:, :, :n, :]), Hq // Hkv, axis=1))
        out[f"kvc_out{sq}"] = np.asarray(K.standard_attention(A(q), kr, vr))
    np.savez_compressed(HERE / "golden_kvcache.npz", **out)


def rnd(rng, shape, bf16=False):
    x = rng.standard_normal(shape, dtype=np.float32)
    if bf16:
        u = x.view(np.uint32).astype(np.uint64)
        u = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16) << 16
        x = u.astype(np.uint32).view(np.float32)
    return x


def A(x):
    return jax_standin.as_array(x)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="attnax checkout (the directory holding the attnax package)")
    ap.add_argument("--only", choices=["kvcache", "rope"], default=None,
                    help="write only this fixture (leaves the other files untouched)")
    args = ap.parse_args()
    K, M, PC = load_reference(pathlib.Path(args.ref))
    if args.only == "kvcache":
        make_kvcache(pathlib.Path(args.ref), K)
        print("golden_kvcache.npz written to", HERE)
        return
    if args.only == "rope":
        make_rope(pathlib.Path(args.ref))
        print("golden_rope.npz written to", HERE)
        return
    out = {}

    # --- score-mod chains through standard_attention ---------------------
    rng = np.random.default_rng(0)
    B, H, S, D = 2, 4, 12, 16
    q, k, v = (rnd(rng, (B, H, S, D)) for _ in range(3))
    bias = rnd(rng, (B, H, S, S))
    ids = np.array([[0, 0, 0, 0, 1, 1, 1, 2, 2, 2, 2, 2],
                    [0, 0, 1, 1, 1, 1, 1, 1, 1, 2, 3, 3]], dtype=np.int32)
    pref = np.array([3, 5], dtype=np.int32)
    fully = np.ones((B, 1, S, S), dtype=bool)
    fully[0, 0, 3, :] = False          # one fully masked query row
    fully[1, 0, :, 5:9] = False        # a masked key stripe
    mods = {
        "none": None,
        "causal": K.causal_mod(),
        "window4": K.sliding_window_mod(4),
        "window3_sym": K.sliding_window_mod(3, causal=False),
        "alibi": K.alibi_mod(H),
        "prefix": K.prefix_lm_mod(A(pref)),
        "document": K.document_mask_mod(A(ids)),
        "bias": K.additive_bias_mod(A(bias)),
        "window4_alibi": K.compose_score_mods(K.sliding_window_mod(4), K.alibi_mod(H)),
        "document_causal": K.compose_score_mods(K.document_mask_mod(A(ids)), K.causal_mod()),
        "maskmod_causal": K.mask_mod_to_score_mod(lambda b, h, qi, kvi: kvi <= qi),
    }
    out["mods_q"], out["mods_k"], out["mods_v"] = q, k, v
    out["mods_bias"], out["mods_ids"], out["mods_pref"] = bias, ids, pref
    for name, mod in mods.items():
        out[f"mods_out_{name}"] = np.asarray(K.standard_attention(A(q), A(k), A(v), score_mod=mod))
    out["mask_fully"] = fully
    out["mods_out_mask_fully"] = np.asarray(K.standard_attention(A(q), A(k), A(v), mask=A(fully)))
    pad_ids = np.array([[5, 3, 0, 0, 7, 1, 2, 0, 4, 4, 0, 9], [0] * 12], dtype=np.int32)
    out["mask_pad_ids"] = pad_ids
    out["mods_out_mask_pad_alibi"] = np.asarray(K.standard_attention(
        A(q), A(k), A(v), mask=M.make_padding_mask(A(pad_ids)), score_mod=K.alibi_mod(H)))

    # --- raw score-mod values and mask helpers --------------------------
    z = np.zeros((1, H, 8, 8), dtype=np.float32)
    bi, hi, qi, kvi = (np.zeros((1, 1, 1, 1), np.int32), np.zeros((1, H, 1, 1), np.int32),
                       np.arange(8, dtype=np.int32)[None, None, :, None],
                       np.arange(8, dtype=np.int32)[None, None, None, :])
    out["raw_alibi"] = np.asarray(K.alibi_mod(H)(A(z), A(bi), A(hi), A(qi), A(kvi)))
    z6 = np.zeros((1, 1, 6, 6), dtype=np.float32)
    out["raw_prefix"] = np.asarray(K.prefix_lm_mod(A(np.array([3])))(
        A(z6), A(bi), A(bi), A(np.arange(6, dtype=np.int32)[None, None, :, None]),
        A(np.arange(6, dtype=np.int32)[None, None, None, :])))
    for n in (1, 4, 6, 8, 12, 16, 32):
        out[f"alibi_slopes_{n}"] = np.asarray(K.alibi_slopes(n))
    out["mask_window_6_3"] = np.asarray(M.make_sliding_window_mask(6, window_size=3, causal=True))
    out["mask_window_5_2_sym"] = np.asarray(M.make_sliding_window_mask(5, window_size=2, causal=False))
    out["mask_window_7_9_3"] = np.asarray(M.make_sliding_window_mask(7, 9, window_size=3))
    out["mask_causal_5"] = np.asarray(M.make_causal_mask(5))
    out["mask_document"] = np.asarray(M.make_document_mask(A(ids)))
    out["mask_boolean_causal"] = np.asarray(K.mask_mod_to_boolean_mask(
        lambda b, h, qi, kvi: kvi <= qi, batch=1, num_heads=2, seq_q=4, seq_kv=4))
    np.savez_compressed(HERE / "golden_mods.npz", **out)

    # --- blockwise online softmax -----------------------------------------
    out = {}
    rng = np.random.default_rng(1)
    q, k, v = (rnd(rng, (1, 2, 128, 8)) for _ in range(3))
    out["me_q"], out["me_k"], out["me_v"] = q, k, v
    out["me_std"] = np.asarray(K.standard_attention(A(q), A(k), A(v)))
    out["me_b32"] = np.asarray(K.memory_efficient_attention(A(q), A(k), A(v), block_size=32))
    out["me_b32_causal"] = np.asarray(K.memory_efficient_attention(
        A(q), A(k), A(v), score_mod=K.causal_mod(), block_size=32))
    out["flash_cpu_b32_causal"] = np.asarray(K.flash_attention(
        A(q), A(k), A(v), score_mod=K.causal_mod(), block_size=32))
    out["pallas_cpu"] = np.asarray(K.pallas_flash_attention(A(q), A(k), A(v)))
    qr, kr, vr = rnd(rng, (1, 2, 100, 8)), rnd(rng, (1, 2, 70, 8)), rnd(rng, (1, 2, 70, 8))
    out["me_rag_q"], out["me_rag_k"], out["me_rag_v"] = qr, kr, vr
    out["me_rag_b32_alibi"] = np.asarray(K.memory_efficient_attention(
        A(qr), A(kr), A(vr), score_mod=K.alibi_mod(2), block_size=32))
    out["me_rag_b32_window"] = np.asarray(K.memory_efficient_attention(
        A(qr), A(kr), A(vr), score_mod=K.sliding_window_mod(20), block_size=32))
    np.savez_compressed(HERE / "golden_blockwise.npz", **out)

    # --- bf16-valued inputs, the long-context mod chain at small size ------
    out = {}
    rng = np.random.default_rng(2)
    B, Hq, Hkv, S, D = 1, 8, 2, 300, 64
    q, k, v = rnd(rng, (B, Hq, S, D), True), rnd(rng, (B, Hkv, S, D), True), rnd(rng, (B, Hkv, S, D), True)
    kr_, vr_ = np.repeat(k, Hq // Hkv, axis=1), np.repeat(v, Hq // Hkv, axis=1)
    out["gqa_q"], out["gqa_k"], out["gqa_v"] = q, k, v
    out["gqa_window64_alibi"] = np.asarray(K.standard_attention(
        A(q), A(kr_), A(vr_),
        score_mod=K.compose_score_mods(K.sliding_window_mod(64), K.alibi_mod(Hq))))
    docs = np.repeat(np.arange(5, dtype=np.int32), [70, 64, 100, 2, 64])[None]
    out["gqa_docs"] = docs
    out["gqa_document_causal"] = np.asarray(K.standard_attention(
        A(q), A(kr_), A(vr_),
        score_mod=K.compose_score_mods(K.document_mask_mod(A(docs)), K.causal_mod())))
    np.savez_compressed(HERE / "golden_gqa_bf16.npz", **out)

    # --- paged cache: allocate / append / gather / attend -----------------
    out = {}
    rng = np.random.default_rng(3)
    nb, bs, hkv, d, nseq, maxb = 12, 4, 2, 8, 3, 4
    cache = PC.init_paged_kv_cache(num_blocks=nb, block_size=bs, num_kv_heads=hkv, head_dim=d,
                                   batch_size=nseq, max_blocks_per_seq=maxb, dtype=np.float32)
    perm = rng.permutation(nb).astype(np.int32)
    lens = [10, 0, 13]
    used = 0
    new_k, new_v = [], []
    for s, n in enumerate(lens):
        cache, got = PC.allocate_blocks(cache, sequence_idx=s, num_new_tokens=n,
                                        free_block_ids=A(perm[used:]))
        used += got
        kk, vv = rnd(rng, (n, hkv, d)), rnd(rng, (n, hkv, d))
        new_k.append(kk)
        new_v.append(vv)
        if n:
            cache = PC.append_kv(cache, s, A(kk), A(vv))
    out["paged_perm"] = perm
    out["paged_lens"] = np.array(lens, np.int32)
    for s in range(nseq):
        out[f"paged_newk_{s}"], out[f"paged_newv_{s}"] = new_k[s], new_v[s]
    out["paged_key_pool"] = np.asarray(cache.key_pool)
    out["paged_value_pool"] = np.asarray(cache.value_pool)
    out["paged_block_table"] = np.asarray(cache.block_table)
    out["paged_seq_lengths"] = np.asarray(cache.seq_lengths)
    for s in range(nseq):
        kb, vb, n = PC.gather_kv(cache, s)
        out[f"paged_gather_k_{s}"], out[f"paged_gather_v_{s}"] = np.asarray(kb), np.asarray(vb)
    qd = rnd(rng, (nseq, 4, 1, d))
    qp = rnd(rng, (nseq, 4, 3, d))
    out["paged_q_decode"], out["paged_q_prefill"] = qd, qp
    for s in range(nseq):
        out[f"paged_out_decode_{s}"] = np.asarray(K.paged_attention(A(qd[s]), cache, s))
        out[f"paged_out_prefill_{s}"] = np.asarray(K.paged_attention(A(qp[s]), cache, s))
    np.savez_compressed(HERE / "golden_paged.npz", **out)

    # --- ring with a bound axis (threads emulate the devices) -------------
    out = {}
    rng = np.random.default_rng(4)
    B, H, S, D = 1, 4, 64, 16
    q, k, v = (rnd(rng, (B, H, S, D)) for _ in range(3))
    out["ring_q"], out["ring_k"], out["ring_v"] = q, k, v
    for P in (2, 4):
        sl = S // P
        shards = [(A(q[:, :, r * sl:(r + 1) * sl]), A(k[:, :, r * sl:(r + 1) * sl]),
                   A(v[:, :, r * sl:(r + 1) * sl])) for r in range(P)]
        for name, mod in (("none", None), ("causal", K.causal_mod()), ("alibi", K.alibi_mod(H))):
            res = jax_standin.run_on_ring(
                lambda a, b, c: K.ring_attention(a, b, c, axis_name="sp", score_mod=mod),
                shards, "sp")
            out[f"ring_P{P}_{name}"] = np.concatenate([np.asarray(x) for x in res], axis=2)
    out["ring_ref_causal"] = np.asarray(K.ring_attention_reference(A(q), A(k), A(v),
                                                                   score_mod=K.causal_mod()))
    out["ring_unbound"] = np.asarray(K.ring_attention(A(q), A(k), A(v), axis_name="not_bound"))
    np.savez_compressed(HERE / "golden_ring.npz", **out)
    make_kvcache(pathlib.Path(args.ref), K)
    make_rope(pathlib.Path(args.ref))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
