"""Flash forward/backward parity on the GPU, through the C ABI, against the oracle."""

import pathlib

import numpy as np
import pytest
import torch

import attnax_b200 as ax
import oracle as O
from tests._util import assert_bf16_close, assert_bf16_grad_close, assert_fp32_close, randn

pytestmark = pytest.mark.gpu
DEV = "cuda"
G = pathlib.Path(__file__).resolve().parent / "golden"


def T(x, dtype=torch.bfloat16, grad=False):
    return torch.tensor(x, dtype=dtype, device=DEV, requires_grad=grad)


def npy(t):
    return t.detach().float().cpu().numpy()


def pair(name, H, S, B):
    """(kernel mod, oracle mod) for a named mod chain."""
    rng = np.random.default_rng(11)
    if name == "none":
        return None, None
    if name == "causal":
        return ax.causal_mod(), O.causal_mod()
    if name == "window":
        return ax.sliding_window_mod(70), O.sliding_window_mod(70)
    if name == "window_sym":
        return ax.sliding_window_mod(50, causal=False), O.sliding_window_mod(50, causal=False)
    if name == "alibi":
        return ax.alibi_mod(H), O.alibi_mod(H)
    if name == "window_alibi":
        return (ax.compose_score_mods(ax.sliding_window_mod(90), ax.alibi_mod(H)),
                O.compose_score_mods(O.sliding_window_mod(90), O.alibi_mod(H)))
    if name == "causal_alibi":
        return (ax.compose_score_mods(ax.causal_mod(), ax.alibi_mod(H)),
                O.compose_score_mods(O.causal_mod(), O.alibi_mod(H)))
    if name == "window_alibi_wide":
        return (ax.compose_score_mods(ax.sliding_window_mod(400), ax.alibi_mod(H)),
                O.compose_score_mods(O.sliding_window_mod(400), O.alibi_mod(H)))
    if name == "prefix":
        pref = np.array([37, 200][:B] + [5] * max(0, B - 2), np.int32)
        return ax.prefix_lm_mod(pref), O.prefix_lm_mod(pref)
    if name == "document_causal":
        lens = [130, 64, 2, 200, 1000]
        ids = np.repeat(np.arange(len(lens)), lens)[:S]
        ids = np.stack([ids, np.sort(rng.integers(0, 4, S))])[:B].astype(np.int32)
        return (ax.compose_score_mods(ax.document_mask_mod(ids), ax.causal_mod()),
                O.compose_score_mods(O.document_mask_mod(ids), O.causal_mod()))
    if name == "bias":
        bias = rng.standard_normal((1, H, S, S)).astype(np.float32)
        return ax.additive_bias_mod(torch.tensor(bias, device=DEV)), O.additive_bias_mod(bias)
    if name == "maskmod":
        f = lambda b, h, q, kv: (q + kv) % 3 != 0  # noqa: E731
        return ax.mask_mod_to_score_mod(f), O.mask_mod_to_score_mod(f)
    raise KeyError(name)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [128, 256, 300])
def test_tensor_core_forward_plain(D, S):
    rng = np.random.default_rng(D + S)
    q, k, v = (randn(rng, (1, 2, S, D), True) for _ in range(3))
    out = ax.flash_attention(T(q), T(k), T(v))
    assert_bf16_close(npy(out), O.standard_attention(q, k, v), f"D={D} S={S}")


@pytest.mark.parametrize("mod", ["none", "causal", "window", "window_sym", "alibi", "window_alibi",
                                 "prefix", "document_causal", "bias", "maskmod"])
def test_tensor_core_forward_mods_gqa(mod):
    rng = np.random.default_rng(1)
    B, Hq, Hkv, S, D = 2, 4, 2, 300, 128
    q = randn(rng, (B, Hq, S, D), True)
    k = randn(rng, (B, Hkv, S, D), True)
    v = randn(rng, (B, Hkv, S, D), True)
    m_ax, m_o = pair(mod, Hq, S, B)
    out = ax.flash_attention(T(q), T(k), T(v), score_mod=m_ax)
    assert_bf16_close(npy(out), O.gqa_attention(q, k, v, score_mod=m_o), mod)


def test_fp32_causal_config():
    """fp32 B2 H8 S1024 D64 causal: within 1e-4 of standard_attention."""
    rng = np.random.default_rng(0)
    q, k, v = (randn(rng, (2, 8, 1024, 64)) for _ in range(3))
    out = ax.flash_attention(T(q, torch.float32), T(k, torch.float32), T(v, torch.float32),
                             score_mod=ax.causal_mod())
    assert_fp32_close(npy(out), O.standard_attention(q, k, v, score_mod=O.causal_mod()), "c1")


def test_golden_mods_fp32():
    d = dict(np.load(G / "golden_mods.npz"))
    q, k, v = d["mods_q"], d["mods_k"], d["mods_v"]
    H = q.shape[1]
    mods = {
        "none": None, "causal": ax.causal_mod(), "window4": ax.sliding_window_mod(4),
        "window3_sym": ax.sliding_window_mod(3, causal=False), "alibi": ax.alibi_mod(H),
        "prefix": ax.prefix_lm_mod(d["mods_pref"]), "document": ax.document_mask_mod(d["mods_ids"]),
        "bias": ax.additive_bias_mod(torch.tensor(d["mods_bias"], device=DEV)),
        "window4_alibi": ax.compose_score_mods(ax.sliding_window_mod(4), ax.alibi_mod(H)),
        "document_causal": ax.compose_score_mods(ax.document_mask_mod(d["mods_ids"]), ax.causal_mod()),
        "maskmod_causal": ax.mask_mod_to_score_mod(lambda b, h, qi, kvi: kvi <= qi),
    }
    tq, tk, tv = (T(x, torch.float32) for x in (q, k, v))
    for name, mod in mods.items():
        out = ax.flash_attention(tq, tk, tv, score_mod=mod)
        assert_fp32_close(npy(out), d[f"mods_out_{name}"], name, atol=2e-5)
    out = ax.flash_attention(tq, tk, tv, mask=torch.tensor(d["mask_fully"], device=DEV))
    assert_fp32_close(npy(out), d["mods_out_mask_fully"], "fully masked row", atol=2e-5)
    out = ax.flash_attention(tq, tk, tv, mask=ax.make_padding_mask(torch.tensor(d["mask_pad_ids"], device=DEV)),
                             score_mod=ax.alibi_mod(H))
    assert_fp32_close(npy(out), d["mods_out_mask_pad_alibi"], "padding + alibi", atol=2e-5)


def test_golden_gqa_bf16():
    d = dict(np.load(G / "golden_gqa_bf16.npz"))
    q, k, v = d["gqa_q"], d["gqa_k"], d["gqa_v"]
    H = q.shape[1]
    out = ax.flash_attention(T(q), T(k), T(v), score_mod=ax.compose_score_mods(
        ax.sliding_window_mod(64), ax.alibi_mod(H)))
    assert_bf16_close(npy(out), d["gqa_window64_alibi"], "window64+alibi")
    out = ax.flash_attention(T(q), T(k), T(v), score_mod=ax.compose_score_mods(
        ax.document_mask_mod(d["gqa_docs"]), ax.causal_mod()))
    assert_bf16_close(npy(out), d["gqa_document_causal"], "document+causal")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fully_masked_rows_average_v(dtype):
    rng = np.random.default_rng(3)
    B, H, S, D = 1, 2, 260, 128 if dtype == torch.bfloat16 else 64
    q, k, v = (randn(rng, (B, H, S, D), True) for _ in range(3))
    mask = np.ones((B, 1, S, S), bool)
    mask[0, 0, 7] = False
    mask[0, 0, 200:210, :] = False
    got = npy(ax.flash_attention(T(q, dtype), T(k, dtype), T(v, dtype), mask=torch.tensor(mask, device=DEV),
                                 score_mod=ax.causal_mod()))
    want = O.standard_attention(q, k, v, mask=mask, score_mod=O.causal_mod())
    if dtype == torch.bfloat16:
        assert_bf16_close(got, want, "fully masked")
    else:
        assert_fp32_close(got, want, "fully masked")


def test_lse_matches_oracle():
    from attnax_b200._spec import build_spec
    from attnax_b200.flash import fwd_raw

    rng = np.random.default_rng(4)
    q, k, v = (randn(rng, (1, 2, 384, 128), True) for _ in range(3))
    spec = build_spec(ax.causal_mod(), None, batch=1, heads_q=2, seq_q=384, seq_kv=384, device=DEV)
    _, lse = fwd_raw(T(q), T(k), T(v), spec)
    _, want = O.standard_attention_lse(q, k, v, score_mod=O.causal_mod())
    assert np.max(np.abs(npy(lse) - want)) < 1e-3


@pytest.mark.parametrize("mod", ["causal", "window", "causal_alibi", "prefix", "document_causal"])
@pytest.mark.parametrize("D", [64, 128])
def test_forward_at_offsets_boundary_tiles(mod, D):
    """Band, prefix and document boundary tiles at global offsets, the calls a
    ring hop makes: queries start before the keys, so the first rows keep no
    key under the causal chains.  Rows that keep a key match the oracle (out
    and LSE); rows that keep none come back with LSE -inf (an empty partial)."""
    from attnax_b200._spec import build_spec
    from attnax_b200.flash import fwd_raw

    rng = np.random.default_rng(12)
    B, Hq, Hkv, Sq, Skv = 2, 4, 2, 300, 260
    q0, k0 = 170, 333
    total = max(q0 + Sq, k0 + Skv)
    if mod == "prefix":
        pref = np.array([400, 100], np.int32)  # batch 0: the prefix reaches into the keys; batch 1: causal only
        m_ax, m_o = ax.prefix_lm_mod(pref), O.prefix_lm_mod(pref)
    else:
        m_ax, m_o = pair(mod, Hq, total, B)
    q = randn(rng, (B, Hq, Sq, D), True)
    k, v = (randn(rng, (B, Hkv, Skv, D), True) for _ in range(2))
    spec = build_spec(m_ax, None, batch=B, heads_q=Hq, seq_q=Sq, seq_kv=Skv, device=torch.device(DEV),
                      q_offset=q0, kv_offset=k0)
    out, lse = fwd_raw(T(q), T(k), T(v), spec)
    kr, vr = O.repeat_kv(k, Hq), O.repeat_kv(v, Hq)
    want_o, want_l = O.standard_attention_lse(q, kr, vr, score_mod=m_o, q_offset=q0, kv_offset=k0)
    s = O.attention_oracle._final_scores(q, kr, None, m_o, q0, k0)
    empty = np.all(s == np.finfo(s.dtype).min, axis=-1)
    got_o, got_l = npy(out), npy(lse)
    assert np.all(np.isneginf(got_l[empty])), "rows that keep no key must return lse -inf"
    keep = ~empty
    assert keep.sum() > 0
    assert_bf16_close(got_o[keep], want_o[keep], f"offsets {mod} D{D}")
    assert np.max(np.abs(got_l[keep] - want_l[keep])) < 1e-3


@pytest.mark.parametrize("mod", ["causal", "window", "causal_alibi", "prefix", "document_causal"])
@pytest.mark.parametrize("D", [64, 128])
def test_backward_at_offsets_boundary_tiles(mod, D):
    """Backward through band, prefix and document boundary tiles at global
    offsets (queries after the start of the keys, so every row keeps a key):
    the gradients of the attention whose mods see positions shifted by the
    offsets."""
    from attnax_b200._spec import build_spec
    from attnax_b200.flash import bwd_raw, fwd_raw

    rng = np.random.default_rng(13)
    B, Hq, Hkv, Sq, Skv = 2, 4, 2, 300, 260
    q0, k0 = 400, 333
    total = max(q0 + Sq, k0 + Skv)
    if mod == "prefix":
        pref = np.array([400, 100], np.int32)
        m_ax, m_o = ax.prefix_lm_mod(pref), O.prefix_lm_mod(pref)
    elif mod == "window":
        m_ax, m_o = ax.sliding_window_mod(150), O.sliding_window_mod(150)
    else:
        m_ax, m_o = pair(mod, Hq, total, B)

    def shifted(scores, b_idx, h_idx, q_idx, kv_idx):
        return m_o(scores, b_idx, h_idx, q_idx + q0, kv_idx + k0)

    q = randn(rng, (B, Hq, Sq, D), True)
    k, v = (randn(rng, (B, Hkv, Skv, D), True) for _ in range(2))
    do = randn(rng, (B, Hq, Sq, D), True)
    spec = build_spec(m_ax, None, batch=B, heads_q=Hq, seq_q=Sq, seq_kv=Skv, device=torch.device(DEV),
                      q_offset=q0, kv_offset=k0)
    tq, tk, tv = T(q), T(k), T(v)
    out, lse = fwd_raw(tq, tk, tv, spec)
    assert np.all(np.isfinite(npy(lse))), "every row keeps a key at these offsets"
    got = bwd_raw(tq, tk, tv, out, lse, T(do), spec)
    want = O.gqa_attention_bwd(q, k, v, do, score_mod=shifted)
    for name, g, w in zip(("dq", "dk", "dv"), got, want):
        assert_bf16_grad_close(npy(g), w, f"offsets {mod} D{D} {name}")


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.bfloat16, 64), (torch.float32, 64)])
@pytest.mark.parametrize("mod", ["causal", "window_alibi", "document_causal"])
def test_backward(dtype, D, mod):
    rng = np.random.default_rng(5)
    bf = dtype == torch.bfloat16
    B, Hq, Hkv, S = 2, 4, 2, 300
    q = randn(rng, (B, Hq, S, D), bf)
    k = randn(rng, (B, Hkv, S, D), bf)
    v = randn(rng, (B, Hkv, S, D), bf)
    do = randn(rng, (B, Hq, S, D), bf)
    m_ax, m_o = pair(mod, Hq, S, B)
    tq, tk, tv = T(q, dtype, True), T(k, dtype, True), T(v, dtype, True)
    out = ax.flash_attention(tq, tk, tv, score_mod=m_ax)
    out.backward(T(do, dtype))
    want = O.gqa_attention_bwd(q, k, v, do, score_mod=m_o)
    for name, got, w in zip(("dq", "dk", "dv"), (tq.grad, tk.grad, tv.grad), want):
        if bf:
            assert_bf16_grad_close(npy(got), w, f"{mod} {name}")
        else:
            assert_fp32_close(npy(got), w, f"{mod} {name}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mod", ["none", "causal_alibi", "window_alibi_wide"])
def test_backward_full_tiles(dtype, mod):
    """Long enough that whole 128x64 / 128x128 tiles lie inside the band, so
    the full-tile path (linear ALiBi, packed arithmetic) runs next to the
    boundary-tile path; ragged length; GQA with per-head slopes."""
    rng = np.random.default_rng(8)
    B, Hq, Hkv, S, D = 1, 4, 2, 700, 128
    q, k, v, do = (randn(rng, (B, h, S, D), True) for h in (Hq, Hkv, Hkv, Hq))
    m_ax, m_o = pair(mod, Hq, S, B)
    tq, tk, tv = T(q, dtype, True), T(k, dtype, True), T(v, dtype, True)
    out = ax.flash_attention(tq, tk, tv, score_mod=m_ax)
    out.backward(T(do, dtype))
    want = O.gqa_attention_bwd(q, k, v, do, score_mod=m_o)
    for name, got, w in zip(("dq", "dk", "dv"), (tq.grad, tk.grad, tv.grad), want):
        assert_bf16_grad_close(npy(got), w, f"{mod} {name}")


@pytest.mark.parametrize("layout", ["packed", "interleaved", "short_q"])
def test_document_mask_many_tiles(layout):
    """Document masks over several 128-row tiles: kernels restrict each tile's
    loop to the tiles whose id ranges overlap (exact for packed documents, a
    superset for interleaved ids) and skip or take the full-tile path from the
    per-tile id ranges.  Forward and backward against the oracle."""
    rng = np.random.default_rng(31)
    B, Hq, Hkv, D = 2, 4, 2, 128
    S = 100 if layout == "short_q" else 1100
    if layout == "interleaved":
        ids = np.stack([(np.arange(S) // 70) % 3, (np.arange(S) // 130) % 4]).astype(np.int32)
    else:
        lens0, lens1 = [300, 5, 129, 400, 266], [128, 256, 700, 16]
        ids = np.stack([np.repeat(np.arange(len(lens0)), lens0)[:S],
                        np.repeat(np.arange(len(lens1)), lens1)[:S]]).astype(np.int32)
    q, k, v, do = (randn(rng, (B, h, S, D), True) for h in (Hq, Hkv, Hkv, Hq))
    m_ax = ax.compose_score_mods(ax.document_mask_mod(ids), ax.causal_mod())
    m_o = O.compose_score_mods(O.document_mask_mod(ids), O.causal_mod())
    tq, tk, tv = T(q, grad=True), T(k, grad=True), T(v, grad=True)
    out = ax.flash_attention(tq, tk, tv, score_mod=m_ax)
    assert_bf16_close(npy(out), O.gqa_attention(q, k, v, score_mod=m_o), f"{layout} fwd")
    out.backward(T(do))
    want = O.gqa_attention_bwd(q, k, v, do, score_mod=m_o)
    for name, got, w in zip(("dq", "dk", "dv"), (tq.grad, tk.grad, tv.grad), want):
        assert_bf16_grad_close(npy(got), w, f"{layout} {name}")


def test_backward_fully_masked_rows():
    rng = np.random.default_rng(6)
    B, H, S, D = 1, 2, 140, 64
    q, k, v, do = (randn(rng, (B, H, S, D)) for _ in range(4))
    mask = np.ones((B, 1, S, S), bool)
    mask[0, 0, 3] = False
    tq, tk, tv = (T(x, torch.float32, True) for x in (q, k, v))
    out = ax.flash_attention(tq, tk, tv, mask=torch.tensor(mask, device=DEV), score_mod=ax.causal_mod())
    out.backward(T(do, torch.float32))
    want = O.standard_attention_bwd(q, k, v, do, mask=mask, score_mod=O.causal_mod())
    for name, got, w in zip(("dq", "dk", "dv"), (tq.grad, tk.grad, tv.grad), want):
        assert_fp32_close(npy(got), w, name)


def test_errors_match_reference_behaviour():
    q = torch.zeros(1, 3, 8, 64, device=DEV, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 8, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ax.flash_attention(q, k, k)
    with pytest.raises(NotImplementedError):
        ax.flash_attention(q, q, q, score_mod=lambda s, b, h, qi, kv: s)
    with pytest.raises(ValueError):
        ax.sliding_window_mod(0)
