"""Parity at the benchmarked shapes, against the oracle, at the stated bars.

The five workloads ``bench.py`` measures run here at their full sizes, on
the same seeded inputs the benchmark uses, and are compared with the oracle
where a full oracle run is out of reach by properties that are exact for
attention:

* a forward output row depends only on its query row and all of K/V, so
  sampled rows (``O.gqa_attention_rows``) are exact;
* a dQ row likewise needs only its query, dO and output rows and all of K/V;
* dK/dV rows of one kv tile need every query row's softmax, which the
  oracle evaluates blockwise over the query rows whose band reaches the tile
  (``O.gqa_kv_rows_grads``; pairs outside its ranges are masked and add 0).

Bars (``tests/_util.py``): bf16 outputs and gradients within 2e-2 max-abs
and 1e-2 mean relative (L1) error of the fp32 oracle; LSE within 1e-3.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import attnax_b200 as ax
import oracle as O
from tests._util import assert_bf16_close, errors

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _normal(shape, seed):
    """N(0,1) drawn in fp32 from default_rng(seed), rounded to bf16 (ties to even)."""
    x = np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)
    return torch.from_numpy(x).to(torch.bfloat16)


def _np(t):
    return t.detach().float().cpu().numpy()


def _check(got, want, what):
    assert_bf16_close(got, want, what)


def _rows(S, extra, seed):
    """Query positions to sample: tile and window edges plus random ones."""
    fixed = [0, 1, 63, 64, 127, 128, 255, 256, S // 2 - 1, S // 2, S - 129, S - 128, S - 2, S - 1] + list(extra)
    rnd = np.random.default_rng(seed).choice(S, size=48, replace=False)
    return np.unique(np.clip(np.concatenate([fixed, rnd]), 0, S - 1))


# ------------------------------------------------------------------ c2 --
C2 = dict(B=4, Hq=32, Hkv=8, S=8192, D=128, W=4096)


@pytest.fixture(scope="module")
def c2():
    """Forward + backward of the flash fwd+bwd benchmark workload:
    B4 Hq32 Hkv8 S8192 D128, sliding_window_mod(4096) + alibi_mod(32)."""
    from attnax_b200._spec import build_spec
    from attnax_b200.flash import bwd_raw, fwd_raw

    B, Hq, Hkv, S, D, W = (C2[k] for k in ("B", "Hq", "Hkv", "S", "D", "W"))
    hq, hk, hv, hdo = (_normal(s, i) for i, s in enumerate([(B, Hq, S, D), (B, Hkv, S, D), (B, Hkv, S, D),
                                                             (B, Hq, S, D)]))
    q, k, v, do = (t.to(DEV) for t in (hq, hk, hv, hdo))
    mod = ax.compose_score_mods(ax.sliding_window_mod(W), ax.alibi_mod(Hq))
    spec = build_spec(mod, None, batch=B, heads_q=Hq, seq_q=S, seq_kv=S, device=q.device)
    out, lse = fwd_raw(q, k, v, spec)
    dq, dk, dv = bwd_raw(q, k, v, out, lse, do, spec)
    torch.cuda.synchronize()
    return dict(q=_np(hq), k=_np(hk), v=_np(hv), do=_np(hdo), out=_np(out), lse=_np(lse), dq=_np(dq),
                dk=_np(dk), dv=_np(dv),
                mod=O.compose_score_mods(O.sliding_window_mod(W), O.alibi_mod(Hq)))


C2_PICKS = [(0, 0), (1, 13), (2, 22), (3, 31)]  # (batch, query head): steepest to flattest ALiBi slope


@pytest.mark.parametrize("b,h", C2_PICKS)
def test_c2_forward_rows(c2, b, h):
    rows = _rows(C2["S"], [C2["W"] - 1, C2["W"], C2["W"] + 1], seed=100 + h)
    o, lse, dq = O.gqa_attention_rows(c2["q"], c2["k"], c2["v"], b, [h], rows, score_mod=c2["mod"],
                                      d_out=c2["do"])
    _check(c2["out"][b, h, rows], o[0], f"c2 out b{b} h{h}")
    dl = float(np.abs(c2["lse"][b, h, rows] - lse[0]).max())
    print(f"[parity] c2 lse b{b} h{h}: max-abs {dl:.3e}")
    assert dl <= 1e-3
    _check(c2["dq"][b, h, rows], dq[0], f"c2 dq b{b} h{h}")


@pytest.mark.parametrize("b,hkv,tile", [(1, 5, 0), (2, 2, 40), (3, 7, 63)])
def test_c2_dk_dv_tile(c2, b, hkv, tile):
    """dK/dV of one 128-row kv tile, summed over the 4 query heads of its group
    and over every query row its window reaches."""
    S, W = C2["S"], C2["W"]
    k0, k1 = tile * 128, min(S, tile * 128 + 128)
    kv_rows = np.arange(k0, k1)
    q_range = (k0, min(S, k1 + W - 1))
    kv_range = (max(0, k0 - W + 1), min(S, k1 + W - 1))
    dk, dv = O.gqa_kv_rows_grads(c2["q"], c2["k"], c2["v"], c2["do"], b, hkv, kv_rows, score_mod=c2["mod"],
                                 q_range=q_range, kv_range=kv_range)
    _check(c2["dk"][b, hkv, k0:k1], dk, f"c2 dk b{b} hkv{hkv} tile{tile}")
    _check(c2["dv"][b, hkv, k0:k1], dv, f"c2 dv b{b} hkv{hkv} tile{tile}")


# ------------------------------------------------------------------ c3 --
def test_c3_paged_decode_full_config():
    """Paged decode over the benchmark's cache: 64 sequences, context lengths
    U[512, 32768], page 16, Hq32 Hkv8 D128, 1.2x pool, permuted block table.
    Every sequence is checked: the oracle attends each sequence's pages in
    table order (``O.paged_attention`` on a cache holding those pages)."""
    import bench

    c = bench.paged_setup("full")
    kp, vp, q = bench.paged_tensors(c, torch.device(DEV))
    cache = ax.PagedKVCache(kp, vp, torch.tensor(c["table"], device=DEV), torch.tensor(c["ctx"], device=DEV))
    got = _np(ax.paged_attention_batched(q, cache, max_context=int(c["ctx"].max())))
    qh = _np(q)
    worst = (0.0, 0.0)
    for s in range(c["nseq"]):
        n = int(c["ctx"][s])
        ids = torch.tensor(c["table"][s, :(n + c["bs"] - 1) // c["bs"]], device=DEV, dtype=torch.long)
        oc = O.PagedKVCache(_np(kp[ids]), _np(vp[ids]), np.arange(len(ids), dtype=np.int32)[None],
                            np.array([n], np.int32))
        want = O.paged_attention(qh[s], oc, 0)
        assert_bf16_close(got[s], want, f"c3 seq {s} (ctx {n})")
        worst = tuple(max(a, b) for a, b in zip(worst, errors(got[s], want)))
    print(f"[parity] c3 all 64 sequences: max-abs {worst[0]:.3e} mean-rel {worst[1]:.3e}")


# ------------------------------------------------------------------ c4 --
@pytest.fixture(scope="module")
def c4():
    """Document mask + causal, B1 S32768 Hq=Hkv=16 D128, geometric document
    lengths (mean 2048, min 64) from seed 0 -- the benchmark's documents."""
    import bench
    from attnax_b200._spec import build_spec
    from attnax_b200.flash import bwd_raw, fwd_raw

    S, H, D = 32768, 16, 128
    lens = bench.doc_lengths(S)
    ids = np.repeat(np.arange(len(lens)), lens)[None].astype(np.int32)
    hq, hk, hv, hdo = (_normal((1, H, S, D), 10 + i) for i in range(4))
    q, k, v, do = (t.to(DEV) for t in (hq, hk, hv, hdo))
    mod = ax.compose_score_mods(ax.document_mask_mod(ids), ax.causal_mod())
    spec = build_spec(mod, None, batch=1, heads_q=H, seq_q=S, seq_kv=S, device=q.device)
    out, lse = fwd_raw(q, k, v, spec)
    dq, dk, dv = bwd_raw(q, k, v, out, lse, do, spec)
    torch.cuda.synchronize()
    return dict(q=_np(hq), k=_np(hk), v=_np(hv), do=_np(hdo), out=_np(out), dq=_np(dq), dk=_np(dk), dv=_np(dv),
                lens=lens, ids=ids[0], mod=O.compose_score_mods(O.document_mask_mod(ids), O.causal_mod()))


def test_c4_forward_and_dq_rows(c4):
    starts = np.cumsum([0] + c4["lens"][:-1])
    ends = starts + np.asarray(c4["lens"]) - 1
    rows = _rows(32768, np.concatenate([starts, ends, starts + 1]), seed=4)
    print(f"[parity] c4 documents: {len(c4['lens'])}, lengths {c4['lens']}")
    for h in (0, 9, 15):
        o, _, dq = O.gqa_attention_rows(c4["q"], c4["k"], c4["v"], 0, [h], rows, score_mod=c4["mod"],
                                        d_out=c4["do"])
        _check(c4["out"][0, h, rows], o[0], f"c4 out h{h}")
        _check(c4["dq"][0, h, rows], dq[0], f"c4 dq h{h}")


def test_c4_dk_dv_tile_across_a_document_boundary(c4):
    ids = c4["ids"]
    S = len(ids)
    bounds = np.nonzero(np.diff(ids))[0] + 1
    tile = int(bounds[len(bounds) // 2]) // 128  # a tile holding the end of one document and the start of the next
    k0, k1 = tile * 128, min(S, tile * 128 + 128)
    d_first, d_last = ids[k0], ids[k1 - 1]
    lo = int(np.nonzero(ids == d_first)[0][0])
    hi = int(np.nonzero(ids == d_last)[0][-1]) + 1
    dk, dv = O.gqa_kv_rows_grads(c4["q"], c4["k"], c4["v"], c4["do"], 0, 3, np.arange(k0, k1),
                                 score_mod=c4["mod"], q_range=(k0, hi), kv_range=(lo, hi))
    _check(c4["dk"][0, 3, k0:k1], dk, f"c4 dk tile {tile}")
    _check(c4["dv"][0, 3, k0:k1], dv, f"c4 dv tile {tile}")


# ------------------------------------------------------------------ c5 --
@pytest.mark.parametrize("S", [16384, 65536])
def test_c5_causal_forward_at_shard_lengths(S):
    """The one-GPU causal forward of the ring workload (B1 Hq32 Hkv8 D128) at
    the per-rank lengths of 8 and 2 ranks."""
    Hq, Hkv, D = 32, 8, 128
    hq, hk, hv = (_normal(s, 20 + i) for i, s in enumerate([(1, Hq, S, D), (1, Hkv, S, D), (1, Hkv, S, D)]))
    out = _np(ax.flash_attention(hq.to(DEV), hk.to(DEV), hv.to(DEV), score_mod=ax.causal_mod()))
    qn, kn, vn = _np(hq), _np(hk), _np(hv)
    rows = _rows(S, [S // 4, 3 * S // 4], seed=S)
    for h in (0, 17, 31):
        o, _ = O.gqa_attention_rows(qn, kn, vn, 0, [h], rows, score_mod=O.causal_mod())
        _check(out[0, h, rows], o[0], f"c5 S{S} out h{h}")


# ------------------------------------------------------------------ c1 --
def test_c1_fp32_causal_backward():
    """fp32 B2 H8 S1024 D64 causal, forward and gradients within 1e-4 max-abs of
    the oracle evaluated in float64 (the fp32 kernels accumulate in fp32)."""
    from tests._util import assert_fp32_close

    rng = np.random.default_rng(0)
    q, k, v, do = (rng.standard_normal((2, 8, 1024, 64), dtype=np.float32) for _ in range(4))
    tq, tk, tv = (torch.tensor(x, device=DEV, requires_grad=True) for x in (q, k, v))
    out = ax.flash_attention(tq, tk, tv, score_mod=ax.causal_mod())
    out.backward(torch.tensor(do, device=DEV))
    d64 = [x.astype(np.float64) for x in (q, k, v, do)]
    want = O.standard_attention_bwd(*d64, score_mod=O.causal_mod())
    w_out = O.standard_attention(*d64[:3], score_mod=O.causal_mod())
    for name, got, w in zip(("out", "dq", "dk", "dv"), (out, tq.grad, tk.grad, tv.grad), (w_out,) + tuple(want)):
        mx, rel = errors(_np(got), w)
        print(f"[parity] c1 fp32 {name}: max-abs {mx:.3e} mean-rel {rel:.3e}")
        assert_fp32_close(_np(got), w, f"c1 {name}")
