"""The library's ring plan (attn_ring_plan, the schedule attn_ring_fwd runs) on CPU.

For every rank the plan's launches are executed with the oracle: each launch
attends its q rows (ring slots) to the K/V rows visiting at its hop, with the
band / ALiBi at the launch's global positions (or none for a batched
position-free launch), and folds the result into a running output by
log-sum-exp, as the kernel epilogue does.  The rows the plan marks final
must be written exactly once and equal the oracle's attention over the
global sequence (what ring_attention_reference computes, attention.py:694-721).
"""

import numpy as np
import pytest

import oracle as O
from attnax_b200 import _ring_capi

BAND_INF = 1 << 62


def _mods(kind, H, W):
    if kind == "causal":
        return O.causal_mod(), (0, BAND_INF), False
    if kind == "causal_alibi":
        return O.compose_score_mods(O.causal_mod(), O.alibi_mod(H)), (0, BAND_INF), True
    if kind == "window":
        return O.sliding_window_mod(W), (0, W - 1), False
    if kind == "window_sym_alibi":
        return O.compose_score_mods(O.sliding_window_mod(W, causal=False), O.alibi_mod(H)), (-(W - 1), W - 1), True
    return None, None, False


def _attend(q, k, v, mod, q0, k0):
    o, lse = O.standard_attention_lse(q, k, v, score_mod=mod, q_offset=q0, kv_offset=k0)
    # rows with nothing kept: an empty partial (the kernel returns lse = -inf)
    if mod is not None:
        s = O.attention_oracle._final_scores(q, k, None, mod, q0, k0)
        empty = np.all(s == np.finfo(s.dtype).min, axis=-1)
        o[empty] = 0.0
        lse[empty] = -np.inf
    return o, lse


def _merge(acc_o, acc_l, o, l):
    m = np.maximum(acc_l, l)
    with np.errstate(invalid="ignore"):
        wa = np.where(np.isinf(acc_l), 0.0, np.exp(acc_l - np.where(np.isinf(m), 0.0, m)))
        wp = np.where(np.isinf(l), 0.0, np.exp(l - np.where(np.isinf(m), 0.0, m)))
    tot = wa + wp
    nz = tot > 0
    ca = np.where(nz, wa / np.where(nz, tot, 1.0), 1.0)
    cp = np.where(nz, wp / np.where(nz, tot, 1.0), 0.0)
    new_o = ca[..., None] * np.nan_to_num(acc_o) + cp[..., None] * o
    new_l = np.where(nz, m + np.log(np.where(nz, tot, 1.0)), acc_l)
    return new_o, new_l


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("kind", ["causal", "causal_alibi", "window", "window_sym_alibi", "none"])
def test_ring_plan_reproduces_global_attention(world, kind):
    rng = np.random.default_rng(world * 7 + len(kind))
    H, Sl, D = 2, 12, 8
    S = Sl * world
    q, k, v = (rng.standard_normal((1, H, S, D)) for _ in range(3))
    mod, band, alibi = _mods(kind, H, W=Sl // 2 + 3)
    want = O.standard_attention(q, k, v, score_mod=mod)
    zig = band is not None and band[0] >= 0
    C = Sl // 2 if zig else Sl

    def held(r):
        return [2 * r, 2 * world - 1 - 2 * r] if zig else [r]

    for r in range(world):
        plan = _ring_capi.plan(world, r, Sl, zig, band, position_free=not alibi)
        mine = held(r)
        nq = len(mine)
        acc_o = np.full((1, H, nq * C, D), np.nan)
        acc_l = np.full((1, H, nq * C), -np.inf)
        out = np.full((1, H, nq * C, D), np.nan)
        written = np.zeros(nq * C, int)
        assert [l["hop"] for l in plan] == sorted(l["hop"] for l in plan)
        for l in plan:
            kvc = held((r - l["hop"]) % world)
            qrows = np.concatenate([np.arange(c * C, (c + 1) * C) for c in mine[l["q_slot"]:l["q_slot"] + l["q_chunks"]]])
            krows = np.concatenate([np.arange(c * C, (c + 1) * C) for c in kvc[l["kv_slot"]:l["kv_slot"] + l["kv_chunks"]]])
            if l["masked"]:
                assert l["q_chunks"] == l["kv_chunks"] == 1
                assert l["q_start"] == qrows[0] and l["kv_start"] == krows[0]
                o, lse = _attend(q[:, :, qrows], k[:, :, krows], v[:, :, krows], mod, l["q_start"], l["kv_start"])
            else:
                assert not alibi  # only position-free chains batch
                o, lse = _attend(q[:, :, qrows], k[:, :, krows], v[:, :, krows], None, 0, 0)
                # a batched pair must be kept whole by the band
                d = qrows[:, None] - krows[None, :]
                if band is not None:
                    assert np.all((d >= band[0]) & (d <= band[1]))
            sl = slice(l["q_slot"] * C, (l["q_slot"] + l["q_chunks"]) * C)
            acc_o[:, :, sl], acc_l[:, :, sl] = _merge(acc_o[:, :, sl], acc_l[:, :, sl], o, lse)
            fin = np.arange(sl.start, sl.stop) >= sl.start + l["final_from"]
            out[:, :, np.arange(sl.start, sl.stop)[fin]] = acc_o[:, :, np.arange(sl.start, sl.stop)[fin]]
            written[np.arange(sl.start, sl.stop)[fin]] += 1
            if zig and l["hop"] == 0 and l["local"]:
                assert (l["q_slot"], l["kv_slot"]) == (0, 0)
        assert np.all(written == 1), f"rank {r}: final rows {written}"
        rows = np.concatenate([np.arange(c * C, (c + 1) * C) for c in mine])
        np.testing.assert_allclose(out, want[:, :, rows], atol=1e-12, err_msg=f"{kind} P={world} rank {r}")


def test_ring_plan_balances_causal_work():
    """Zig-zag: every rank attends the same number of (q, kv) positions per hop."""
    world, Sl = 8, 64
    C = Sl // 2
    for hop in range(world):
        per_rank = []
        for r in range(world):
            held = lambda x: [2 * x, 2 * world - 1 - 2 * x]  # noqa: E731
            n = 0
            for l in _ring_capi.plan(world, r, Sl, True, (0, BAND_INF), position_free=True):
                if l["hop"] != hop:
                    continue
                kvc = held((r - hop) % world)
                for qc in held(r)[l["q_slot"]:l["q_slot"] + l["q_chunks"]]:
                    for kc in kvc[l["kv_slot"]:l["kv_slot"] + l["kv_chunks"]]:
                        qi = np.arange(qc * C, (qc + 1) * C)[:, None]
                        ki = np.arange(kc * C, (kc + 1) * C)[None, :]
                        n += int(np.sum(ki <= qi))
            per_rank.append(n)
        assert len(set(per_rank)) == 1, (hop, per_rank)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ring_plan_batches_q_chunks_only_in_final_launches(world):
    """A launch over both q chunks writes their finished rows (final_from 0):
    the batched shape that folds rows into the fp32 running result measured
    slower than two separate launches, so the plan never issues it."""
    for r in range(world):
        for l in _ring_capi.plan(world, r, 64, True, (0, BAND_INF), position_free=True):
            if l["q_chunks"] == 2:
                assert l["final_from"] == 0, (world, r, l)
