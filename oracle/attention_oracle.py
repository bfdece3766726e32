"""Numpy restatement of attnax's attention hot path (test infrastructure).

Every function here is the checker for the CUDA kernels in ``attnax_b200``;
none of it is shipped or called by the product.  Each function cites the
reference file:line (paths inside the attnax project) whose behaviour it
restates.  Arithmetic follows the reference: scores are computed in the
dtype of the query (float32 in every parity test, float64 when the checker
itself is being checked), masked scores become ``finfo(dtype).min`` rather
than ``-inf``, and a fully masked row therefore averages V uniformly.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import numpy as np

__all__ = [
    "position_indices", "apply_score_mod", "compose_score_mods",
    "mask_mod_to_boolean_mask", "alibi_slopes", "alibi_mod", "causal_mod",
    "sliding_window_mod", "prefix_lm_mod", "document_mask_mod",
    "additive_bias_mod", "mask_mod_to_score_mod", "make_padding_mask",
    "make_causal_mask", "make_sliding_window_mask", "make_document_mask",
    "combine_masks", "standard_attention", "standard_attention_lse",
    "memory_efficient_attention", "attention_rows", "gqa_attention_rows", "gqa_kv_rows_grads",
    "standard_attention_bwd",
    "repeat_kv", "gqa_attention", "gqa_attention_bwd",
    "ring_attention_partitioned", "PagedKVCache", "init_paged_kv_cache",
    "allocate_blocks", "append_kv", "gather_kv", "paged_attention",
    "paged_attention_batched", "softmax_scale", "bf16_round", "KVLayerCache",
    "init_kv_layer_cache", "update_kv_layer_cache", "kv_cache_attention", "rope_inv_freq",
    "rope_cos_sin_table", "rope_cos_sin_from_positions", "apply_rope", "mha_attention_core",
]


# ----------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------

def bf16_round(x: np.ndarray) -> np.ndarray:
    """Rounds float32 values to the nearest bfloat16 (ties to even).

    Returns float32 holding bf16-representable values; the same rounding as
    ``torch.Tensor.to(torch.bfloat16)``.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    u = ((u + rounding) >> 16) << 16
    out = u.astype(np.uint32).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, x, out)
    return out


def softmax_scale(head_dim: int, dtype=np.float32):
    """``rsqrt(head_dim)`` in the query dtype (kernels/attention.py:54-55)."""
    dtype = np.dtype(dtype)
    return dtype.type(1.0) / np.sqrt(dtype.type(head_dim))


def _softmax(x: np.ndarray) -> np.ndarray:
    """``jax.nn.softmax`` along the last axis (max-subtracted)."""
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=-1, keepdims=True)


# ----------------------------------------------------------------------------
# kernels/_api.py
# ----------------------------------------------------------------------------

def position_indices(batch, num_heads, seq_q, seq_kv, q_offset=0, kv_offset=0):
    """Broadcast index arrays ``(b, h, q, kv)`` (kernels/_api.py:115-123).

    ``q_offset``/``kv_offset`` give global positions, as the blockwise and
    ring paths pass them (kernels/attention.py:168-177, :651-656).
    """
    b = np.arange(batch, dtype=np.int32)[:, None, None, None]
    h = np.arange(num_heads, dtype=np.int32)[None, :, None, None]
    q = (np.arange(seq_q, dtype=np.int32) + q_offset)[None, None, :, None]
    kv = (np.arange(seq_kv, dtype=np.int32) + kv_offset)[None, None, None, :]
    return b, h, q, kv


def apply_score_mod(scores, score_mod, q_offset=0, kv_offset=0):
    """Applies ``score_mod`` with position indices (kernels/_api.py:126-136)."""
    if score_mod is None:
        return scores
    bsz, nh, sq, skv = scores.shape
    return score_mod(scores, *position_indices(bsz, nh, sq, skv, q_offset, kv_offset))


def compose_score_mods(*score_mods):
    """Left-to-right composition, ``None`` skipped (kernels/_api.py:166-196)."""
    active = [m for m in score_mods if m is not None]
    if not active:
        return None
    if len(active) == 1:
        return active[0]

    def composed(scores, b_idx, h_idx, q_idx, kv_idx):
        for m in active:
            scores = m(scores, b_idx, h_idx, q_idx, kv_idx)
        return scores

    return composed


def mask_mod_to_boolean_mask(mask_mod, *, batch, num_heads, seq_q, seq_kv):
    """Materialises a MaskMod (kernels/_api.py:139-163)."""
    out = mask_mod(*position_indices(batch, num_heads, seq_q, seq_kv))
    return np.broadcast_to(out, (batch, num_heads, seq_q, seq_kv))


# ----------------------------------------------------------------------------
# kernels/score_mods.py
# ----------------------------------------------------------------------------

def alibi_slopes(num_heads: int) -> np.ndarray:
    """Per-head ALiBi slopes (kernels/score_mods.py:14-45)."""

    def power_of_two(n):
        start = 2.0 ** (-(2.0 ** -(math.log2(n) - 3)))
        return [start * (start ** i) for i in range(n)]

    if (num_heads & (num_heads - 1)) == 0:
        return np.asarray(power_of_two(num_heads), dtype=np.float32)
    closest = 2 ** math.floor(math.log2(num_heads))
    base = power_of_two(closest)
    extra = power_of_two(2 * closest)[0::2][: num_heads - closest]
    return np.asarray(base + extra, dtype=np.float32)


def alibi_mod(num_heads: int):
    """``s - m_h * |q - kv|`` (kernels/score_mods.py:48-81).

    The reference broadcasts a ``(1, H, 1, 1)`` slope array against the full
    head axis; gathering the slopes with ``h_idx`` gives the same values for
    that index array and also serves score tiles of a subset of heads (the
    row-sampled checks below pass the real head ids).
    """
    slopes = alibi_slopes(num_heads)

    def _mod(scores, b_idx, h_idx, q_idx, kv_idx):
        dt = scores.dtype
        dist = np.abs(q_idx.astype(dt) - kv_idx.astype(dt))
        return scores - slopes.astype(dt)[np.asarray(h_idx)] * dist

    return _mod


def causal_mod():
    """Keep ``kv <= q`` (kernels/score_mods.py:84-104)."""

    def _mod(scores, b_idx, h_idx, q_idx, kv_idx):
        return np.where(kv_idx <= q_idx, scores, np.finfo(scores.dtype).min)

    return _mod


def sliding_window_mod(window_size: int, *, causal: bool = True):
    """Window mask (kernels/score_mods.py:107-145); ``W <= 0`` raises."""
    if window_size <= 0:
        raise ValueError(f"window_size must be positive, got {window_size}")

    def _mod(scores, b_idx, h_idx, q_idx, kv_idx):
        if causal:
            keep = (kv_idx <= q_idx) & (q_idx - kv_idx < window_size)
        else:
            keep = np.abs(q_idx - kv_idx) < window_size
        return np.where(keep, scores, np.finfo(scores.dtype).min)

    return _mod


def prefix_lm_mod(prefix_lengths):
    """Bidirectional prefix, causal after (kernels/score_mods.py:148-178)."""
    prefix_lengths = np.asarray(prefix_lengths, dtype=np.int32)

    def _mod(scores, b_idx, h_idx, q_idx, kv_idx):
        pref = prefix_lengths[b_idx[..., 0, 0, 0]][:, None, None, None]
        keep = (kv_idx < pref) | (kv_idx <= q_idx)
        return np.where(keep, scores, np.finfo(scores.dtype).min)

    return _mod


def document_mask_mod(document_ids):
    """Same-document mask (kernels/score_mods.py:181-213).

    The reference precomputes ``ids[:, :, None] == ids[:, None, :]`` and
    indexes it with the q/kv positions; comparing the gathered ids is the
    same selection without the ``(B, S, S)`` table.
    """
    ids = np.asarray(document_ids, dtype=np.int32)

    def _mod(scores, b_idx, h_idx, q_idx, kv_idx):
        # Rows of the batches in b_idx (all of them for the full index array).
        rows = ids[np.asarray(b_idx)[:, 0, 0, 0]]
        qi = rows[:, q_idx[0, 0, :, 0]]
        ki = rows[:, kv_idx[0, 0, 0, :]]
        keep = (qi[:, :, None] == ki[:, None, :])[:, None, :, :]
        return np.where(keep, scores, np.finfo(scores.dtype).min)

    return _mod


def additive_bias_mod(bias):
    """``s + bias`` (kernels/score_mods.py:216-237)."""
    bias = np.asarray(bias)

    def _mod(scores, b_idx, h_idx, q_idx, kv_idx):
        return scores + bias.astype(scores.dtype)

    return _mod


def mask_mod_to_score_mod(mask_mod):
    """MaskMod → ScoreMod (kernels/score_mods.py:240-264)."""

    def _mod(scores, b_idx, h_idx, q_idx, kv_idx):
        keep = mask_mod(b_idx, h_idx, q_idx, kv_idx)
        return np.where(keep, scores, np.finfo(scores.dtype).min)

    return _mod


# ----------------------------------------------------------------------------
# masking.py
# ----------------------------------------------------------------------------

def make_padding_mask(input_ids, pad_token_id=0):
    """Key-padding mask ``(B,1,1,S)`` (masking.py:10-24)."""
    return (np.asarray(input_ids) != pad_token_id)[:, None, None, :]


def make_causal_mask(seq_len):
    """Lower-triangular mask ``(1,1,S,S)`` (masking.py:27-38)."""
    return np.tril(np.ones((seq_len, seq_len), dtype=bool))[None, None]


def make_sliding_window_mask(seq_q, seq_kv=None, *, window_size, causal=True):
    """Window mask ``(1,1,Sq,Skv)`` (masking.py:41-72)."""
    if window_size <= 0:
        raise ValueError(f"window_size must be positive, got {window_size}")
    if seq_kv is None:
        seq_kv = seq_q
    q = np.arange(seq_q)[:, None]
    kv = np.arange(seq_kv)[None, :]
    if causal:
        m = (kv <= q) & (q - kv < window_size)
    else:
        m = np.abs(q - kv) < window_size
    return m[None, None]


def make_document_mask(document_ids):
    """Same-document mask ``(B,1,S,S)`` (masking.py:75-89)."""
    ids = np.asarray(document_ids)
    return (ids[:, :, None] == ids[:, None, :])[:, None]


def combine_masks(*masks):
    """Logical AND, ``None`` skipped (masking.py:92-109)."""
    out = None
    for m in masks:
        if m is None:
            continue
        out = m if out is None else (out & m)
    return out


# ----------------------------------------------------------------------------
# kernels/attention.py
# ----------------------------------------------------------------------------

def _final_scores(q, k, mask, score_mod, q_offset=0, kv_offset=0, q_positions=None):
    """Scores after scale, score_mod and mask (kernels/attention.py:54-62)."""
    dt = q.dtype
    scale = softmax_scale(q.shape[-1], dt)
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
    if score_mod is not None:
        bsz, nh, sq, skv = s.shape
        b, h, qi, kvi = position_indices(bsz, nh, sq, skv, q_offset, kv_offset)
        if q_positions is not None:
            qi = np.asarray(q_positions, dtype=np.int32)[None, None, :, None]
        s = score_mod(s, b, h, qi, kvi)
    if mask is not None:
        s = np.where(mask, s, np.finfo(s.dtype).min)
    return s


def standard_attention(query, key, value, *, mask=None, score_mod=None):
    """Dense softmax attention (kernels/attention.py:17-71), no dropout."""
    s = _final_scores(query, key, mask, score_mod)
    p = _softmax(s)
    return np.einsum("bhqk,bhkd->bhqd", p, value).astype(query.dtype)


def standard_attention_lse(query, key, value, *, mask=None, score_mod=None, q_offset=0, kv_offset=0):
    """``standard_attention`` plus the natural-log LSE of each score row.

    ``q_offset``/``kv_offset`` are the global positions of row/column 0 given
    to ``score_mod`` (one ring step, attention.py:641-657).
    """
    s = _final_scores(query, key, mask, score_mod, q_offset, kv_offset)
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp(s - m)
    l = np.sum(e, axis=-1, keepdims=True)
    out = np.einsum("bhqk,bhkd->bhqd", e / l, value).astype(query.dtype)
    return out, (m + np.log(l))[..., 0]


def memory_efficient_attention(query, key, value, *, mask=None, score_mod=None,
                               block_size=512):
    """Blockwise online softmax (kernels/attention.py:74-206), no dropout.

    Same block loop, accumulators in the query dtype, ``l + 1e-10``
    denominator, and the fall-back to ``standard_attention`` when both
    sequence axes fit one block (:122-132).
    """
    bsz, nh, sq, d = query.shape
    skv = key.shape[2]
    if sq <= block_size and skv <= block_size:
        return standard_attention(query, key, value, mask=mask, score_mod=score_mod)
    dt = query.dtype
    scale = softmax_scale(d, dt)
    neg = np.finfo(dt).min
    out = np.zeros_like(query)
    if mask is not None:
        mask = np.broadcast_to(mask, mask.shape[:-2] + (sq, skv))
    for q0 in range(0, sq, block_size):
        q1 = min(q0 + block_size, sq)
        qb = query[:, :, q0:q1]
        m_run = np.full((bsz, nh, q1 - q0, 1), neg, dtype=dt)
        l_run = np.zeros((bsz, nh, q1 - q0, 1), dtype=dt)
        o_run = np.zeros((bsz, nh, q1 - q0, d), dtype=dt)
        for k0 in range(0, skv, block_size):
            k1 = min(k0 + block_size, skv)
            s = np.einsum("bhqd,bhkd->bhqk", qb, key[:, :, k0:k1]) * scale
            if score_mod is not None:
                b, h, qi, kvi = position_indices(bsz, nh, q1 - q0, k1 - k0, q0, k0)
                s = score_mod(s, b, h, qi, kvi)
            if mask is not None:
                s = np.where(mask[..., q0:q1, k0:k1], s, neg)
            m_blk = np.max(s, axis=-1, keepdims=True)
            m_new = np.maximum(m_run, m_blk)
            alpha = np.exp(m_run - m_new)
            p = np.exp(s - m_new)
            l_run = l_run * alpha + np.sum(p, axis=-1, keepdims=True)
            o_run = o_run * alpha + np.einsum("bhqk,bhkd->bhqd", p, value[:, :, k0:k1])
            m_run = m_new
        out[:, :, q0:q1] = o_run / (l_run + dt.type(1e-10))
    return out


def attention_rows(query, key, value, rows, *, mask=None, score_mod=None):
    """Exact output rows ``rows`` of ``standard_attention``.

    One output row depends only on its query row and all of K/V, so a row
    subset is exact for shapes whose full score matrix does not fit.  Query
    positions passed to ``score_mod`` are the global ``rows``.
    """
    rows = np.asarray(rows)
    q = query[:, :, rows]
    m = None
    if mask is not None:
        full = np.broadcast_to(mask, mask.shape[:-2] + (query.shape[2], key.shape[2]))
        m = full[..., rows, :]
    s = _final_scores(q, key, m, score_mod, q_positions=rows)
    p = _softmax(s)
    return np.einsum("bhqk,bhkd->bhqd", p, value).astype(query.dtype)


def _mod_tile(score_mod, scores, b, heads, rows, cols):
    """``score_mod`` on a score tile of batch ``b``, heads ``heads``, global
    query positions ``rows`` and key positions ``cols``: the index arrays
    carry those ids, so the tile sees exactly the values the full
    ``(B, H, Sq, Skv)`` evaluation gives it (kernels/_api.py:115-136).
    Returns the modified scores and the 0/1 Jacobian of the mod chain
    (built-in mods are additive or ``where`` selections; see
    ``_score_jacobian``)."""
    if score_mod is None:
        return scores, np.ones(scores.shape, dtype=scores.dtype)
    b_idx = np.asarray([b], dtype=np.int32)[:, None, None, None]
    h_idx = np.asarray(heads, dtype=np.int32)[None, :, None, None]
    q_idx = np.asarray(rows, dtype=np.int32)[None, None, :, None]
    kv_idx = np.asarray(cols, dtype=np.int32)[None, None, None, :]
    out = score_mod(scores, b_idx, h_idx, q_idx, kv_idx)
    z = np.zeros((1, 1) + scores.shape[2:], dtype=np.float64)
    jac = np.empty(scores.shape, dtype=scores.dtype)
    for i, h in enumerate(heads):
        hi = np.asarray([h], dtype=np.int32)[None, :, None, None]
        f0 = np.asarray(score_mod(z, b_idx, hi, q_idx, kv_idx), dtype=np.float64)
        f1 = np.asarray(score_mod(z + 1.0, b_idx, hi, q_idx, kv_idx), dtype=np.float64)
        jac[:, i] = np.rint(f1 - f0)[0, 0]
    return np.asarray(out, dtype=scores.dtype), jac


def gqa_attention_rows(query, key, value, b, heads, rows, *, score_mod=None, d_out=None, q_offset=0):
    """Exact rows of ``gqa_attention`` (repeat K/V, then ``standard_attention``,
    kernels/attention.py:54-71 after attention.py:32-39) and, with ``d_out``,
    the matching rows of its query gradient.

    One output row depends only on its query row and all of K/V, so rows of a
    shape whose full score matrix does not fit are still exact.  ``b`` is one
    batch index, ``heads`` query heads, ``rows`` query positions (0-based,
    global); ``d_out`` is the full upstream gradient (B, Hq, Sq, D).  Returns
    ``out (len(heads), len(rows), D)``, natural-log ``lse (len(heads),
    len(rows))`` and, with ``d_out``, ``dq`` of the same shape as ``out``
    (``dS = P ∘ (dO Vᵀ − rowsum(dO ∘ O))`` masked by the mod Jacobian,
    ``dQ = scale · dS K``).  ``query``/``d_out`` may hold only the rows from
    global position ``q_offset`` on (one rank's shard of a sequence whose
    keys are all given).
    """
    rows = np.asarray(rows)
    hq, hkv = query.shape[1], key.shape[1]
    grp = hq // hkv
    dt = query.dtype
    scale = softmax_scale(query.shape[-1], dt)
    cols = np.arange(key.shape[2])
    outs, lses, dqs = [], [], []
    for h in heads:
        kh, vh = key[b, h // grp], value[b, h // grp]
        qr = query[b, h, rows - q_offset]
        s = (qr @ kh.T * scale)[None, None]
        s, jac = _mod_tile(score_mod, s, b, [h], rows, cols)
        s, jac = s[0, 0], jac[0, 0]
        m = np.max(s, axis=-1, keepdims=True)
        e = np.exp(s - m)
        l = np.sum(e, axis=-1, keepdims=True)
        p = e / l
        o = p @ vh
        outs.append(o.astype(dt))
        lses.append((m + np.log(l))[:, 0])
        if d_out is not None:
            dor = d_out[b, h, rows - q_offset]
            delta = np.sum(dor * o, axis=-1, keepdims=True)
            ds = p * (dor @ vh.T - delta) * jac
            dqs.append((ds @ kh * scale).astype(dt))
    res = (np.stack(outs), np.stack(lses))
    return res + (np.stack(dqs),) if d_out is not None else res


def gqa_kv_rows_grads(query, key, value, d_out, b, hkv, kv_rows, *, score_mod=None, q_block=512,
                      q_range=None, kv_range=None):
    """dK and dV rows ``kv_rows`` of kv head ``hkv`` (batch ``b``) of
    ``gqa_attention``: the gradient autodiff gives through ``jnp.repeat``
    (attention.py:32-39), i.e. the per-head ``dK = scale · dSᵀ Q``,
    ``dV = Pᵀ dO`` summed over the query heads sharing the kv head.

    Each query row's softmax needs its whole score row, so the rows are
    processed in blocks of ``q_block`` against all keys.  ``q_range`` /
    ``kv_range`` ((lo, hi) positions) restrict the work; the result stays
    exact when every (q, kv) pair outside them is masked (finfo.min scores
    contribute exactly 0 to a softmax row that keeps any key).
    """
    kv_rows = np.asarray(kv_rows)
    hq, nh_kv = query.shape[1], key.shape[1]
    grp = hq // nh_kv
    dt = query.dtype
    scale = softmax_scale(query.shape[-1], dt)
    q_lo, q_hi = q_range if q_range is not None else (0, query.shape[2])
    k_lo, k_hi = kv_range if kv_range is not None else (0, key.shape[2])
    cols = np.arange(k_lo, k_hi)
    kh, vh = key[b, hkv, k_lo:k_hi], value[b, hkv, k_lo:k_hi]
    sel = kv_rows - k_lo
    dk = np.zeros((len(kv_rows), key.shape[-1]), dtype=np.float64)
    dv = np.zeros_like(dk)
    for h in range(hkv * grp, (hkv + 1) * grp):
        for r0 in range(q_lo, q_hi, q_block):
            rows = np.arange(r0, min(q_hi, r0 + q_block))
            qr, dor = query[b, h, rows], d_out[b, h, rows]
            s = (qr @ kh.T * scale)[None, None]
            s, jac = _mod_tile(score_mod, s, b, [h], rows, cols)
            s, jac = s[0, 0], jac[0, 0]
            m = np.max(s, axis=-1, keepdims=True)
            e = np.exp(s - m)
            p = e / np.sum(e, axis=-1, keepdims=True)
            o = p @ vh
            delta = np.sum(dor * o, axis=-1, keepdims=True)
            ps = p[:, sel]
            ds = ps * (dor @ vh[sel].T - delta) * jac[:, sel]
            dv += ps.T.astype(np.float64) @ dor
            dk += (ds.T.astype(np.float64) @ qr) * scale
    return dk.astype(dt), dv.astype(dt)


def _score_jacobian(q, k, mask, score_mod):
    """d(final score)/d(scaled score), elementwise, for the built-in mods.

    Every built-in ScoreMod is either additive (Jacobian 1) or a
    ``where(keep, s, finfo.min)`` selection (Jacobian ``keep``), and the
    ``mask=`` argument is a selection too.  Evaluating the mod chain at
    ``s`` and ``s + 1`` recovers that 0/1 Jacobian exactly.
    """
    bsz, nh, sq, _ = q.shape
    skv = k.shape[2]
    s0 = np.zeros((bsz, nh, sq, skv), dtype=np.float64)
    b, h, qi, kvi = position_indices(bsz, nh, sq, skv)
    f0 = s0 if score_mod is None else score_mod(s0, b, h, qi, kvi)
    f1 = s0 + 1.0 if score_mod is None else score_mod(s0 + 1.0, b, h, qi, kvi)
    g = np.rint(np.asarray(f1, dtype=np.float64) - np.asarray(f0, dtype=np.float64))
    if mask is not None:
        g = np.where(mask, g, 0.0)
    return np.broadcast_to(g, (bsz, nh, sq, skv))


def standard_attention_bwd(query, key, value, d_out, *, mask=None, score_mod=None):
    """Gradients of ``standard_attention`` w.r.t. q, k, v.

    The reference has no hand-written backward: its gradient is JAX autodiff
    of kernels/attention.py:54-71.  This is that derivative in closed form:
    ``dV = Pᵀ dO``, ``dS = P ∘ (dO Vᵀ − rowsum(dO ∘ O))`` masked by the
    score Jacobian (0 where a ``where`` replaced the score), and
    ``dQ = scale · dS K``, ``dK = scale · dSᵀ Q``.  A fully masked row keeps
    its uniform P in ``dV`` and contributes nothing to ``dQ``/``dK``.
    """
    dt = query.dtype
    scale = softmax_scale(query.shape[-1], dt)
    s = _final_scores(query, key, mask, score_mod)
    p = _softmax(s)
    out = np.einsum("bhqk,bhkd->bhqd", p, value)
    dv = np.einsum("bhqk,bhqd->bhkd", p, d_out)
    dp = np.einsum("bhqd,bhkd->bhqk", d_out, value)
    delta = np.sum(d_out * out, axis=-1, keepdims=True)
    ds = p * (dp - delta) * _score_jacobian(query, key, mask, score_mod).astype(dt)
    dq = np.einsum("bhqk,bhkd->bhqd", ds, key) * scale
    dk = np.einsum("bhqk,bhqd->bhkd", ds, query) * scale
    return dq.astype(dt), dk.astype(dt), dv.astype(dt)


def repeat_kv(x, num_heads):
    """KV-head repeat before the kernel call (attention.py:32-39)."""
    hkv = x.shape[1]
    if hkv == num_heads:
        return x
    return np.repeat(x, num_heads // hkv, axis=1)


def gqa_attention(query, key, value, *, mask=None, score_mod=None):
    """What ``MultiHeadAttention`` computes for ``Hkv < Hq``: repeat, then attend."""
    hq = query.shape[1]
    return standard_attention(query, repeat_kv(key, hq), repeat_kv(value, hq),
                              mask=mask, score_mod=score_mod)


def gqa_attention_bwd(query, key, value, d_out, *, mask=None, score_mod=None):
    """Autodiff through ``jnp.repeat``: dK/dV summed over each head group."""
    hq, hkv = query.shape[1], key.shape[1]
    dq, dk, dv = standard_attention_bwd(query, repeat_kv(key, hq), repeat_kv(value, hq),
                                        d_out, mask=mask, score_mod=score_mod)
    if hkv != hq:
        g = hq // hkv
        dk = dk.reshape(dk.shape[0], hkv, g, *dk.shape[2:]).sum(axis=2)
        dv = dv.reshape(dv.shape[0], hkv, g, *dv.shape[2:]).sum(axis=2)
    return dq, dk, dv


def ring_attention_partitioned(query, key, value, num_shards, *, mask=None,
                               score_mod=None):
    """The ring recurrence of kernels/attention.py:617-684 over ``num_shards``.

    ``query/key/value`` are the global ``(B, H, S, D)`` arrays; shard ``r``
    holds rows ``[r*S/P, (r+1)*S/P)``.  Each shard runs the reference's scan:
    at step ``i`` it holds the K/V of owner ``(r - i) mod P`` (:640), uses
    global offsets for the score_mod (:641-656), applies the same local
    ``mask`` every step (:659-660), and finishes with ``o / (l + 1e-10)``
    (:684).  Returns the concatenated shard outputs.
    """
    bsz, nh, s_glob, d = query.shape
    P = num_shards
    assert s_glob % P == 0
    sl = s_glob // P
    dt = query.dtype
    scale = softmax_scale(d, dt)
    neg = np.finfo(dt).min
    outs = []
    for r in range(P):
        q = query[:, :, r * sl:(r + 1) * sl]
        m_run = np.full((bsz, nh, sl, 1), neg, dtype=dt)
        l_run = np.zeros((bsz, nh, sl, 1), dtype=dt)
        o_run = np.zeros_like(q)
        for i in range(P):
            owner = (r - i) % P
            k = key[:, :, owner * sl:(owner + 1) * sl]
            v = value[:, :, owner * sl:(owner + 1) * sl]
            s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
            if score_mod is not None:
                s = score_mod(s, *position_indices(bsz, nh, sl, sl, r * sl, owner * sl))
            if mask is not None:
                s = np.where(mask, s, neg)
            m_new = np.maximum(m_run, np.max(s, axis=-1, keepdims=True))
            alpha = np.exp(m_run - m_new)
            p = np.exp(s - m_new)
            l_run = l_run * alpha + np.sum(p, axis=-1, keepdims=True)
            o_run = o_run * alpha + np.einsum("bhqk,bhkd->bhqd", p, v)
            m_run = m_new
        outs.append(o_run / (l_run + dt.type(1e-10)))
    return np.concatenate(outs, axis=2)


# ----------------------------------------------------------------------------
# paged_cache.py and kernels/paged.py
# ----------------------------------------------------------------------------

@dataclass
class PagedKVCache:
    """Pool ``(num_blocks, block_size, Hkv, D)`` + block table (paged_cache.py:12-48)."""

    key_pool: np.ndarray
    value_pool: np.ndarray
    block_table: np.ndarray
    seq_lengths: np.ndarray

    @property
    def num_blocks(self):
        return int(self.key_pool.shape[0])

    @property
    def block_size(self):
        return int(self.key_pool.shape[1])

    @property
    def num_kv_heads(self):
        return int(self.key_pool.shape[2])

    @property
    def head_dim(self):
        return int(self.key_pool.shape[3])


def init_paged_kv_cache(*, num_blocks, block_size, num_kv_heads, head_dim,
                        batch_size, max_blocks_per_seq, dtype=np.float32):
    """Zero pools, ``-1`` block table, zero lengths (paged_cache.py:51-89)."""
    kp = np.zeros((num_blocks, block_size, num_kv_heads, head_dim), dtype=dtype)
    return PagedKVCache(kp, np.zeros_like(kp),
                        np.full((batch_size, max_blocks_per_seq), -1, dtype=np.int32),
                        np.zeros((batch_size,), dtype=np.int32))


def allocate_blocks(cache, *, sequence_idx, num_new_tokens, free_block_ids):
    """Fills block-table slots from ``free_block_ids`` (paged_cache.py:92-141)."""
    bs = cache.block_size
    cur = int(cache.seq_lengths[sequence_idx])
    have = (cur + bs - 1) // bs
    need = (cur + num_new_tokens + bs - 1) // bs
    new = need - have
    free_block_ids = np.asarray(free_block_ids)
    if new > int(free_block_ids.shape[0]):
        raise ValueError(f"free_block_ids has {int(free_block_ids.shape[0])} entries but "
                         f"{new} are needed")
    table = cache.block_table.copy()
    for i in range(new):
        table[sequence_idx, have + i] = free_block_ids[i]
    return PagedKVCache(cache.key_pool, cache.value_pool, table, cache.seq_lengths), new


def append_kv(cache, sequence_idx, keys_new, values_new):
    """Per-token scatter into the pool (paged_cache.py:144-198)."""
    if keys_new.shape != values_new.shape:
        raise ValueError(f"keys_new shape {keys_new.shape} != values_new shape "
                         f"{values_new.shape}")
    bs = cache.block_size
    start = int(cache.seq_lengths[sequence_idx])
    kp = cache.key_pool.copy()
    vp = cache.value_pool.copy()
    for t in range(keys_new.shape[0]):
        logical, off = divmod(start + t, bs)
        phys = int(cache.block_table[sequence_idx, logical])
        if phys < 0:
            raise ValueError(f"block_table[{sequence_idx}, {logical}] is unallocated; call "
                             "allocate_blocks before append_kv.")
        kp[phys, off] = keys_new[t]
        vp[phys, off] = values_new[t]
    lens = cache.seq_lengths.copy()
    lens[sequence_idx] += keys_new.shape[0]
    return PagedKVCache(kp, vp, cache.block_table, lens)


def gather_kv(cache, sequence_idx):
    """Contiguous ``(seq_len, Hkv, D)`` view of one sequence (paged_cache.py:201-231)."""
    seq_len = int(cache.seq_lengths[sequence_idx])
    bs = cache.block_size
    nblk = (seq_len + bs - 1) // bs
    if nblk == 0:
        empty = np.zeros((0, cache.num_kv_heads, cache.head_dim), dtype=cache.key_pool.dtype)
        return empty, empty, 0
    ids = cache.block_table[sequence_idx, :nblk]
    k = cache.key_pool[ids].reshape(nblk * bs, cache.num_kv_heads, cache.head_dim)[:seq_len]
    v = cache.value_pool[ids].reshape(nblk * bs, cache.num_kv_heads, cache.head_dim)[:seq_len]
    return k, v, seq_len


def paged_attention(query, cache, sequence_idx, *, mask=None, score_mod=None):
    """One sequence: gather, repeat KV heads, attend (kernels/paged.py:17-84)."""
    keys, values, _ = gather_kv(cache, sequence_idx)
    if keys.shape[0] == 0:
        return np.zeros_like(query)
    hq = query.shape[0]
    q = query[None]
    k = np.transpose(keys, (1, 0, 2))[None]
    v = np.transpose(values, (1, 0, 2))[None]
    hkv = k.shape[1]
    if hkv != hq:
        if hq % hkv != 0:
            raise ValueError(f"num_heads ({hq}) must be divisible by num_kv_heads "
                             f"({hkv}) for paged attention")
        k = np.repeat(k, hq // hkv, axis=1)
        v = np.repeat(v, hq // hkv, axis=1)
    if mask is not None:
        mask = mask[None]
    return standard_attention(q, k, v, mask=mask, score_mod=score_mod)[0]


def paged_attention_batched(query, cache):
    """``paged_attention`` for every sequence: ``query`` is ``(B, Hq, Sq, D)``."""
    return np.stack([paged_attention(query[i], cache, i) for i in range(query.shape[0])])


# ----------------------------------------------------------------------------
# cache.py: the contiguous per-layer KV cache used for decoding
# ----------------------------------------------------------------------------

@dataclass
class KVLayerCache:
    """``keys``/``values`` ``(B, Hkv, max_len, D)`` + scalar ``length`` (cache.py:15-36)."""

    keys: np.ndarray
    values: np.ndarray
    length: int

    @property
    def max_len(self):
        return int(self.keys.shape[2])


def init_kv_layer_cache(batch_size, num_kv_heads, head_dim, max_len, dtype=np.float32):
    """Zero buffers, length 0 (cache.py:39-64)."""
    z = np.zeros((batch_size, num_kv_heads, max_len, head_dim), dtype=dtype)
    return KVLayerCache(z, z.copy(), 0)


def update_kv_layer_cache(cache, keys_new, values_new, start):
    """Writes ``[start, start + chunk)`` and sets ``length = start + chunk``;
    ``ValueError`` past ``max_len`` (cache.py:67-98)."""
    end = start + keys_new.shape[2]
    if end > cache.max_len:
        raise ValueError(f"KV cache overflow: end={end} exceeds max_len={cache.max_len}")
    k, v = cache.keys.copy(), cache.values.copy()
    k[:, :, start:end] = keys_new
    v[:, :, start:end] = values_new
    return KVLayerCache(k, v, end)


def kv_cache_attention(query, cache, *, mask=None, score_mod=None):
    """``query (B, Hq, Sq, D)`` over the cache's first ``length`` positions with
    kv heads repeated -- what ``MultiHeadAttention`` computes from the
    concatenated history (attnax/attention.py:386-400, :32-39)."""
    n = int(cache.length)
    return gqa_attention(query, cache.keys[:, :, :n], cache.values[:, :, :n], mask=mask, score_mod=score_mod)


def mha_attention_core(query, key, value, *, num_heads, num_kv_heads, use_rope=False, rope_base=10000.0,
                       rope_max_positions=4096, position_ids_q=None, position_ids_kv=None, kv_cache=None,
                       attention_window=None, self_attention=True, mask=None, score_mod=None,
                       base_score_mod=None, activation_dtype=None, rope_tables=None):
    """``MultiHeadAttention.__call__`` between the projections (attnax/attention.py:340-445):
    head split and transpose, RoPE of Q and K with table rows gathered at the
    positions (``arange(seq)`` by default), the KV-cache concatenation and
    update, the KV-head repeat (:395-407), the boolean sliding-window mask with
    query positions shifted by the cached length (:417-431), and
    ``standard_attention`` with the layer's mod composed before the call's.
    ``query (B, Sq, Hq*D)``, ``key``/``value (B, Skv, Hkv*D)``; returns the
    ``(B, Sq, Hq*D)`` result (and the updated cache when one is given).

    ``activation_dtype`` is the dtype the layer runs in (default: the inputs'):
    the reference builds its RoPE tables with ``out_dtype=query.dtype``
    (attention.py:356-363), so a bf16 layer gets bf16-rounded positions and
    frequencies, and its rotated q/k are bf16 values; ``"bfloat16"`` emulates
    that on float32 inputs holding bf16 values.  ``rope_tables=(cos, sin)``
    gives the ``(rope_max_positions, head_dim // 2)`` tables directly (a bf16
    table depends on how ``pow`` rounds, which differs by one bf16 ulp between
    libraries in a few entries; the tables are checked on their own)."""
    b, sq, fq = query.shape
    act = query.dtype if activation_dtype is None else activation_dtype
    _, act_round = _rounder(act)
    d = fq // num_heads
    skv = key.shape[1]
    q = query.reshape(b, sq, num_heads, d).transpose(0, 2, 1, 3)
    k = key.reshape(b, skv, num_kv_heads, d).transpose(0, 2, 1, 3)
    v = value.reshape(b, skv, num_kv_heads, d).transpose(0, 2, 1, 3)
    if use_rope:
        pq = np.broadcast_to(np.arange(sq)[None], (b, sq)) if position_ids_q is None else position_ids_q
        pk = np.broadcast_to(np.arange(skv)[None], (b, skv)) if position_ids_kv is None else position_ids_kv
        if rope_tables is None:
            cos_t, sin_t = rope_cos_sin_table(rope_max_positions, d, rope_base, act)
        else:
            cos_t, sin_t = (np.asarray(t, dtype=np.float32) for t in rope_tables)
        pq, pk = np.asarray(pq), np.asarray(pk)
        q = act_round(apply_rope(q, cos_t[pq][:, None], sin_t[pq][:, None]))
        k = act_round(apply_rope(k, cos_t[pk][:, None], sin_t[pk][:, None]))
    new_cache = None
    if kv_cache is not None:
        past = int(kv_cache.length)
        kc = np.concatenate([kv_cache.keys[:, :, :past], k], axis=2)
        vc = np.concatenate([kv_cache.values[:, :, :past], v], axis=2)
        new_cache = update_kv_layer_cache(kv_cache, k, v, past)
        k, v = kc, vc
    k, v = repeat_kv(k, num_heads), repeat_kv(v, num_heads)
    if attention_window is not None and self_attention:
        seq_kv_eff = k.shape[2]
        if kv_cache is None:
            win = make_sliding_window_mask(sq, seq_kv_eff, window_size=attention_window, causal=True)
        else:
            past = int(kv_cache.length)
            qi = np.arange(sq) + past
            ki = np.arange(seq_kv_eff)
            win = ((ki[None, :] <= qi[:, None]) & (qi[:, None] - ki[None, :] < attention_window))[None, None]
        mask = win if mask is None else (mask & win)
    out = standard_attention(q, k, v, mask=mask, score_mod=compose_score_mods(base_score_mod, score_mod))
    out = out.transpose(0, 2, 1, 3).reshape(b, sq, fq)
    return (out, new_cache) if kv_cache is not None else out


# ----------------------------------------------------------------------------
# embeddings.py: rotary position embedding (RoPE)
# ----------------------------------------------------------------------------

def _rounder(dtype):
    """Rounding after each op in ``dtype``; ``"bfloat16"`` (which numpy lacks)
    computes in float32 and rounds every result to bf16, as JAX's bf16 ops do."""
    if isinstance(dtype, str) and dtype == "bfloat16":
        return np.float32, bf16_round
    return dtype, lambda x: np.asarray(x).astype(dtype)


def rope_inv_freq(head_dim, base, dtype=np.float32):
    """``base ** (-2i / head_dim)`` computed in ``dtype`` (embeddings.py:86-100)."""
    half = head_dim // 2
    dt, r = _rounder(dtype)
    ar = r(np.arange(0, half, dtype=dt))
    return r(1.0 / r(base ** r(ar / half)))


def rope_cos_sin_table(max_seq_len, head_dim, base, dtype=np.float32):
    """cos/sin of ``position * inv_freq`` with positions and products in
    ``dtype`` (embeddings.py:103-123): ``(max_seq_len, head_dim // 2)`` each.
    ``dtype="bfloat16"`` rounds positions, frequencies and their products to
    bf16 as the reference does for a bf16 model."""
    dt, r = _rounder(dtype)
    inv = rope_inv_freq(head_dim, base, dtype)
    freqs = r(np.outer(r(np.arange(max_seq_len, dtype=dt)), inv))
    return r(np.cos(freqs)), r(np.sin(freqs))


def rope_cos_sin_from_positions(position_ids, head_dim, base, table_len, dtype=np.float32):
    """Table rows gathered by ``position_ids (B, S)`` (embeddings.py:162-184)."""
    cos_t, sin_t = rope_cos_sin_table(table_len, head_dim, base, dtype)
    return cos_t[position_ids], sin_t[position_ids]


def apply_rope(x, cos, sin):
    """Split-half rotation ``(x1 cos - x2 sin, x1 sin + x2 cos)`` (embeddings.py:126-159)."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * cos - x2 * sin, x1 * sin + x2 * cos], axis=-1)
