"""Kernel protocols and score-mod composition (attnax/kernels/_api.py).

``ScoreMod``/``MaskMod``/``AttentionFn`` keep the reference's call
signatures, with torch tensors in place of JAX arrays.
``compose_score_mods`` keeps its rules (left to right, ``None`` skipped, a
single mod returned as itself, attnax/kernels/_api.py:166-196) and returns a
:class:`ComposedScoreMod` whose parts the kernels can read.
"""

from __future__ import annotations

from typing import Optional, Protocol

import torch


class ScoreMod(Protocol):
    """``(scores, b_idx, h_idx, q_idx, kv_idx) -> scores`` (attnax/kernels/_api.py:13-42)."""

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx): ...


class MaskMod(Protocol):
    """``(b_idx, h_idx, q_idx, kv_idx) -> bool`` (attnax/kernels/_api.py:45-72)."""

    def __call__(self, b_idx, h_idx, q_idx, kv_idx): ...


class AttentionFn(Protocol):
    """``(query, key, value, *, mask, score_mod, dropout_rng, dropout_rate,
    deterministic) -> out`` on ``(batch, heads, seq, head_dim)`` tensors
    (attnax/kernels/_api.py:75-112)."""

    def __call__(self, query, key, value, *, mask=None, score_mod=None, dropout_rng=None,
                 dropout_rate: float = 0.0, deterministic: bool = True): ...


def position_indices(batch, num_heads, seq_q, seq_kv, device=None, q_offset=0, kv_offset=0):
    """Broadcast ``(b, h, q, kv)`` int32 index tensors (attnax/kernels/_api.py:115-123)."""
    i = lambda n, off=0: torch.arange(n, dtype=torch.int32, device=device) + off  # noqa: E731
    return (i(batch)[:, None, None, None], i(num_heads)[None, :, None, None],
            i(seq_q, q_offset)[None, None, :, None], i(seq_kv, kv_offset)[None, None, None, :])


class ComposedScoreMod:
    """Left-to-right composition of several ScoreMods."""

    def __init__(self, parts):
        self.parts = tuple(parts)

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        for m in self.parts:
            scores = m(scores, b_idx, h_idx, q_idx, kv_idx)
        return scores

    def __repr__(self):
        return f"compose_score_mods({', '.join(map(repr, self.parts))})"


def compose_score_mods(*score_mods: Optional[ScoreMod]) -> Optional[ScoreMod]:
    """Composes ScoreMods left to right; ``None`` arguments are skipped."""
    active = [m for m in score_mods if m is not None]
    if not active:
        return None
    if len(active) == 1:
        return active[0]
    return ComposedScoreMod(active)


def mask_mod_to_boolean_mask(mask_mod: MaskMod, *, batch: int, num_heads: int, seq_q: int,
                             seq_kv: int, device=None) -> torch.Tensor:
    """Materialises a MaskMod into a ``(batch, heads, seq_q, seq_kv)`` bool tensor."""
    out = mask_mod(*position_indices(batch, num_heads, seq_q, seq_kv, device))
    return torch.as_tensor(out).expand(batch, num_heads, seq_q, seq_kv)
