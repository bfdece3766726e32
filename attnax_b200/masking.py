"""Boolean attention masks (attnax/masking.py), as torch tensors."""

from __future__ import annotations

import torch


def make_padding_mask(input_ids, pad_token_id: int = 0):
    """``(B, 1, 1, S)``, True for non-padding (masking.py:10-24)."""
    return (torch.as_tensor(input_ids) != pad_token_id)[:, None, None, :]


def make_causal_mask(seq_len: int, device=None):
    """``(1, 1, S, S)`` lower triangle (masking.py:27-38)."""
    return torch.tril(torch.ones(seq_len, seq_len, dtype=torch.bool, device=device))[None, None]


def make_sliding_window_mask(seq_q: int, seq_kv=None, *, window_size: int, causal: bool = True,
                             device=None):
    """``(1, 1, Sq, Skv)`` window mask (masking.py:41-72)."""
    if window_size <= 0:
        raise ValueError(f"window_size must be positive, got {window_size}")
    if seq_kv is None:
        seq_kv = seq_q
    q = torch.arange(seq_q, device=device)[:, None]
    kv = torch.arange(seq_kv, device=device)[None, :]
    if causal:
        m = (kv <= q) & (q - kv < window_size)
    else:
        m = (q - kv).abs() < window_size
    return m[None, None]


def make_document_mask(document_ids):
    """``(B, 1, S, S)`` same-document mask (masking.py:75-89)."""
    ids = torch.as_tensor(document_ids)
    return (ids[:, :, None] == ids[:, None, :])[:, None]


def combine_masks(*masks):
    """Logical AND; ``None`` skipped (masking.py:92-109)."""
    out = None
    for m in masks:
        if m is None:
            continue
        out = m if out is None else (out & m)
    return out
