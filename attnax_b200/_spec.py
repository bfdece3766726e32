"""Flattens composed ScoreMods and ``mask=`` into the kernel's ``attn_mask_t``.

Selections (causal, window, prefix, document, MaskMods, ``mask=``) AND
together and additive terms (ALiBi, bias) sum, so a left-to-right chain of
built-in mods (attnax/kernels/_api.py:166-196) reduces to one static spec:
a band ``lo <= q - kv <= hi``, an optional prefix-length vector, an optional
document-id vector, summed ALiBi slopes, one summed bias tensor and one
boolean mask.  Callables that are not built-in mods raise
``NotImplementedError``: there is no fallback.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _lib
from ._api import ComposedScoreMod, position_indices
from .score_mods import (AdditiveBiasMod, AlibiMod, CausalMod, DocumentMaskMod, MaskModScoreMod,
                         PrefixLMMod, SlidingWindowMod)

BAND_INF = 1 << 62

_DTYPE_CODE = {torch.float32: _lib.ATTN_F32, torch.bfloat16: _lib.ATTN_BF16, torch.float16: _lib.ATTN_F16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}; expected float32, bfloat16 or float16") from None


def flatten_mods(score_mod):
    if score_mod is None:
        return []
    if isinstance(score_mod, ComposedScoreMod):
        out = []
        for p in score_mod.parts:
            out.extend(flatten_mods(p))
        return out
    return [score_mod]


@dataclass
class MaskSpec:
    struct: _lib.AttnMask
    keep: list = field(default_factory=list)   # tensors the struct points into
    fix_masked_rows: bool = False
    has_selection: bool = False


def _expand4(t: torch.Tensor, shape):
    """Broadcast view to 4-D; returns (tensor, element strides)."""
    while t.dim() < 4:
        t = t[None]
    t = t.expand(*shape)
    return t, [int(s) for s in t.stride()]


def build_spec(score_mod, mask, *, batch, heads_q, seq_q, seq_kv, device, q_offset=0, kv_offset=0):
    """Returns the MaskSpec for one attention call."""
    m = _lib.AttnMask()
    keep = []
    lo, hi = -BAND_INF, BAND_INF
    has_band = False
    prefix = doc = slopes = bias = bmask = None
    for p in flatten_mods(score_mod):
        if isinstance(p, CausalMod):
            lo, has_band = max(lo, 0), True
        elif isinstance(p, SlidingWindowMod):
            w = p.window_size
            lo = max(lo, 0 if p.causal else -(w - 1))
            hi = min(hi, w - 1)
            has_band = True
        elif isinstance(p, AlibiMod):
            if p.num_heads != heads_q:
                raise ValueError(f"alibi_mod({p.num_heads}) used with {heads_q} query heads")
            s = p.slopes
            slopes = s if slopes is None else slopes + s
        elif isinstance(p, PrefixLMMod):
            pl = p.prefix_lengths
            prefix = pl if prefix is None else torch.minimum(prefix, pl)
        elif isinstance(p, DocumentMaskMod):
            if doc is not None and not torch.equal(doc, p.document_ids):
                raise NotImplementedError("two different document_mask_mod id tensors in one chain")
            doc = p.document_ids
        elif isinstance(p, AdditiveBiasMod):
            b = p.bias.to(device)
            bias = b if bias is None else bias + b
        elif isinstance(p, MaskModScoreMod):
            # MaskMods see global positions (attention.py:651-657), like every other mod.
            idx = position_indices(batch, heads_q, seq_q, seq_kv, device, q_offset, kv_offset)
            bm = torch.as_tensor(p.mask_mod(*idx)).expand(batch, heads_q, seq_q, seq_kv)
            bmask = bm if bmask is None else (bmask & bm)
        else:
            raise NotImplementedError(
                f"score_mod {p!r} is not a built-in ScoreMod; the B200 kernels compile only "
                "causal/sliding-window/ALiBi/prefix-LM/document/additive-bias/mask_mod mods")
    if mask is not None:
        mk = torch.as_tensor(mask, device=device).to(torch.bool)
        bmask = mk if bmask is None else (bmask & mk)

    if has_band:
        m.has_band, m.band_lo, m.band_hi = 1, lo, hi
    if prefix is not None:
        if prefix.numel() != batch:
            raise ValueError(f"prefix_lengths has {prefix.numel()} entries for batch {batch}")
        t = prefix.to(device=device, dtype=torch.int32).contiguous()
        keep.append(t)
        m.prefix_len = t.data_ptr()
    if doc is not None:
        if doc.shape[0] != batch:
            raise ValueError(f"document_ids batch {doc.shape[0]} != {batch}")
        t = doc.to(device=device, dtype=torch.int32).contiguous()
        if t.shape[1] < max(q_offset + seq_q, kv_offset + seq_kv):
            raise ValueError("document_ids shorter than the sequence")
        keep.append(t)
        m.doc_q = m.doc_kv = t.data_ptr()
        m.doc_q_bstride = m.doc_kv_bstride = t.stride(0)
    if slopes is not None:
        t = slopes.to(device=device, dtype=torch.float32).contiguous()
        keep.append(t)
        m.alibi_slopes = t.data_ptr()
    if bias is not None:
        if bias.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            bias = bias.float()
        t, st = _expand4(bias, (batch, heads_q, seq_q, seq_kv))
        keep.append(t)
        m.bias = t.data_ptr()
        m.bias_dtype = dtype_code(t.dtype)
        for i in range(4):
            m.bias_strides[i] = st[i]
    if bmask is not None:
        t, st = _expand4(bmask, (batch, heads_q, seq_q, seq_kv))
        keep.append(t)
        m.bool_mask = t.data_ptr()
        for i in range(4):
            m.mask_strides[i] = st[i]
    m.q_offset, m.kv_offset = q_offset, kv_offset

    has_sel = has_band or prefix is not None or doc is not None or bmask is not None
    diag_kept = (q_offset == kv_offset and seq_q <= seq_kv and lo <= 0 <= hi)
    fix = bmask is not None or (has_sel and not diag_kept)
    return MaskSpec(m, keep, fix, has_sel)


def band_of(score_mod):
    """(lo, hi) of the causal/window selection of a mod chain, or None."""
    lo, hi, has = -BAND_INF, BAND_INF, False
    for p in flatten_mods(score_mod):
        if isinstance(p, CausalMod):
            lo, has = max(lo, 0), True
        elif isinstance(p, SlidingWindowMod):
            lo = max(lo, 0 if p.causal else -(p.window_size - 1))
            hi = min(hi, p.window_size - 1)
            has = True
    return (lo, hi) if has else None


def may_empty_rows(score_mod, mask) -> bool:
    """Whether some query row could keep no key at all (needs the mean-of-V rule)."""
    for p in flatten_mods(score_mod):
        if isinstance(p, (MaskModScoreMod, DocumentMaskMod, PrefixLMMod)):
            return True
    band = band_of(score_mod)
    return mask is not None or (band is not None and not (band[0] <= 0 <= band[1]))
