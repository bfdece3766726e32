"""Built-in ScoreMods as tagged callables (attnax/kernels/score_mods.py).

Each constructor returns an object that is still a ScoreMod — callable as
``mod(scores, b_idx, h_idx, q_idx, kv_idx)`` on torch tensors with the
reference's semantics — and also carries its parameters, so the kernels can
compile it into a mask/bias epilogue instead of materialising scores.
Dropped scores are ``finfo(scores.dtype).min``, as in the reference.
"""

from __future__ import annotations

import math

import torch

from ._api import MaskMod, ScoreMod, compose_score_mods  # noqa: F401


def _neg(scores):
    return torch.finfo(scores.dtype).min


def alibi_slopes(num_heads: int) -> torch.Tensor:
    """Per-head ALiBi slopes, float32 ``(num_heads,)`` (score_mods.py:14-45)."""

    def power_of_two(n):
        start = 2.0 ** (-(2.0 ** -(math.log2(n) - 3)))
        return [start * (start ** i) for i in range(n)]

    if (num_heads & (num_heads - 1)) == 0:
        return torch.tensor(power_of_two(num_heads), dtype=torch.float32)
    closest = 2 ** math.floor(math.log2(num_heads))
    base = power_of_two(closest)
    extra = power_of_two(2 * closest)[0::2][: num_heads - closest]
    return torch.tensor(base + extra, dtype=torch.float32)


class TaggedScoreMod:
    """Base class of the built-in mods the kernels understand."""

    kind = "tagged"

    def _device_tensor(self, name, t, device):
        cache = self.__dict__.setdefault("_dev_cache", {})
        key = (name, str(device))
        if key not in cache:
            cache[key] = t.to(device).contiguous()
        return cache[key]


class CausalMod(TaggedScoreMod):
    """Keep ``kv_idx <= q_idx`` (score_mods.py:84-104)."""

    kind = "causal"

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        return torch.where(kv_idx <= q_idx, scores, _neg(scores))

    def __repr__(self):
        return "causal_mod()"


class SlidingWindowMod(TaggedScoreMod):
    """Window of ``window_size`` keys (score_mods.py:107-145)."""

    kind = "window"

    def __init__(self, window_size: int, causal: bool):
        self.window_size = int(window_size)
        self.causal = bool(causal)

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        if self.causal:
            keep = (kv_idx <= q_idx) & (q_idx - kv_idx < self.window_size)
        else:
            keep = (q_idx - kv_idx).abs() < self.window_size
        return torch.where(keep, scores, _neg(scores))

    def __repr__(self):
        return f"sliding_window_mod({self.window_size}, causal={self.causal})"


class AlibiMod(TaggedScoreMod):
    """``scores - slope[h] * |q - kv|`` (score_mods.py:48-81)."""

    kind = "alibi"

    def __init__(self, num_heads: int):
        self.num_heads = int(num_heads)
        self.slopes = alibi_slopes(num_heads)

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        dt = scores.dtype
        dist = (q_idx.to(dt) - kv_idx.to(dt)).abs()
        return scores - self.slopes.to(scores.device, dt)[None, :, None, None] * dist

    def __repr__(self):
        return f"alibi_mod({self.num_heads})"


class PrefixLMMod(TaggedScoreMod):
    """Bidirectional below ``prefix_lengths[b]``, causal after (score_mods.py:148-178)."""

    kind = "prefix"

    def __init__(self, prefix_lengths):
        self.prefix_lengths = torch.as_tensor(prefix_lengths).to(torch.int32).reshape(-1)

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        pref = self.prefix_lengths.to(scores.device)[b_idx.reshape(-1).long()][:, None, None, None]
        keep = (kv_idx < pref) | (kv_idx <= q_idx)
        return torch.where(keep, scores, _neg(scores))

    def __repr__(self):
        return "prefix_lm_mod(...)"


class DocumentMaskMod(TaggedScoreMod):
    """Same-document mask for packed sequences (score_mods.py:181-213)."""

    kind = "document"

    def __init__(self, document_ids):
        self.document_ids = torch.as_tensor(document_ids).to(torch.int32)
        if self.document_ids.dim() != 2:
            raise ValueError("document_ids must have shape (batch, seq_len)")

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        ids = self.document_ids.to(scores.device)
        qi = ids[:, q_idx[0, 0, :, 0].long()]
        ki = ids[:, kv_idx[0, 0, 0, :].long()]
        keep = (qi[:, :, None] == ki[:, None, :])[:, None]
        return torch.where(keep, scores, _neg(scores))

    def __repr__(self):
        return "document_mask_mod(...)"


class AdditiveBiasMod(TaggedScoreMod):
    """``scores + bias`` with ``bias`` broadcastable to (B, H, Sq, Skv) (score_mods.py:216-237)."""

    kind = "bias"

    def __init__(self, bias):
        self.bias = torch.as_tensor(bias)

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        return scores + self.bias.to(scores.device, scores.dtype)

    def __repr__(self):
        return f"additive_bias_mod(shape={tuple(self.bias.shape)})"


class MaskModScoreMod(TaggedScoreMod):
    """``where(mask_mod(...), scores, finfo.min)`` (score_mods.py:240-264)."""

    kind = "mask_mod"

    def __init__(self, mask_mod):
        self.mask_mod = mask_mod

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        keep = self.mask_mod(b_idx, h_idx, q_idx, kv_idx)
        return torch.where(torch.as_tensor(keep, device=scores.device), scores, _neg(scores))

    def __repr__(self):
        return f"mask_mod_to_score_mod({self.mask_mod!r})"


def causal_mod() -> ScoreMod:
    return CausalMod()


def sliding_window_mod(window_size: int, *, causal: bool = True) -> ScoreMod:
    if window_size <= 0:
        raise ValueError(f"window_size must be positive, got {window_size}")
    return SlidingWindowMod(window_size, causal)


def alibi_mod(num_heads: int) -> ScoreMod:
    return AlibiMod(num_heads)


def prefix_lm_mod(prefix_lengths) -> ScoreMod:
    return PrefixLMMod(prefix_lengths)


def document_mask_mod(document_ids) -> ScoreMod:
    return DocumentMaskMod(document_ids)


def additive_bias_mod(bias) -> ScoreMod:
    return AdditiveBiasMod(bias)


def mask_mod_to_score_mod(mask_mod: MaskMod) -> ScoreMod:
    return MaskModScoreMod(mask_mod)
