"""GQA-aware attention core of ``MultiHeadAttention`` on the sm_100a kernels.

``attention_core`` is everything ``MultiHeadAttention.__call__`` does between
its input projections and its output projection (attnax/attention.py:330-450):
head split, RoPE of Q and K (``attn_rope``, positions gathered in the kernel),
the KV-cache update and concatenation (in place: the cache buffer already
holds the concatenated history), the sliding-window selection and the
attention call.  K and V keep their ``num_kv_heads`` heads: the kernels
index the shared head of each query head instead of the ``jnp.repeat`` of
attention.py:32-39 / :395-407, so the repeated copies (Hq/Hkv x the K/V
bytes) are never materialised.  The projections are the model's weights and
stay with the caller.
"""

from __future__ import annotations

import torch

from ._api import compose_score_mods
from .flash import flash_attention
from .kv_cache import KVLayerCache, update_kv_layer_cache
from .rope import apply_rope_table, rope_cos_sin_table
from .score_mods import sliding_window_mod


def _split_heads(x: torch.Tensor, heads: int) -> torch.Tensor:
    b, s, f = x.shape
    return x.view(b, s, heads, f // heads).transpose(1, 2)


def attention_core(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *, num_heads: int,
                   num_kv_heads: int, use_rope: bool = False, rope_base: float = 10000.0,
                   rope_max_positions: int = 4096, position_ids_q=None, position_ids_kv=None,
                   kv_cache: KVLayerCache | None = None, attention_window: int | None = None,
                   self_attention: bool = True, mask=None, score_mod=None, base_score_mod=None,
                   attention_fn=flash_attention, dropout_rate: float = 0.0, deterministic: bool = True):
    """``query (B, Sq, Hq*D)``, ``key``/``value (B, Skv, Hkv*D)`` -- the projected
    inputs -- to the pre-output-projection result ``(B, Sq, Hq*D)``; with
    ``kv_cache`` returns ``(result, updated_cache)`` like the reference.

    ``self_attention=False`` is the reference's ``context`` (cross-attention)
    branch: no window and no cache.  ``base_score_mod`` is the mod the layer
    was built with, composed before the per-call ``score_mod``
    (attention.py:436).  ``attention_fn`` must accept K/V with fewer heads
    than Q (every function of this package does).
    """
    if kv_cache is not None and not self_attention:
        raise ValueError("kv_cache is only supported for self-attention (context must be None).")
    if num_heads % num_kv_heads:
        raise ValueError(f"num_heads ({num_heads}) must be divisible by num_kv_heads ({num_kv_heads})")
    q = _split_heads(query, num_heads)
    k = _split_heads(key, num_kv_heads)
    v = _split_heads(value, num_kv_heads).contiguous()
    b, _, seq_q, head_dim = q.shape
    if use_rope:
        cos_t, sin_t = rope_cos_sin_table(rope_max_positions, head_dim, rope_base, q.dtype, q.device)
        q = apply_rope_table(q, cos_t, sin_t, position_ids_q)
        k = apply_rope_table(k, cos_t, sin_t, position_ids_kv)
    else:
        q, k = q.contiguous(), k.contiguous()

    new_cache = None
    past = 0
    if kv_cache is not None:
        past = int(kv_cache.length)
        new_cache = update_kv_layer_cache(kv_cache, k, v, past)
        k = new_cache.keys[:, :, :new_cache.length]
        v = new_cache.values[:, :, :new_cache.length]

    mods = compose_score_mods(base_score_mod, score_mod)
    if attention_window is not None and self_attention:
        if past == 0:
            # the reference's boolean window mask (attention.py:417-431) is this band
            mods = compose_score_mods(sliding_window_mod(attention_window), mods)
        else:
            # query positions shifted by the cached length, as the reference does
            qi = torch.arange(seq_q, device=q.device)[:, None] + past
            ki = torch.arange(k.shape[2], device=q.device)[None, :]
            win = ((ki <= qi) & (qi - ki < attention_window))[None, None]
            mask = win if mask is None else (torch.as_tensor(mask, device=q.device) & win)

    out = attention_fn(q, k, v, mask=mask, score_mod=mods, dropout_rng=None, dropout_rate=dropout_rate,
                       deterministic=deterministic)
    out = out.transpose(1, 2).reshape(b, seq_q, num_heads * head_dim)
    return (out, new_cache) if kv_cache is not None else out
