"""attnax_b200 — attnax's attention hot path, rebuilt for NVIDIA B200 (sm_100a).

Drop-in ``AttentionFn``s with the reference's names and signatures, backed by
hand-written CUDA in ``libattnb200.so`` (C ABI: ``include/attnb200.h``):

* ``flash_attention`` / ``pallas_flash_attention`` / ``memory_efficient_attention``
  / ``standard_attention`` — fused forward + backward with GQA/MQA and the
  built-in ScoreMods compiled into the kernel;
* ``paged_attention`` / ``paged_attention_batched`` over ``PagedKVCache``;
* ``kv_cache_attention`` over the contiguous per-layer ``KVLayerCache``;
* ``apply_rope`` (+ the reference's cos/sin table builders) for Q/K rotation;
* ``ring_attention`` — sequence parallel over NCCL.
"""

from . import score_mods
from ._api import AttentionFn, MaskMod, ScoreMod, compose_score_mods, mask_mod_to_boolean_mask
from .flash import (flash_attention, memory_efficient_attention, pallas_flash_attention,
                    standard_attention)
from .masking import (combine_masks, make_causal_mask, make_document_mask, make_padding_mask,
                      make_sliding_window_mask)
from .paged import (PagedKVCache, allocate_blocks, append_kv, gather_kv, init_paged_kv_cache,
                    paged_attention, paged_attention_batched)
from .kv_cache import (KVLayerCache, init_decoder_kv_caches, init_kv_layer_cache, kv_cache_attention,
                       update_kv_layer_cache)
from .ring import ring_attention, ring_attention_reference
from .rope import (apply_rope, apply_rope_table, rope_cos_sin_from_positions, rope_cos_sin_table,
                   rope_inv_freq)
from .score_mods import (additive_bias_mod, alibi_mod, alibi_slopes, causal_mod, document_mask_mod,
                         mask_mod_to_score_mod, prefix_lm_mod, sliding_window_mod)

__all__ = [
    "AttentionFn", "MaskMod", "ScoreMod", "PagedKVCache", "KVLayerCache", "init_kv_layer_cache",
    "update_kv_layer_cache", "init_decoder_kv_caches", "kv_cache_attention", "apply_rope", "apply_rope_table",
    "rope_cos_sin_from_positions", "rope_cos_sin_table", "rope_inv_freq", "additive_bias_mod", "alibi_mod",
    "alibi_slopes", "allocate_blocks", "append_kv", "causal_mod", "combine_masks",
    "compose_score_mods", "document_mask_mod", "flash_attention", "gather_kv",
    "init_paged_kv_cache", "make_causal_mask", "make_document_mask", "make_padding_mask",
    "make_sliding_window_mask", "mask_mod_to_boolean_mask", "mask_mod_to_score_mod",
    "memory_efficient_attention", "paged_attention", "paged_attention_batched",
    "pallas_flash_attention", "prefix_lm_mod", "ring_attention", "ring_attention_reference",
    "score_mods", "sliding_window_mod", "standard_attention",
]
