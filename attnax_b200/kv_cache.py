"""Contiguous per-layer KV cache and decode over it (attnax/cache.py).

``KVLayerCache`` keeps the reference's layout: ``keys``/``values`` of shape
``(batch, num_kv_heads, max_len, head_dim)`` on the GPU and the number of
valid positions ``length``.  Like ``append_kv`` for the paged cache,
``update_kv_layer_cache`` writes the new positions into the buffers in
place and returns a new ``KVLayerCache`` that shares them (the reference
returns fresh arrays); ``length`` is a host ``int`` (the reference keeps an
int32 scalar and reads it with ``int()``, which works on both).

``kv_cache_attention`` is the attention ``MultiHeadAttention`` runs during
decoding (attnax/attention.py:386-400): every query row attends to the first
``length`` cached positions, kv heads shared by ``num_heads / num_kv_heads``
query heads.  Without masks or score mods it runs the split-K paged decode
kernel on the cache itself: the buffer is viewed as a pool of
``block_size``-token blocks holding one kv head, each (batch, kv head) is a
sequence whose block table is the identity, and the query heads of a kv
head are that sequence's rows -- no copy, K/V read once per kv head.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .paged import PagedKVCache, paged_decode_raw

_BLOCK_SIZES = (256, 128, 64, 32, 16)  # tensor-core decode units; the largest dividing max_len


@dataclass(frozen=True)
class KVLayerCache:
    """KV cache buffers of one attention layer (cache.py:15-36)."""

    keys: torch.Tensor
    values: torch.Tensor
    length: int

    @property
    def max_len(self) -> int:
        return int(self.keys.shape[2])


def init_kv_layer_cache(batch_size: int, num_kv_heads: int, head_dim: int, max_len: int,
                        dtype: torch.dtype, device="cuda") -> KVLayerCache:
    """Zero-filled buffers with ``length = 0`` (cache.py:39-64)."""
    shape = (batch_size, num_kv_heads, max_len, head_dim)
    return KVLayerCache(torch.zeros(shape, dtype=dtype, device=device),
                        torch.zeros(shape, dtype=dtype, device=device), 0)


def update_kv_layer_cache(cache: KVLayerCache, keys_new: torch.Tensor, values_new: torch.Tensor,
                          start: int) -> KVLayerCache:
    """Writes ``keys_new``/``values_new`` ``(batch, num_kv_heads, chunk, head_dim)``
    at ``[start, start + chunk)`` and returns the cache with
    ``length = start + chunk``; ``ValueError`` past ``max_len`` (cache.py:67-98)."""
    chunk = int(keys_new.shape[2])
    end = int(start) + chunk
    if end > cache.max_len:
        raise ValueError(f"KV cache overflow: end={end} exceeds max_len={cache.max_len}")
    cache.keys[:, :, start:end].copy_(keys_new)
    cache.values[:, :, start:end].copy_(values_new)
    return KVLayerCache(cache.keys, cache.values, end)


def init_decoder_kv_caches(*, num_layers: int, batch_size: int, num_kv_heads: int, head_dim: int,
                           max_len: int, dtype: torch.dtype, device="cuda") -> tuple[KVLayerCache, ...]:
    """One empty cache per layer (cache.py:101-128)."""
    return tuple(init_kv_layer_cache(batch_size, num_kv_heads, head_dim, max_len, dtype, device)
                 for _ in range(num_layers))


_tables: dict = {}


def _identity_table(nseq: int, nblocks: int, device) -> torch.Tensor:
    """Block table ``[s, i] = s * nblocks + i`` (cached per shape and device)."""
    key = (nseq, nblocks, str(device))
    t = _tables.get(key)
    if t is None:
        t = torch.arange(nseq * nblocks, dtype=torch.int32, device=device).view(nseq, nblocks)
        _tables[key] = t
    return t


def _decode_block_size(cache: KVLayerCache, query: torch.Tensor):
    k, v = cache.keys, cache.values
    if not (k.is_cuda and query.is_cuda and k.dtype in (torch.bfloat16, torch.float16)
            and v.dtype == k.dtype and k.shape[3] == 128 and k.is_contiguous() and v.is_contiguous()):
        return None
    return next((bs for bs in _BLOCK_SIZES if cache.max_len % bs == 0), None)


def kv_cache_attention(query: torch.Tensor, cache: KVLayerCache, *, mask=None, score_mod=None) -> torch.Tensor:
    """``query (batch, num_heads, seq_q, head_dim)`` against the first
    ``cache.length`` cached positions; returns the query's shape and dtype.

    bf16/f16 buffers with head_dim 128, ``max_len`` a multiple of 16 and no
    mask/score_mod take the split-K decode kernel; otherwise the flash kernel
    runs on the ``[:length]`` views (score_mod positions start at 0 on both
    axes, as when the reference's attention function sees the concatenated
    history).
    """
    if query.dim() != 4:
        raise ValueError("query must be (batch, num_heads, seq_q, head_dim)")
    b, hq, sq, d = query.shape
    _, hkv, _, dk = cache.keys.shape
    if cache.keys.shape[0] != b or dk != d:
        raise ValueError(f"query {tuple(query.shape)} does not match cache {tuple(cache.keys.shape)}")
    if hq % hkv != 0:
        raise ValueError(f"num_heads ({hq}) must be divisible by num_kv_heads ({hkv})")
    if not query.is_cuda:
        raise RuntimeError("attnax_b200 kernels need CUDA tensors; there is no CPU path")
    n = int(cache.length)
    if n == 0:
        return torch.zeros_like(query)
    bs = _decode_block_size(cache, query) if mask is None and score_mod is None else None
    if bs is not None:
        nseq, nblk = b * hkv, cache.max_len // bs
        pool = PagedKVCache(cache.keys.view(nseq * nblk, bs, 1, d), cache.values.view(nseq * nblk, bs, 1, d),
                            _identity_table(nseq, nblk, query.device),
                            torch.full((nseq,), n, dtype=torch.int32, device=query.device))
        q = query.to(cache.keys.dtype).contiguous().view(nseq, hq // hkv, sq, d)
        return paged_decode_raw(q, pool, max_context=n).view(b, hq, sq, d).to(query.dtype)
    from .flash import attention

    k, v = cache.keys[:, :, :n], cache.values[:, :, :n]
    return attention(query.to(k.dtype), k, v, mask=mask, score_mod=score_mod).to(query.dtype)
