"""Paged KV cache and paged decode (attnax/paged_cache.py, attnax/kernels/paged.py).

The cache keeps the reference's layout: pools ``(num_blocks, block_size,
num_kv_heads, head_dim)``, a ``(batch, max_blocks_per_seq)`` int32 block
table with ``-1`` for unused slots, and ``(batch,)`` sequence lengths, all
on the GPU.  The functions return new ``PagedKVCache`` objects like the
reference's functional API; ``append_kv`` writes the new tokens into the
pool tensors in place (the returned cache shares them) rather than copying
the whole pool, so slots past an older cache's ``seq_lengths`` see the
new tokens too.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from ._spec import dtype_code
from .flash import softmax_scale


@dataclass(frozen=True)
class PagedKVCache:
    """Paged KV cache storage and per-sequence block table (paged_cache.py:12-48)."""

    key_pool: torch.Tensor
    value_pool: torch.Tensor
    block_table: torch.Tensor
    seq_lengths: torch.Tensor

    @property
    def num_blocks(self) -> int:
        return int(self.key_pool.shape[0])

    @property
    def block_size(self) -> int:
        return int(self.key_pool.shape[1])

    @property
    def num_kv_heads(self) -> int:
        return int(self.key_pool.shape[2])

    @property
    def head_dim(self) -> int:
        return int(self.key_pool.shape[3])


def init_paged_kv_cache(*, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                        batch_size: int, max_blocks_per_seq: int, dtype=torch.bfloat16,
                        device="cuda") -> PagedKVCache:
    """Zero pools, ``-1`` block table, zero lengths (paged_cache.py:51-89)."""
    kp = torch.zeros(num_blocks, block_size, num_kv_heads, head_dim, dtype=dtype, device=device)
    return PagedKVCache(kp, torch.zeros_like(kp),
                        torch.full((batch_size, max_blocks_per_seq), -1, dtype=torch.int32, device=device),
                        torch.zeros(batch_size, dtype=torch.int32, device=device))


def allocate_blocks(cache: PagedKVCache, *, sequence_idx: int, num_new_tokens: int,
                    free_block_ids) -> tuple[PagedKVCache, int]:
    """Fills block-table slots from ``free_block_ids`` (paged_cache.py:92-141)."""
    bs = cache.block_size
    cur = int(cache.seq_lengths[sequence_idx])
    have = (cur + bs - 1) // bs
    need = (cur + num_new_tokens + bs - 1) // bs
    new = need - have
    free = torch.as_tensor(free_block_ids)
    if new > int(free.shape[0]):
        raise ValueError(f"free_block_ids has {int(free.shape[0])} entries but {new} are needed")
    table = cache.block_table.clone()
    if new > 0:
        table[sequence_idx, have:have + new] = free[:new].to(device=table.device, dtype=torch.int32)
    return PagedKVCache(cache.key_pool, cache.value_pool, table, cache.seq_lengths), new


def append_kv(cache: PagedKVCache, sequence_idx: int, keys_new: torch.Tensor,
              values_new: torch.Tensor) -> PagedKVCache:
    """Scatters ``(chunk, Hkv, D)`` new tokens into the pool (paged_cache.py:144-198)."""
    if keys_new.shape != values_new.shape:
        raise ValueError(f"keys_new shape {tuple(keys_new.shape)} != values_new shape "
                         f"{tuple(values_new.shape)}")
    lib = _lib.load()
    chunk = int(keys_new.shape[0])
    start = int(cache.seq_lengths[sequence_idx])
    dev = cache.key_pool.device
    kn = keys_new.to(device=dev, dtype=cache.key_pool.dtype).contiguous()
    vn = values_new.to(device=dev, dtype=cache.key_pool.dtype).contiguous()
    row = cache.block_table[sequence_idx].contiguous()
    if (start + chunk + cache.block_size - 1) // cache.block_size > row.numel():
        raise ValueError("append_kv past max_blocks_per_seq")
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    args = (dtype_code(cache.key_pool.dtype), cache.key_pool.data_ptr(), cache.value_pool.data_ptr(),
            cache.num_blocks, cache.block_size, cache.num_kv_heads, cache.head_dim, row.data_ptr(), row.numel(),
            start, chunk, kn.data_ptr(), vn.data_ptr())
    bad = torch.full((1,), 2**31 - 1, dtype=torch.int32, device=dev)
    _lib.check(lib.attn_paged_append(*args, bad.data_ptr(), stream), "attn_paged_append")
    bad_slot = int(bad.item())
    if bad_slot != 2**31 - 1:
        raise ValueError(f"block_table[{sequence_idx}, {bad_slot}] is unallocated; call "
                         "allocate_blocks before append_kv.")
    _lib.check(lib.attn_paged_append(*args, None, stream), "attn_paged_append")
    lens = cache.seq_lengths.clone()
    lens[sequence_idx] += chunk
    return PagedKVCache(cache.key_pool, cache.value_pool, cache.block_table, lens)


def gather_kv(cache: PagedKVCache, sequence_idx: int):
    """Contiguous ``(seq_len, Hkv, D)`` keys/values of one sequence (paged_cache.py:201-231)."""
    lib = _lib.load()
    seq_len = int(cache.seq_lengths[sequence_idx])
    shape = (seq_len, cache.num_kv_heads, cache.head_dim)
    k = torch.empty(shape, dtype=cache.key_pool.dtype, device=cache.key_pool.device)
    v = torch.empty_like(k)
    if seq_len:
        row = cache.block_table[sequence_idx].contiguous()
        stream = C.c_void_p(torch.cuda.current_stream(k.device).cuda_stream)
        _lib.check(lib.attn_paged_gather(dtype_code(k.dtype), cache.key_pool.data_ptr(),
                                         cache.value_pool.data_ptr(), cache.num_blocks, cache.block_size,
                                         cache.num_kv_heads, cache.head_dim, row.data_ptr(), row.numel(),
                                         seq_len, k.data_ptr(), v.data_ptr(), stream), "attn_paged_gather")
    return k, v, seq_len


def paged_decode_raw(query, cache: PagedKVCache, *, block_table=None, seq_lengths=None,
                     max_context=None, out=None, workspace=None):
    """One ``attn_paged_decode`` over every row of ``block_table``.

    ``query`` is ``(num_seqs, Hq, Sq, D)``; returns the same shape.  With
    ``max_context`` given (an upper bound of the lengths) no host sync
    happens; the bound is then the caller's promise, and a length above it
    (or past its block-table row) is processed by the documented clamping
    and reported by ``_lib.device_status()`` (``NOTICE_CONTEXT_OVERRUN`` /
    ``NOTICE_TABLE_OVERRUN``) instead of raising.
    """
    lib = _lib.load()
    bt = cache.block_table if block_table is None else block_table
    sl = cache.seq_lengths if seq_lengths is None else seq_lengths
    if query.dim() != 4:
        raise ValueError("query must be (num_seqs, num_heads, seq_q, head_dim)")
    n, hq, sq, d = query.shape
    if hq % cache.num_kv_heads != 0:
        raise ValueError(f"num_heads ({hq}) must be divisible by num_kv_heads "
                         f"({cache.num_kv_heads}) for paged attention")
    if d != cache.head_dim:
        raise ValueError(f"query head_dim {d} != cache head_dim {cache.head_dim}")
    if not query.is_cuda:
        raise RuntimeError("attnax_b200 kernels need CUDA tensors; there is no CPU path")
    if max_context is None:
        # (one host sync; the lengths are then known to fit their table rows,
        # which gather_kv in the reference needs to reshape them)
        max_context = int(sl.max()) if sl.numel() else 0
        if max_context > bt.shape[1] * cache.block_size:
            raise ValueError(f"a sequence length ({max_context}) exceeds max_blocks_per_seq * block_size "
                             f"({bt.shape[1]} * {cache.block_size})")
    q = query.to(cache.key_pool.dtype).contiguous()
    out = torch.empty_like(q) if out is None else out
    p = _lib.PagedParams()
    p.dtype = dtype_code(q.dtype)
    p.num_seqs, p.num_heads_q, p.num_heads_kv, p.head_dim, p.seq_q = n, hq, cache.num_kv_heads, d, sq
    p.num_blocks, p.block_size, p.max_blocks_per_seq = cache.num_blocks, cache.block_size, bt.shape[1]
    p.max_context = int(max_context)
    bt = bt.contiguous()
    sl = sl.contiguous()
    p.q, p.key_pool, p.value_pool = q.data_ptr(), cache.key_pool.data_ptr(), cache.value_pool.data_ptr()
    p.block_table, p.seq_lengths, p.out = bt.data_ptr(), sl.data_ptr(), out.data_ptr()
    p.softmax_scale = softmax_scale(d)
    nbytes = lib.attn_paged_decode_workspace_size(C.byref(p))
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    p.workspace, p.workspace_bytes = workspace.data_ptr(), workspace.numel()
    _lib.check(lib.attn_paged_decode(C.byref(p), C.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)),
               "attn_paged_decode")
    return out


def _fast_decode_ok(query, cache: PagedKVCache) -> bool:
    # Block sizes: multiples of 16 up to 256 (tensor-core decode, 16/32-token
    # TMA units), other sizes up to 48 (whole-page TMA ring); the rest gather.
    bs = cache.block_size
    return (cache.head_dim == 128 and cache.key_pool.dtype in (torch.bfloat16, torch.float16)
            and ((bs % 16 == 0 and bs <= 256) or bs <= 48)
            and query.dtype in (torch.bfloat16, torch.float16, torch.float32))


def paged_attention(query, cache: PagedKVCache, sequence_idx: int, *, mask=None, score_mod=None,
                    dropout_rng=None, dropout_rate: float = 0.0, deterministic: bool = True):
    """Attention of ``query (Hq, Sq, D)`` against one cached sequence (kernels/paged.py:17-84).

    bf16/f16 pools with head_dim 128 and no mods run the split-K decode
    kernel on the block table directly; other pools, masks and score mods
    gather the sequence (``gather_kv``) and run the flash kernel on it, with
    score_mod positions starting at 0 as in the reference.
    """
    if not deterministic and dropout_rate > 0.0 and dropout_rng is not None:
        raise NotImplementedError("attention-weight dropout is not implemented in the fused kernel")
    if query.dim() != 3:
        raise ValueError("query must be (num_heads, seq_q, head_dim)")
    if query.shape[0] % cache.num_kv_heads != 0:
        raise ValueError(f"num_heads ({query.shape[0]}) must be divisible by num_kv_heads "
                         f"({cache.num_kv_heads}) for paged attention")
    if mask is None and score_mod is None and _fast_decode_ok(query, cache):
        bt = cache.block_table[sequence_idx:sequence_idx + 1]
        sl = cache.seq_lengths[sequence_idx:sequence_idx + 1]
        return paged_decode_raw(query[None], cache, block_table=bt, seq_lengths=sl)[0].to(query.dtype)
    from .flash import attention

    keys, values, n = gather_kv(cache, sequence_idx)
    if n == 0:
        return torch.zeros_like(query)
    k = keys.permute(1, 0, 2)[None]
    v = values.permute(1, 0, 2)[None]
    m = None if mask is None else torch.as_tensor(mask, device=query.device)[None]
    out = attention(query[None].to(keys.dtype), k, v, mask=m, score_mod=score_mod)[0]
    return out.to(query.dtype)


def paged_attention_batched(query, cache: PagedKVCache, *, max_context=None):
    """Every sequence of the cache at once: ``query (B, Hq, Sq, D)``.

    The batched form the reference cannot express without a host sync per
    sequence (paged_cache.py:214); no host sync when ``max_context`` is given.
    """
    if _fast_decode_ok(query, cache):
        return paged_decode_raw(query, cache, max_context=max_context).to(query.dtype)
    return torch.stack([paged_attention(query[i], cache, i) for i in range(query.shape[0])])
