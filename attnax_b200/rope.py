"""Rotary position embedding (attnax/embeddings.py:86-184).

The cos/sin tables are built exactly as the reference builds them: positions,
inverse frequencies and their products in the requested dtype (so bf16 and
f16 tables carry the reference's rounding).  ``apply_rope`` runs the
split-half rotation in ``attn_rope`` (fp32 math, one pass over the tensor);
the cos/sin it is given are read as a table indexed by position, which covers
the shapes ``MultiHeadAttention`` passes (``(B or 1, 1, S, half)``,
attnax/attention.py:340-381) without materialising a broadcast.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._spec import dtype_code


def rope_inv_freq(head_dim: int, base: float, dtype: torch.dtype, device="cuda") -> torch.Tensor:
    """``base ** (-2i / head_dim)`` for ``i < head_dim // 2``, in ``dtype`` (embeddings.py:86-100)."""
    half = head_dim // 2
    return 1.0 / (base ** (torch.arange(0, half, dtype=dtype, device=device) / half))


def rope_cos_sin_table(max_seq_len: int, head_dim: int, base: float, dtype: torch.dtype, device="cuda"):
    """``(cos, sin)`` of shape ``(max_seq_len, head_dim // 2)`` (embeddings.py:103-123)."""
    inv = rope_inv_freq(head_dim, base, dtype, device)
    freqs = torch.outer(torch.arange(max_seq_len, dtype=dtype, device=device), inv)
    return torch.cos(freqs).to(dtype), torch.sin(freqs).to(dtype)


def rope_cos_sin_from_positions(position_ids: torch.Tensor, head_dim: int, base: float, table_len: int,
                                out_dtype: torch.dtype):
    """Table rows at ``position_ids (B, S)``: ``(cos, sin)`` each ``(B, S, head_dim // 2)``
    (embeddings.py:162-184)."""
    cos_t, sin_t = rope_cos_sin_table(table_len, head_dim, base, out_dtype, position_ids.device)
    idx = position_ids.long()
    return cos_t[idx], sin_t[idx]


_rows: dict = {}


def _row_positions(b: int, s: int, device) -> torch.Tensor:
    key = (b, s, str(device))
    t = _rows.get(key)
    if t is None:
        t = torch.arange(b * s, dtype=torch.int32, device=device).view(b, s)
        _rows[key] = t
    return t


def _as_table(t: torch.Tensor, batch: int, seq: int, half: int, dtype: torch.dtype) -> torch.Tensor:
    if t.dim() == 4:
        if t.shape[1] != 1:
            raise ValueError("cos/sin must broadcast over heads (shape (B or 1, 1, S, head_dim // 2))")
        t = t[:, 0]
    if t.dim() == 2:
        t = t[None]
    if t.dim() != 3 or t.shape[0] not in (1, batch) or tuple(t.shape[1:]) != (seq, half):
        raise ValueError(f"cos/sin of shape {tuple(t.shape)} do not match (B or 1, [1,] {seq}, {half})")
    return t.to(dtype).reshape(-1, half).contiguous()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *, out=None) -> torch.Tensor:
    """Split-half RoPE of ``x (batch, heads, seq, head_dim)`` (embeddings.py:126-159):
    ``(x1 cos - x2 sin, x1 sin + x2 cos)``.  ``cos``/``sin``: ``(seq, half)``,
    ``(B or 1, seq, half)`` or ``(B or 1, 1, seq, half)``.  ``out`` may be ``x``."""
    if x.dim() != 4:
        raise ValueError("x must be (batch, heads, seq, head_dim)")
    if not x.is_cuda:
        raise RuntimeError("attnax_b200 kernels need CUDA tensors; there is no CPU path")
    B, H, S, D = x.shape
    if D % 2:
        raise ValueError("head_dim must be even for RoPE")
    half = D // 2
    ct, st = _as_table(cos, B, S, half, x.dtype), _as_table(sin, B, S, half, x.dtype)
    per_batch = ct.shape[0] == B * S and B > 1
    xx = x if x.stride(-1) == 1 else x.contiguous()
    out = torch.empty_like(xx) if out is None else out
    p = _lib.RopeParams()
    p.dtype = dtype_code(x.dtype)
    p.batch, p.heads, p.seq, p.head_dim = B, H, S, D
    for i in range(3):
        p.x_strides[i], p.out_strides[i] = xx.stride(i), out.stride(i)
    p.x, p.out, p.cos, p.sin = xx.data_ptr(), out.data_ptr(), ct.data_ptr(), st.data_ptr()
    p.table_len = ct.shape[0]
    pos = _row_positions(B, S, x.device) if per_batch else None
    p.positions = pos.data_ptr() if pos is not None else None
    _lib.check(_lib.load().attn_rope(C.byref(p), C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)),
               "attn_rope")
    return out


def apply_rope_table(x: torch.Tensor, cos_table: torch.Tensor, sin_table: torch.Tensor,
                     position_ids: torch.Tensor | None = None, *, out=None) -> torch.Tensor:
    """RoPE with the gather fused: rows of ``(table_len, half)`` tables at
    ``position_ids (batch, seq)`` (default: positions ``0..seq-1``), without the
    ``(B, S, half)`` gathered copies ``rope_cos_sin_from_positions`` builds."""
    if x.dim() != 4 or not x.is_cuda:
        raise ValueError("x must be a CUDA tensor (batch, heads, seq, head_dim)")
    B, H, S, D = x.shape
    half = D // 2
    if D % 2 or cos_table.shape[-1] != half or sin_table.shape != cos_table.shape:
        raise ValueError("tables must be (table_len, head_dim // 2) for an even head_dim")
    ct, st = cos_table.to(x.dtype).contiguous(), sin_table.to(x.dtype).contiguous()
    xx = x if x.stride(-1) == 1 else x.contiguous()
    out = torch.empty_like(xx) if out is None else out
    pos = None
    if position_ids is not None:
        pos = position_ids.to(device=x.device, dtype=torch.int32).expand(B, S).contiguous()
    p = _lib.RopeParams()
    p.dtype = dtype_code(x.dtype)
    p.batch, p.heads, p.seq, p.head_dim = B, H, S, D
    for i in range(3):
        p.x_strides[i], p.out_strides[i] = xx.stride(i), out.stride(i)
    p.x, p.out, p.cos, p.sin = xx.data_ptr(), out.data_ptr(), ct.data_ptr(), st.data_ptr()
    p.table_len = ct.shape[0]
    p.positions = pos.data_ptr() if pos is not None else None
    _lib.check(_lib.load().attn_rope(C.byref(p), C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)),
               "attn_rope")
    return out
