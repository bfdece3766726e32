"""Drop-in flash-attention ``AttentionFn``s backed by the sm_100a kernels.

``flash_attention``, ``pallas_flash_attention``, ``memory_efficient_attention``
and ``standard_attention`` keep the reference's signatures
(attnax/kernels/attention.py:17-283, attnax/kernels/pallas.py:27-115) and all
compute the same function the reference's ``standard_attention`` defines;
their block-size arguments are accepted for signature compatibility (the
kernel tiles at 128).  Forward and backward run in ``libattnb200.so``
through a ``torch.autograd.Function`` (the reference differentiates with JAX
autodiff; pallas.py:45-47).  K/V may have fewer heads than Q (GQA/MQA): the
kernels index the shared KV head instead of repeating it.
"""

from __future__ import annotations

import ctypes as C
import math
from typing import Optional

import torch

from . import _lib
from ._spec import build_spec, dtype_code


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _strides3(t: torch.Tensor):
    s = t.stride()
    return (C.c_int64 * 3)(s[0], s[1], s[2])


def _prep(t: torch.Tensor) -> torch.Tensor:
    if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:3]) or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def check_qkv(query, key, value):
    """Validates shapes like the reference and returns (B, Hq, Hkv, Sq, Skv, D)."""
    for name, t in (("query", query), ("key", key), ("value", value)):
        if not isinstance(t, torch.Tensor) or t.dim() != 4:
            raise ValueError(f"{name} must be a 4-D (batch, heads, seq, head_dim) tensor")
    if not (query.is_cuda and key.is_cuda and value.is_cuda):
        raise RuntimeError("attnax_b200 kernels need CUDA tensors; there is no CPU path")
    if key.shape != value.shape:
        raise ValueError(f"key shape {tuple(key.shape)} != value shape {tuple(value.shape)}")
    B, Hq, Sq, D = query.shape
    Bk, Hkv, Skv, Dk = key.shape
    if Bk != B or Dk != D:
        raise ValueError(f"query {tuple(query.shape)} and key {tuple(key.shape)} disagree")
    if Hq % Hkv != 0:
        raise ValueError(f"num_heads ({Hq}) must be divisible by num_kv_heads ({Hkv})")
    if not (query.dtype == key.dtype == value.dtype):
        raise ValueError("query, key and value must share a dtype")
    return B, Hq, Hkv, Sq, Skv, D


def softmax_scale(head_dim: int) -> float:
    """``rsqrt(head_dim)`` rounded to float32, as the reference computes it."""
    return float(torch.tensor(1.0 / math.sqrt(head_dim), dtype=torch.float32))


def fwd_raw(q, k, v, spec, *, want_lse=True, out=None, lse=None):
    """One ``attn_fwd`` call; returns ``(out, lse)``."""
    lib = _lib.load()
    B, Hq, Hkv, Sq, Skv, D = check_qkv(q, k, v)
    out = torch.empty_like(q, memory_format=torch.contiguous_format) if out is None else out
    if lse is None and want_lse:
        lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=q.device)
    p = _lib.FwdParams()
    p.dtype = dtype_code(q.dtype)
    p.batch, p.num_heads_q, p.num_heads_kv, p.seq_q, p.seq_kv, p.head_dim = B, Hq, Hkv, Sq, Skv, D
    p.q, p.k, p.v, p.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.q_strides, p.k_strides, p.v_strides, p.o_strides = (_strides3(q), _strides3(k), _strides3(v),
                                                          _strides3(out))
    p.lse = lse.data_ptr() if lse is not None else None
    p.softmax_scale = softmax_scale(D)
    p.fix_masked_rows = int(spec.fix_masked_rows)
    p.mask = spec.struct
    nbytes = lib.attn_fwd_workspace_size(C.byref(p))
    ws = None
    if nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        p.workspace, p.workspace_bytes = ws.data_ptr(), nbytes
    _lib.check(lib.attn_fwd(C.byref(p), C.c_void_p(_stream_ptr(q.device))), "attn_fwd")
    return out, lse


def bwd_raw(q, k, v, out, lse, dout, spec):
    lib = _lib.load()
    B, Hq, Hkv, Sq, Skv, D = check_qkv(q, k, v)
    dq = torch.empty_like(q, memory_format=torch.contiguous_format)
    dk = torch.empty_like(k, memory_format=torch.contiguous_format)
    dv = torch.empty_like(v, memory_format=torch.contiguous_format)
    p = _lib.BwdParams()
    p.dtype = dtype_code(q.dtype)
    p.batch, p.num_heads_q, p.num_heads_kv, p.seq_q, p.seq_kv, p.head_dim = B, Hq, Hkv, Sq, Skv, D
    p.q, p.k, p.v, p.out, p.d_out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr()
    p.lse = lse.data_ptr()
    p.dq, p.dk, p.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    p.q_strides, p.k_strides, p.v_strides = _strides3(q), _strides3(k), _strides3(v)
    p.o_strides, p.do_strides = _strides3(out), _strides3(dout)
    p.dq_strides, p.dk_strides, p.dv_strides = _strides3(dq), _strides3(dk), _strides3(dv)
    p.softmax_scale = softmax_scale(D)
    p.fix_masked_rows = int(spec.fix_masked_rows)
    p.mask = spec.struct
    nbytes = lib.attn_bwd_workspace_size(C.byref(p))
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.attn_bwd(C.byref(p), C.c_void_p(_stream_ptr(q.device))), "attn_bwd")
    return dq, dk, dv


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, spec):
        out, lse = fwd_raw(q, k, v, spec)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.spec = spec
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = bwd_raw(q, k, v, out, lse, _prep(dout), ctx.spec)
        return dq, dk, dv, None


def _output_dropout(out, dropout_rng, dropout_rate, deterministic):
    """Output dropout of memory_efficient_attention (attnax/kernels/attention.py:201-204)."""
    if deterministic or dropout_rate <= 0.0 or dropout_rng is None:
        return out
    gen = dropout_rng
    if not isinstance(gen, torch.Generator):
        gen = torch.Generator(device=out.device)
        gen.manual_seed(int(dropout_rng))
    keep_prob = 1.0 - dropout_rate
    keep = torch.rand(out.shape, generator=gen, device=out.device) < keep_prob
    return torch.where(keep, out / keep_prob, torch.zeros((), dtype=out.dtype, device=out.device))


def attention(query, key, value, *, mask=None, score_mod=None):
    """The kernel call shared by every AttentionFn in this module."""
    B, Hq, Hkv, Sq, Skv, D = check_qkv(query, key, value)
    spec = build_spec(score_mod, mask, batch=B, heads_q=Hq, seq_q=Sq, seq_kv=Skv, device=query.device)
    q, k, v = _prep(query), _prep(key), _prep(value)
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return _FlashAttnFn.apply(q, k, v, spec)
    out, _ = fwd_raw(q, k, v, spec, want_lse=False)
    return out


def flash_attention(query, key, value, *, mask=None, score_mod=None, dropout_rng=None,
                    dropout_rate: float = 0.0, deterministic: bool = True, block_size: int = 512):
    """Flash attention on sm_100a (replaces attnax/kernels/attention.py:209-283)."""
    out = attention(query, key, value, mask=mask, score_mod=score_mod)
    return _output_dropout(out, dropout_rng, dropout_rate, deterministic)


def pallas_flash_attention(query, key, value, *, mask=None, score_mod=None, dropout_rng=None,
                           dropout_rate: float = 0.0, deterministic: bool = True,
                           block_q: int = 128, block_kv: int = 128, force_fallback: bool = False):
    """Same kernel under the Pallas entry point's name (attnax/kernels/pallas.py:27-115)."""
    out = attention(query, key, value, mask=mask, score_mod=score_mod)
    return _output_dropout(out, dropout_rng, dropout_rate, deterministic)


def memory_efficient_attention(query, key, value, *, mask=None, score_mod=None, dropout_rng=None,
                               dropout_rate: float = 0.0, deterministic: bool = True,
                               block_size: int = 512):
    """Same kernel under the blockwise entry point's name (attention.py:74-206)."""
    out = attention(query, key, value, mask=mask, score_mod=score_mod)
    return _output_dropout(out, dropout_rng, dropout_rate, deterministic)


def standard_attention(query, key, value, *, mask=None, score_mod=None, dropout_rng=None,
                       dropout_rate: float = 0.0, deterministic: bool = True):
    """Same function as attention.py:17-71; weight dropout is not fused."""
    if not deterministic and dropout_rate > 0.0 and dropout_rng is not None:
        raise NotImplementedError("attention-weight dropout is not implemented in the fused kernel")
    return attention(query, key, value, mask=mask, score_mod=score_mod)
