"""The C-ABI ring forward (``attn_ring_fwd``) driven from torch.

``attn_ring_fwd`` runs the whole ring of ``ring_attention``
(attnax/kernels/attention.py:540-691) -- zig-zag re-deal, K/V rotation over
NCCL, per-hop attention with the log-sum-exp merge fused into the kernel --
from C++.  Its NCCL communicator is made once per process group: rank 0
asks the library for a unique id and the group's own broadcast hands it to
every rank.  The chains it takes are the ones whose masks depend only on
positions: causal and sliding windows and ALiBi (no ``mask=``, bias,
prefix or document masks; those run the host schedule in ``_ring_impl``).
"""

from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib
from ._spec import build_spec, dtype_code, flatten_mods
from .score_mods import AlibiMod, CausalMod, SlidingWindowMod

_COMMS = {}
_STREAMS = {}


def eligible(query, key, value, score_mod, mask) -> bool:
    if mask is not None or query.dtype not in (torch.bfloat16, torch.float16):
        return False
    if query.shape[-1] not in (64, 128) or not (query.dtype == key.dtype == value.dtype):
        return False
    mods = flatten_mods(score_mod)
    if not all(isinstance(p, (CausalMod, SlidingWindowMod, AlibiMod)) for p in mods):
        return False
    return all(p.num_heads == query.shape[1] for p in mods if isinstance(p, AlibiMod))


def comm_for(group, device):
    """The library's NCCL communicator for ``group`` on ``device`` (made once)."""
    key = (id(group), device.index)
    c = _COMMS.get(key)
    if c is not None:
        return c
    lib = _lib.load()
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    buf = torch.zeros(_lib.COMM_ID_BYTES, dtype=torch.uint8, device=device)
    if rank == 0:
        raw = (C.c_char * _lib.COMM_ID_BYTES)()
        _lib.check(lib.attn_comm_unique_id(raw, _lib.COMM_ID_BYTES), "attn_comm_unique_id")
        buf.copy_(torch.frombuffer(bytearray(raw.raw), dtype=torch.uint8))
    src = dist.get_global_rank(group, 0) if group is not None else 0
    dist.broadcast(buf, src=src, group=group)
    ident = bytes(buf.cpu().numpy().tobytes())
    c = C.c_void_p()
    with torch.cuda.device(device):
        _lib.check(lib.attn_comm_init(C.byref(c), world, rank, ident, _lib.COMM_ID_BYTES), "attn_comm_init")
    _COMMS[key] = c
    return c


def release_comms():
    """Destroys the communicators made by ``comm_for`` (every rank, before exit)."""
    lib = _lib.load()
    for key, c in list(_COMMS.items()):
        lib.attn_comm_destroy(c)
        del _COMMS[key]


def _comm_stream(device):
    """The stream of the ring's NCCL transfers, at the highest priority: the
    attention kernel of a hop fills every SM, and the block scheduler hands
    SMs that free up to the higher-priority stream's CTAs first, so the next
    hop's K/V transfer starts during this hop instead of after its last wave."""
    s = _STREAMS.get(device.index)
    if s is None:
        lo, hi = torch.cuda.Stream.priority_range() if hasattr(torch.cuda.Stream, "priority_range") else (0, -1)
        s = _STREAMS[device.index] = torch.cuda.Stream(device=device, priority=min(lo, hi))
    return s


def ring_fwd(query, key, value, score_mod, group, zigzag=None):
    """(out, lse) of the ring over ``group`` for this rank's contiguous shards."""
    from ._spec import band_of
    from .flash import softmax_scale

    lib = _lib.load()
    q, k, v = (t.contiguous() for t in (query, key, value))
    B, Hq, S, D = q.shape
    world = dist.get_world_size(group)
    band = band_of(score_mod)
    if zigzag is None:
        zigzag = band is not None and band[0] >= 0 and world > 1 and S % 2 == 0
    spec = build_spec(score_mod, None, batch=B, heads_q=Hq, seq_q=S, seq_kv=S, device=q.device)
    out = torch.empty_like(q)
    lse = torch.empty(B, Hq, S, dtype=torch.float32, device=q.device)
    p = _lib.RingParams()
    p.dtype = dtype_code(q.dtype)
    p.batch, p.num_heads_q, p.num_heads_kv, p.seq_local, p.head_dim = B, Hq, k.shape[1], S, D
    p.q, p.k, p.v, p.out, p.lse = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr()
    p.softmax_scale = softmax_scale(D)
    if band is not None:
        p.has_band, p.band_lo, p.band_hi = 1, band[0], band[1]
    p.alibi_slopes = spec.struct.alibi_slopes
    p.zigzag = int(bool(zigzag))
    nbytes = lib.attn_ring_fwd_workspace_size(C.byref(p), world)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    cs = torch.cuda.current_stream(q.device)
    ms = _comm_stream(q.device)
    comm = comm_for(group, q.device)
    _lib.check(lib.attn_ring_fwd(C.byref(p), comm, C.c_void_p(cs.cuda_stream), C.c_void_p(ms.cuda_stream)),
               "attn_ring_fwd")
    # the comm stream reads the inputs and the workspace; keep their memory
    # from being handed out again before that work is done
    for t in (q, k, v, ws, out, lse):
        t.record_stream(ms)
    del spec
    return out, lse


def ring_bwd(query, key, value, out, lse, dout, score_mod, group, zigzag):
    """(dq, dk, dv) of ``ring_fwd`` through ``attn_ring_bwd`` (public layout in and out)."""
    from ._spec import band_of
    from .flash import softmax_scale

    lib = _lib.load()
    q, k, v, o, do = (t.contiguous() for t in (query, key, value, out, dout.to(query.dtype)))
    lse = lse.contiguous()
    B, Hq, S, D = q.shape
    world = dist.get_world_size(group)
    band = band_of(score_mod)
    spec = build_spec(score_mod, None, batch=B, heads_q=Hq, seq_q=S, seq_kv=S, device=q.device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    p = _lib.RingBwdParams()
    p.dtype = dtype_code(q.dtype)
    p.batch, p.num_heads_q, p.num_heads_kv, p.seq_local, p.head_dim = B, Hq, k.shape[1], S, D
    p.q, p.k, p.v, p.out, p.lse, p.d_out = (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                            do.data_ptr())
    p.dq, p.dk, p.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    p.softmax_scale = softmax_scale(D)
    if band is not None:
        p.has_band, p.band_lo, p.band_hi = 1, band[0], band[1]
    p.alibi_slopes = spec.struct.alibi_slopes
    p.zigzag = int(bool(zigzag))
    nbytes = lib.attn_ring_bwd_workspace_size(C.byref(p), world)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    cs = torch.cuda.current_stream(q.device)
    ms = _comm_stream(q.device)
    comm = comm_for(group, q.device)
    _lib.check(lib.attn_ring_bwd(C.byref(p), comm, C.c_void_p(cs.cuda_stream), C.c_void_p(ms.cuda_stream)),
               "attn_ring_bwd")
    for t in (q, k, v, o, do, lse, ws, dq, dk, dv):
        t.record_stream(ms)
    del spec
    return dq, dk, dv


def plan(world, rank, seq_local, zigzag, band, position_free):
    """The library's launch plan for one rank, as a list of dicts (no GPU)."""
    lib = _lib.load()
    has, lo, hi = (0, 0, 0) if band is None else (1, band[0], band[1])
    cap = 4 * world + 8
    arr = (C.c_int64 * (10 * cap))()
    n = lib.attn_ring_plan(world, rank, seq_local, int(zigzag), has, lo, hi, int(position_free), arr, cap)
    if n < 0:
        _lib.check(-n, "attn_ring_plan")
    return [dict(zip(_lib.RING_PLAN_FIELDS, arr[10 * i:10 * i + 10])) for i in range(n)]
