"""Sequence-parallel ring attention (attnax/kernels/attention.py:540-721).

In the reference, ``axis_name`` names a JAX mesh axis bound by
``shard_map``/``pmap``; an unbound name falls back to the local kernel
(:590-616).  Here an axis is a ``torch.distributed`` process group (one
process per GPU) registered under a name with :func:`bind_axis`; unbound
names fall back to the local flash kernel the same way.
"""

from __future__ import annotations

import torch

from . import _ring_capi
from .flash import _output_dropout, attention

_AXES = {}


def bind_axis(name: str, process_group=None):
    """Binds ``name`` to a process group (the default group when ``None``)."""
    import torch.distributed as dist

    if not dist.is_initialized():
        raise RuntimeError("torch.distributed is not initialised")
    _AXES[name] = process_group if process_group is not None else dist.group.WORLD


def unbind_axis(name: str):
    _AXES.pop(name, None)


def ring_attention(query, key, value, *, mask=None, score_mod=None, dropout_rng=None,
                   dropout_rate: float = 0.0, deterministic: bool = True, axis_name=None,
                   block_size: int = 512):
    """Ring attention over the ranks bound to ``axis_name``; local when unbound."""
    if axis_name is None or axis_name not in _AXES:
        out = attention(query, key, value, mask=mask, score_mod=score_mod)
        return _output_dropout(out, dropout_rng, dropout_rate, deterministic)
    out = ring_forward(query, key, value, mask=mask, score_mod=score_mod, group=_AXES[axis_name])
    return _output_dropout(out, dropout_rng, dropout_rate, deterministic)


def ring_forward(query, key, value, *, mask=None, score_mod=None, group=None, zigzag=None):
    """Ring attention of the local shards over every rank of ``group``.

    ``query`` (B, Hq, S, D) and ``key``/``value`` (B, Hkv, S, D) are this
    rank's contiguous shard of the global sequence; returns this rank's
    output shard.  ``mask`` (and an additive bias) are local
    ``(.., S, S)`` tensors applied at every step, as in the reference
    (attention.py:659-660).  Differentiable in ``query``/``key``/``value``:
    the backward runs the ring again (``ring_schedule_backward``), where the
    reference differentiates its ``lax.scan``/``ppermute`` with JAX autodiff.
    """
    import torch

    from .flash import check_qkv

    B, Hq, Hkv, S, Skv, D = check_qkv(query, key, value)
    if S != Skv:
        raise ValueError("ring_attention needs equal local query and key/value shard lengths")
    if torch.is_grad_enabled() and (query.requires_grad or key.requires_grad or value.requires_grad):
        return _RingFn.apply(query, key, value, score_mod, mask, group, zigzag)
    return _ring_run(query, key, value, score_mod, mask, group, zigzag, None)


def _ring_run(query, key, value, score_mod, mask, group, zigzag, state):
    import torch.distributed as dist

    from ._ring_impl import KernelOps, RingSchedule, ring_schedule_forward
    from ._spec import band_of, may_empty_rows

    B, Hq, S = query.shape[0], query.shape[1], query.shape[2]
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    band = band_of(score_mod)
    if zigzag is None:
        zigzag = band is not None and band[0] >= 0 and world > 1
    sched = RingSchedule(world, rank, S, zigzag)
    ops = KernelOps(group, score_mod, mask, B, Hq, S, query.device)
    if world > 1 and _ring_capi.eligible(query, key, value, score_mod, mask) and (
            band is None or band[0] <= 0 <= band[1]):
        # Position-only chains: the whole ring runs in the library (attn_ring_fwd).
        out, lse = _ring_capi.ring_fwd(query, key, value, score_mod, group, zigzag=sched.zigzag)
        if state is not None:
            state.update(public=True, q=query.contiguous(), k=key.contiguous(), v=value.contiguous(), out=out,
                         lse=lse, sched=sched, ops=ops, band=band, empty=False, score_mod=score_mod, group=group)
        return out
    out, acc = ring_schedule_forward(query.contiguous(), key.contiguous(), value.contiguous(),
                                     ops=ops, sched=sched, band=band, state=state)
    empty = may_empty_rows(score_mod, mask)
    if empty:
        out = _fill_empty_rows(out, sched, acc, value, group)
    if state is not None:
        state.update(sched=sched, ops=ops, band=band, empty=empty)
    return out


class _RingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, score_mod, mask, group, zigzag):
        st = {}
        out = _ring_run(q, k, v, score_mod, mask, group, zigzag, st)
        ctx.st, ctx.dtypes = st, (q.dtype, k.dtype, v.dtype)
        return out

    @staticmethod
    def backward(ctx, dout):
        from ._ring_impl import ring_schedule_backward

        st = ctx.st
        if st.get("public"):
            # the library ran the forward ring; its backward ring (attn_ring_bwd)
            # takes the same public-layout shards
            dq, dk, dv = _ring_capi.ring_bwd(st["q"], st["k"], st["v"], st["out"], st["lse"], dout,
                                             st["score_mod"], st["group"], st["sched"].zigzag)
            ctx.st = None
            tq, tk, tv = ctx.dtypes
            return dq.to(tq), dk.to(tk), dv.to(tv), None, None, None, None
        dq, dk, dv = ring_schedule_backward(st["q"], st["k"], st["v"], st["out"], st["lse"],
                                            dout.to(st["q"].dtype).contiguous(), ops=st["ops"],
                                            sched=st["sched"], band=st["band"], empty_rows=st["empty"])
        ctx.st = None
        tq, tk, tv = ctx.dtypes
        return dq.to(tq), dk.to(tk), dv.to(tv), None, None, None, None


def _fill_empty_rows(out, sched, acc, value, group):
    """Rows that kept no key anywhere average the whole global V (the reference's softmax of
    an all-finfo.min row); every rank joins the all-reduce so the collective order matches."""
    import torch
    import torch.distributed as dist

    from ._ring_impl import redeal

    vsum = value.float().sum(dim=2)                      # (B, Hkv, D)
    dist.all_reduce(vsum, group=group)
    n_glob = value.shape[2] * dist.get_world_size(group)
    lse = torch.cat([a[1] for a in acc], dim=2)[..., None]  # (B, Hq, S, 1) in ring layout
    if sched.zigzag:
        (lse,) = redeal(sched, _Xchg(group), [lse], to_work=False)
    grp = out.shape[1] // value.shape[1]
    mean = (vsum / n_glob).repeat_interleave(grp, dim=1)[:, :, None, :].to(out.dtype)
    return torch.where(lse == float("-inf"), mean, out)


class _Xchg:
    def __init__(self, group):
        from ._ring_impl import DistExchange

        self._x = DistExchange(group)

    def exchange(self, sends, recvs):
        self._x.exchange(sends, recvs)


def ring_attention_reference(query, key, value, *, mask=None, score_mod=None):
    """Single-device equivalent of the ring on the global sequence (attention.py:694-721)."""
    return attention(query, key, value, mask=mask, score_mod=score_mod)
