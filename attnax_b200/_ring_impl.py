"""Host-side ring schedule for ``ring_attention`` (attnax/kernels/attention.py:540-691).

One process per GPU; ``group`` is the process group bound to the axis name.
Rank r holds the contiguous shard ``[r*S, (r+1)*S)`` of the global sequence,
as in the reference.  Each ring step attends the local queries to one visiting
K/V shard with global position offsets (:640-657), and folds the result into
a running output by log-sum-exp (the per-step update of :662-671); the K/V
shard then moves one rank forward (:673-674, ``lax.ppermute`` there, NCCL
send/recv here, overlapped with the next step's attention).  K/V travel with
their own ``Hkv`` heads rather than repeated to ``Hq``.

For causal masks the work of a contiguous ring is lopsided (rank P-1 attends
P blocks, rank 0 one), so the shards are re-dealt "zig-zag": the sequence is
cut into 2P chunks and every rank works on two chunks whose indices sum to
2P-1, which gives every rank the same number of unmasked chunk pairs at
every step.  The pairs are (2r, 2P-1-2r): rank r keeps the first chunk of
its own shard and swaps its second one with rank P-1-r, so the re-deal is
one exchange between mirror ranks and the diagonal block of the kept chunk
can run while it is in flight.  The re-deal and the final return of the
outputs are point-to-point copies; results are identical, only the order of
work changes.

``RingSchedule`` holds the schedule and is independent of the device: it
calls an ``ops`` object for attention, merging and point-to-point exchange,
so the multi-rank host logic can run on CPU ranks with a reference ``ops``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class Chunk:
    cid: int          # global chunk index
    start: int        # global position of its first row
    local_start: int  # position within the contiguous shard that owns it in the public layout
    owner: int        # rank owning it in the public (contiguous) layout


class RingSchedule:
    def __init__(self, world: int, rank: int, seq_local: int, zigzag: bool):
        if zigzag and seq_local % 2:
            zigzag = False
        self.P, self.r, self.S, self.zigzag = world, rank, seq_local, zigzag
        self.C = seq_local // 2 if zigzag else seq_local
        self.nchunks = 2 * world if zigzag else world

    def chunk(self, cid: int) -> Chunk:
        start = cid * self.C
        owner = start // self.S
        return Chunk(cid, start, start - owner * self.S, owner)

    def worker_of(self, cid: int) -> int:
        """Rank that works on chunk ``cid`` during the ring."""
        if not self.zigzag:
            return cid
        return cid // 2 if cid % 2 == 0 else (2 * self.P - 1 - cid) // 2

    def held(self, rank: int):
        """Chunks rank ``rank`` works on, in its buffer order."""
        if not self.zigzag:
            return [rank]
        return [2 * rank, 2 * self.P - 1 - 2 * rank]

    def public(self, rank: int):
        """Chunks rank ``rank`` holds in the public layout, in shard order."""
        per = self.S // self.C
        return [rank * per + h for h in range(per)]


def _pairs_all_masked(band, q_start, kv_start, n):
    """True when the band drops every (q, kv) pair of two n-row chunks."""
    if band is None:
        return False
    lo, hi = band
    dmax = (q_start + n - 1) - kv_start
    dmin = q_start - (kv_start + n - 1)
    return dmax < lo or dmin > hi


def redeal(sched: RingSchedule, ops, tensors, to_work: bool):
    """Moves chunk buffers between the public layout and the ring layout.

    ``tensors`` is a list of tensors (B, H, rows, D) in the source layout;
    returns the same tensors in the destination layout.  All tensors travel
    in one batched exchange (messages between two ranks pair up in tensor
    order on both sides).
    """
    P, r = sched.P, sched.r
    src_chunks = sched.public(r) if to_work else sched.held(r)
    dst_chunks = sched.held(r) if to_work else sched.public(r)
    dst_of = sched.worker_of if to_work else (lambda c: sched.chunk(c).owner)
    src_of = (lambda c: sched.chunk(c).owner) if to_work else sched.worker_of
    sends, recvs, all_dst = [], [], []
    for t in tensors:
        parts_src = list(torch.split(t, sched.C, dim=2))
        parts_dst = [None] * len(dst_chunks)
        for i, c in enumerate(src_chunks):
            peer = dst_of(c)
            if peer == r:
                parts_dst[dst_chunks.index(c)] = parts_src[i]
            else:
                sends.append((parts_src[i].contiguous(), peer))
        for j, c in enumerate(dst_chunks):
            if parts_dst[j] is None:
                buf = torch.empty_like(parts_src[0], memory_format=torch.contiguous_format)
                parts_dst[j] = buf
                recvs.append((buf, src_of(c)))
        all_dst.append(parts_dst)
    ops.exchange(sends, recvs)
    return [torch.cat(p, dim=2) if len(p) > 1 else p[0].contiguous() for p in all_dst]


def _pair_full(band, q_start, kv_start, n):
    """True when the band keeps every (q, kv) pair of two n-row chunks."""
    if band is None:
        return True
    lo, hi = band
    return q_start - (kv_start + n - 1) >= lo and (q_start + n - 1) - kv_start <= hi


def ring_schedule_forward(q, k, v, *, ops, sched: RingSchedule, band, state=None):
    """Runs the ring; returns the local output shard in the public layout.

    ``band``: (lo, hi) of the causal/window selection, used to skip chunk
    pairs with nothing kept (the kernel would return an empty partial).
    ``state``: if a dict, receives what the backward needs, in the ring
    layout: ``q``, ``k``, ``v``, the output ``out`` and the merged ``lse``.
    """
    P, r, C = sched.P, sched.r, sched.C
    if sched.zigzag:
        q, k, v = redeal(sched, ops, [q, k, v], to_work=True)
    my_chunks = [sched.chunk(c) for c in sched.held(r)]
    q_parts = list(torch.split(q, C, dim=2))
    acc = [ops.new_acc(qp) for qp in q_parts]
    kv = (k.contiguous(), v.contiguous())
    for i in range(P):
        owner = (r - i) % P
        nxt = None
        if i < P - 1:
            nxt = ops.start_rotate(kv, to=(r + 1) % P, frm=(r - 1) % P)
        kv_chunks = [sched.chunk(c) for c in sched.held(owner)]
        k_parts = torch.split(kv[0], C, dim=2)
        v_parts = torch.split(kv[1], C, dim=2)
        pairs = [(qi, ki) for qi, qc in enumerate(my_chunks) for ki, kc in enumerate(kv_chunks)
                 if not _pairs_all_masked(band, qc.start, kc.start, C)]
        if getattr(ops, "position_free", False) and len(my_chunks) == 2 and len(pairs) == 2 and all(
                _pair_full(band, my_chunks[qi].start, kv_chunks[ki].start, C) for qi, ki in pairs):
            # Two fully kept pairs that share a kv chunk (or a q chunk) and whose
            # scores do not depend on positions: one kernel over both q chunks
            # (or both kv chunks) of the ring buffers.
            (qa, ka), (qb, kb) = pairs
            if ka == kb and qa != qb:
                o_p, lse_p = ops.attend_full(q, k_parts[ka], v_parts[ka])
                for qi in (0, 1):
                    ops.merge(acc[qi], o_p[:, :, qi * C:(qi + 1) * C].contiguous(),
                              lse_p[:, :, qi * C:(qi + 1) * C].contiguous())
                pairs = []
            elif qa == qb and ka != kb:
                o_p, lse_p = ops.attend_full(q_parts[qa], kv[0], kv[1])
                ops.merge(acc[qa], o_p, lse_p)
                pairs = []
        for qi, ki in pairs:
            o_p, lse_p = ops.attend(q_parts[qi], k_parts[ki], v_parts[ki], my_chunks[qi], kv_chunks[ki])
            ops.merge(acc[qi], o_p, lse_p)
        if nxt is not None:
            kv = ops.finish_rotate(nxt)
    outs = [ops.finalize(a, q_parts[0].dtype) for a in acc]
    out = torch.cat(outs, dim=2) if len(outs) > 1 else outs[0]
    if state is not None:
        state.update(q=q, k=k.contiguous(), v=v.contiguous(), out=out,
                     lse=torch.cat([a[1] for a in acc], dim=2) if len(acc) > 1 else acc[0][1])
    if sched.zigzag:
        (out,) = redeal(sched, ops, [out], to_work=False)
    return out, acc


def ring_schedule_backward(q, k, v, out, lse, dout, *, ops, sched: RingSchedule, band, empty_rows=False):
    """Gradients of the ring for this rank's shards.

    ``q``, ``k``, ``v``, ``out``, ``lse`` are in the ring layout (as the
    forward left them in ``state``), ``dout`` in the public layout.  The K/V
    shards travel the ring again; at every hop each kept (q chunk, kv chunk)
    pair gives exact partial gradients from the global ``lse`` and
    ``rowsum(dout * out)`` (the softmax of the whole row), dQ accumulates
    here and dK/dV accumulate in fp32 buffers that travel with their K/V --
    one rotation per hop brings every rank's own dK/dV home after the last
    hop.  ``empty_rows``: rows with no kept key anywhere (lse = -inf) get the
    reference's uniform-softmax term, dV += dout / S_global for every key
    (one all-reduce; their dQ and dK are zero).  Returns fp32
    ``(dq, dk, dv)`` in the public layout.
    """
    P, r, C = sched.P, sched.r, sched.C
    if sched.zigzag:
        (dout,) = redeal(sched, ops, [dout], to_work=True)
    my_chunks = [sched.chunk(c) for c in sched.held(r)]
    q_parts = torch.split(q, C, dim=2)
    o_parts = torch.split(out, C, dim=2)
    do_parts = torch.split(dout, C, dim=2)
    lse_parts = torch.split(lse, C, dim=2)
    dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    dq_parts = torch.split(dq, C, dim=2)
    kv = (k, v)
    dkv = (torch.zeros(k.shape, dtype=torch.float32, device=k.device),
           torch.zeros(v.shape, dtype=torch.float32, device=v.device))
    for i in range(P):
        owner = (r - i) % P
        nxt = ops.start_rotate(kv, to=(r + 1) % P, frm=(r - 1) % P) if i < P - 1 else None
        kv_chunks = [sched.chunk(c) for c in sched.held(owner)]
        k_parts, v_parts = torch.split(kv[0], C, dim=2), torch.split(kv[1], C, dim=2)
        dk_parts, dv_parts = torch.split(dkv[0], C, dim=2), torch.split(dkv[1], C, dim=2)
        for qi, qc in enumerate(my_chunks):
            for ki, kc in enumerate(kv_chunks):
                if _pairs_all_masked(band, qc.start, kc.start, C):
                    continue
                gq, gk, gv = ops.grad(q_parts[qi], k_parts[ki], v_parts[ki], o_parts[qi], lse_parts[qi],
                                      do_parts[qi], qc, kc)
                dq_parts[qi].add_(gq)
                dk_parts[ki].add_(gk)
                dv_parts[ki].add_(gv)
        # the accumulators follow their K/V: after hop i rank r holds owner (r - i - 1)'s
        dkv = ops.finish_rotate(ops.start_rotate(dkv, to=(r + 1) % P, frm=(r - 1) % P))
        if nxt is not None:
            kv = ops.finish_rotate(nxt)
    dk, dv = dkv
    if empty_rows:
        dv = dv + ops.empty_rows_dv(dout, lse, k.shape[1], C * sched.nchunks)[:, :, None, :]
    if sched.zigzag:
        dq, dk, dv = redeal(sched, ops, [dq, dk, dv], to_work=False)
    return dq, dk, dv


class DistExchange:
    """Point-to-point exchange over a ``torch.distributed`` group."""

    def __init__(self, group):
        self.group = group

    def _peer(self, group_rank):
        return dist.get_global_rank(self.group, group_rank) if self.group is not None else group_rank

    def exchange(self, sends, recvs):
        ops = [dist.P2POp(dist.isend, t, self._peer(p), self.group) for t, p in sends]
        ops += [dist.P2POp(dist.irecv, t, self._peer(p), self.group) for t, p in recvs]
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()

    def start_rotate(self, ts, to, frm):
        """Sends every tensor of ``ts`` to ``to`` and receives same-shaped ones from ``frm``."""
        new = tuple(torch.empty_like(t) for t in ts)
        ops = [dist.P2POp(dist.isend, t, self._peer(to), self.group) for t in ts]
        ops += [dist.P2POp(dist.irecv, t, self._peer(frm), self.group) for t in new]
        return dist.batch_isend_irecv(ops), new

    def finish_rotate(self, pending):
        works, kv = pending
        for w in works:
            w.wait()
        return kv

    def empty_rows_dv(self, dout, lse, heads_kv, n_global):
        """sum over this rank's rows with lse = -inf of dout, per kv head, summed
        over the ranks and divided by the global sequence length: (B, Hkv, D)."""
        B, Hq, _, D = dout.shape
        keep = (lse == float("-inf")).to(torch.float32 if dout.dtype != torch.float64 else torch.float64)
        s = (dout.to(keep.dtype) * keep[..., None]).sum(dim=2)
        s = s.view(B, heads_kv, Hq // heads_kv, D).sum(dim=2)
        dist.all_reduce(s, group=self.group)
        return s / n_global


class KernelOps(DistExchange):
    """Ring ops backed by libattnb200 (flash forward + LSE merge)."""

    def __init__(self, group, score_mod, mask, batch, heads_q, seq_local, device):
        super().__init__(group)
        self.score_mod, self.mask = score_mod, mask
        self.batch, self.heads_q, self.S, self.device = batch, heads_q, seq_local, device
        from ._spec import flatten_mods
        from .score_mods import CausalMod, SlidingWindowMod

        # Only band selections (causal / sliding window): a fully kept pair's
        # scores do not depend on positions.
        self.position_free = mask is None and all(isinstance(p, (CausalMod, SlidingWindowMod))
                                                  for p in flatten_mods(score_mod))

    def new_acc(self, q_part):
        B, H, n, D = q_part.shape
        return (torch.zeros(B, H, n, D, dtype=torch.float32, device=q_part.device),
                torch.full((B, H, n), float("-inf"), dtype=torch.float32, device=q_part.device))

    def _local(self, t, qc, kc, n):
        if t is None:
            return None
        t = torch.as_tensor(t, device=self.device)
        while t.dim() < 4:
            t = t[None]
        if t.shape[-2] != 1:
            t = t[..., qc.local_start:qc.local_start + n, :]
        if t.shape[-1] != 1:
            t = t[..., kc.local_start:kc.local_start + n]
        return t

    def _spec(self, q, k, qc, kc):
        from ._spec import build_spec
        from .score_mods import AdditiveBiasMod
        from ._spec import flatten_mods
        from ._api import compose_score_mods

        n = q.shape[2]
        mods = []
        for p in flatten_mods(self.score_mod):
            # The reference adds the same (local) bias every step (attention.py:646-657).
            mods.append(AdditiveBiasMod(self._local(p.bias, qc, kc, n)) if isinstance(p, AdditiveBiasMod) else p)
        spec = build_spec(compose_score_mods(*mods), self._local(self.mask, qc, kc, n), batch=self.batch,
                          heads_q=self.heads_q, seq_q=n, seq_kv=k.shape[2], device=self.device,
                          q_offset=qc.start, kv_offset=kc.start)
        spec.fix_masked_rows = False  # an empty partial must stay empty (lse = -inf)
        return spec

    def attend(self, q, k, v, qc, kc):
        from .flash import fwd_raw

        return fwd_raw(q.contiguous(), k.contiguous(), v.contiguous(), self._spec(q, k, qc, kc))

    def attend_full(self, q, k, v):
        """Unmasked attention of any q rows on any kv rows (pairs the band keeps whole)."""
        from ._spec import build_spec
        from .flash import fwd_raw

        spec = build_spec(None, None, batch=self.batch, heads_q=self.heads_q, seq_q=q.shape[2],
                          seq_kv=k.shape[2], device=self.device)
        spec.fix_masked_rows = False
        return fwd_raw(q.contiguous(), k.contiguous(), v.contiguous(), spec)

    def grad(self, q, k, v, o, lse, do, qc, kc):
        """Partial (dq, dk, dv) of one chunk pair from the global lse (rows with no
        key anywhere have lse = -inf: P = 0, their dV term is added by the caller)."""
        from .flash import bwd_raw

        return bwd_raw(q.contiguous(), k.contiguous(), v.contiguous(), o.contiguous(), lse.contiguous(),
                       do.contiguous(), self._spec(q, k, qc, kc))

    def merge(self, acc, o_p, lse_p):
        import ctypes as C

        from . import _lib
        from ._spec import dtype_code

        o_acc, lse_acc = acc
        rows = lse_acc.numel()
        _lib.check(_lib.load().attn_lse_merge(dtype_code(o_p.dtype), rows, o_p.shape[-1], o_acc.data_ptr(),
                                              lse_acc.data_ptr(), o_p.data_ptr(), lse_p.data_ptr(), None,
                                              C.c_void_p(torch.cuda.current_stream(o_p.device).cuda_stream)),
                   "attn_lse_merge")

    def finalize(self, acc, dtype):
        return acc[0].to(dtype)
