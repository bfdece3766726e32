"""Ring schedule host logic on CPU ranks (gloo), world sizes 2 and 4.

The schedule (zig-zag re-deal, K/V rotation, global offsets, LSE merge
order, return of the outputs) runs exactly as on GPUs; only the per-step
attention and the merge are the numpy oracle instead of the kernels.  Each
rank's output shard must equal the oracle's attention on the global
sequence (what ring_attention_reference computes, attention.py:694-721).
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleOps:
    """Ring ops with the numpy oracle standing in for the kernels."""

    def __init__(self, group, mod, mask, hq, hkv):
        from attnax_b200._ring_impl import DistExchange

        self.x = DistExchange(group)
        self.mod, self.mask, self.rep = mod, mask, hq // hkv
        # True when the chain only selects a band (none / causal / window), as
        # KernelOps decides from the tagged mods: the schedule may then batch
        # fully kept pairs into position-free calls (attend_full).  The workers
        # set it per case and count the batched calls.
        self.position_free = False
        self.full_calls = 0

    def exchange(self, sends, recvs):
        self.x.exchange(sends, recvs)

    def start_rotate(self, kv, to, frm):
        return self.x.start_rotate(kv, to, frm)

    def finish_rotate(self, pending):
        return self.x.finish_rotate(pending)

    def new_acc(self, qp):
        B, H, n, D = qp.shape
        return (torch.zeros(B, H, n, D, dtype=torch.float64), torch.full((B, H, n), -np.inf, dtype=torch.float64))

    def attend(self, q, k, v, qc, kc):
        n = q.shape[2]
        qn, kn, vn = (t.double().numpy() for t in (q, k, v))
        kn, vn = np.repeat(kn, self.rep, 1), np.repeat(vn, self.rep, 1)
        m = None
        if self.mask is not None:
            m = self.mask[..., qc.local_start:qc.local_start + n, kc.local_start:kc.local_start + n]
        s = O.attention_oracle._final_scores(qn, kn, m, self.mod, qc.start, kc.start)
        empty = np.all(s == np.finfo(s.dtype).min, axis=-1)
        o, lse = O.standard_attention_lse(qn, kn, vn, mask=m, score_mod=self.mod,
                                          q_offset=qc.start, kv_offset=kc.start)
        o[empty] = 0.0
        lse[empty] = -np.inf
        return torch.from_numpy(o), torch.from_numpy(lse)

    def attend_full(self, q, k, v):
        self.full_calls += 1
        qn, kn, vn = (t.double().numpy() for t in (q, k, v))
        kn, vn = np.repeat(kn, self.rep, 1), np.repeat(vn, self.rep, 1)
        o, lse = O.standard_attention_lse(qn, kn, vn)
        return torch.from_numpy(o), torch.from_numpy(lse)

    def grad(self, q, k, v, o, lse, do, qc, kc):
        """Partial (dq, dk, dv) of one chunk pair from the global lse:
        P = exp(s - lse), dS = P (dP - rowsum(dO o)), zero where the score
        was dropped (the reference's ``where`` blocks the gradient)."""
        n, D = q.shape[2], q.shape[3]
        qn, kn, vn, on, dn = (t.double().numpy() for t in (q, k, v, o, do))
        ln = lse.double().numpy()[..., None]
        kr, vr = np.repeat(kn, self.rep, 1), np.repeat(vn, self.rep, 1)
        m = None
        if self.mask is not None:
            m = self.mask[..., qc.local_start:qc.local_start + n, kc.local_start:kc.local_start + n]
        s = O.attention_oracle._final_scores(qn, kr, m, self.mod, qc.start, kc.start)
        keep = s != np.finfo(s.dtype).min
        with np.errstate(over="ignore", invalid="ignore"):
            p = np.where(np.isinf(ln), 0.0, np.exp(s - ln))
        dv = np.einsum("bhqk,bhqd->bhkd", p, dn)
        dp = np.einsum("bhqd,bhkd->bhqk", dn, vr)
        ds = np.where(keep, p * (dp - (dn * on).sum(-1, keepdims=True)), 0.0)
        sc = O.softmax_scale(D, np.float64)
        dq = np.einsum("bhqk,bhkd->bhqd", ds, kr) * sc
        dk = np.einsum("bhqk,bhqd->bhkd", ds, qn) * sc
        fold = lambda x: x.reshape(x.shape[0], -1, self.rep, *x.shape[2:]).sum(2)  # noqa: E731
        return torch.from_numpy(dq), torch.from_numpy(fold(dk)), torch.from_numpy(fold(dv))

    def merge(self, acc, o_p, lse_p):
        o_a, l_a = acc
        m = torch.maximum(l_a, lse_p)
        safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
        wa = torch.where(torch.isinf(l_a), torch.zeros_like(l_a), torch.exp(l_a - safe))
        wp = torch.where(torch.isinf(lse_p), torch.zeros_like(lse_p), torch.exp(lse_p - safe))
        tot = wa + wp
        nz = tot > 0
        ca = torch.where(nz, wa / torch.where(nz, tot, torch.ones_like(tot)), torch.ones_like(tot))
        cp = torch.where(nz, wp / torch.where(nz, tot, torch.ones_like(tot)), torch.zeros_like(tot))
        o_a.mul_(ca[..., None]).add_(cp[..., None] * o_p)
        l_a.copy_(torch.where(nz, safe + torch.log(torch.where(nz, tot, torch.ones_like(tot))), l_a))

    def finalize(self, acc, dtype):
        return acc[0].to(dtype)


CASES = ("none", "causal", "causal_alibi_window", "local_mask", "causal_local_mask")


def _worker(rank, world, port, q, k, v, want):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from attnax_b200._ring_impl import RingSchedule, ring_schedule_forward

        S = q.shape[2] // world
        sl = slice(rank * S, (rank + 1) * S)
        H = q.shape[1]
        local_mask = np.random.default_rng(5).random((1, 1, S, S)) > 0.3
        for case in CASES:
            mod, mask, band, zig = None, None, None, False
            if case in ("causal", "causal_local_mask"):
                mod, band, zig = O.causal_mod(), (0, 1 << 62), True
            elif case == "causal_alibi_window":
                mod = O.compose_score_mods(O.sliding_window_mod(S // 2 + 3), O.alibi_mod(H))
                band, zig = (0, S // 2 + 2), True
            if case in ("local_mask", "causal_local_mask"):
                mask = local_mask
            sched = RingSchedule(world, rank, S, zig)
            ops = OracleOps(None, mod, mask, q.shape[1], k.shape[1])
            ops.position_free = case in ("none", "causal")
            tq, tk, tv = (torch.from_numpy(np.ascontiguousarray(x[:, :, sl])).double() for x in (q, k, v))
            out, _ = ring_schedule_forward(tq, tk, tv, ops=ops, sched=sched, band=band)
            np.testing.assert_allclose(out.numpy(), want[case][:, :, sl], atol=1e-10, rtol=1e-10,
                                       err_msg=case)
            if case == "causal":
                # zig-zag causal hops whose two kept chunk pairs are whole run as one
                # batched position-free call (every rank has at least one such hop)
                assert ops.full_calls > 0, "the batched hop path did not run"
            if case == "none":
                # no band: every hop's 4 pairs are kept, none is batched (2 chunks per
                # rank only under zig-zag)
                assert ops.full_calls == 0
    finally:
        dist.destroy_process_group()


def _bwd_worker(rank, world, port, q, k, v, do, want):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from attnax_b200._ring_impl import RingSchedule, ring_schedule_backward, ring_schedule_forward

        S = q.shape[2] // world
        sl = slice(rank * S, (rank + 1) * S)
        H = q.shape[1]
        for case in ("none", "causal", "causal_alibi_window"):
            mod, band, zig = None, None, False
            if case == "causal":
                mod, band, zig = O.causal_mod(), (0, 1 << 62), True
            elif case == "causal_alibi_window":
                mod = O.compose_score_mods(O.sliding_window_mod(S // 2 + 3), O.alibi_mod(H))
                band, zig = (0, S // 2 + 2), True
            sched = RingSchedule(world, rank, S, zig)
            ops = OracleOps(None, mod, None, q.shape[1], k.shape[1])
            ops.position_free = case in ("none", "causal")
            tq, tk, tv, tdo = (torch.from_numpy(np.ascontiguousarray(x[:, :, sl])).double() for x in (q, k, v, do))
            st = {}
            ring_schedule_forward(tq, tk, tv, ops=ops, sched=sched, band=band, state=st)
            dq, dk, dv = ring_schedule_backward(st["q"], st["k"], st["v"], st["out"], st["lse"], tdo, ops=ops,
                                                sched=sched, band=band)
            for name, got, w in zip(("dq", "dk", "dv"), (dq, dk, dv), want[case]):
                # (1e-6: the oracle's closed-form backward rounds the scale to float32)
                np.testing.assert_allclose(got.numpy(), w[:, :, sl], atol=1e-6, rtol=1e-6,
                                           err_msg=f"{case} {name}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ring_backward_schedule_matches_global_gradients(world):
    """dK/dV travel with their K/V and come home after P hops; every rank's
    gradient shards equal the global attention's gradients."""
    rng = np.random.default_rng(10 + world)
    B, Hq, Hkv, S, D = 1, 4, 2, 16 * world, 8
    q, k, v, do = (rng.standard_normal((B, h, S, D)) for h in (Hq, Hkv, Hkv, Hq))
    Sl = S // world
    want = {
        "none": O.gqa_attention_bwd(q, k, v, do),
        "causal": O.gqa_attention_bwd(q, k, v, do, score_mod=O.causal_mod()),
        "causal_alibi_window": O.gqa_attention_bwd(q, k, v, do, score_mod=O.compose_score_mods(
            O.sliding_window_mod(Sl // 2 + 3), O.alibi_mod(Hq))),
    }
    mp.spawn(_bwd_worker, args=(world, _free_port(), q, k, v, do, want), nprocs=world, join=True)


@pytest.mark.parametrize("world", [2, 4])
def test_ring_schedule_matches_global_attention(world):
    rng = np.random.default_rng(world)
    B, Hq, Hkv, S, D = 1, 4, 2, 16 * world, 8
    q = rng.standard_normal((B, Hq, S, D))
    k = rng.standard_normal((B, Hkv, S, D))
    v = rng.standard_normal((B, Hkv, S, D))
    Sl = S // world
    want = {
        "none": O.gqa_attention(q, k, v),
        "causal": O.gqa_attention(q, k, v, score_mod=O.causal_mod()),
        "causal_alibi_window": O.gqa_attention(q, k, v, score_mod=O.compose_score_mods(
            O.sliding_window_mod(Sl // 2 + 3), O.alibi_mod(Hq))),
    }
    # A local mask is applied at every step with local indices (attention.py:659-660):
    mask = np.random.default_rng(5).random((1, 1, Sl, Sl)) > 0.3
    kr, vr = np.repeat(k, 2, 1), np.repeat(v, 2, 1)
    want["local_mask"] = O.ring_attention_partitioned(q, kr, vr, world, mask=mask)
    want["causal_local_mask"] = O.ring_attention_partitioned(q, kr, vr, world, mask=mask,
                                                             score_mod=O.causal_mod())
    mp.spawn(_worker, args=(world, _free_port(), q, k, v, want), nprocs=world, join=True)
