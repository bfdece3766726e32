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
            tq, tk, tv = (torch.from_numpy(np.ascontiguousarray(x[:, :, sl])).double() for x in (q, k, v))
            out, _ = ring_schedule_forward(tq, tk, tv, ops=ops, sched=sched, band=band)
            np.testing.assert_allclose(out.numpy(), want[case][:, :, sl], atol=1e-10, rtol=1e-10,
                                       err_msg=case)
    finally:
        dist.destroy_process_group()


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
