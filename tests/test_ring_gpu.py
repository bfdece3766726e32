"""Ring attention over NCCL on 2 GPUs against the oracle's global attention.

Skipped on boxes with fewer than two GPUs; the host-side schedule is covered
on CPU ranks by test_ring_cpu.py.
"""

import os
import socket

import numpy as np
import pytest
import torch

import oracle as O
from tests._util import BF16_MAX_ABS, BF16_MEAN_REL, BF16_STORE_REL, errors

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, k, v, want, result_dir):
    import datetime

    import torch.distributed as dist

    import attnax_b200 as ax
    from attnax_b200.ring import bind_axis

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        bind_axis("sp")
        S = q.shape[2] // world
        sl = slice(rank * S, (rank + 1) * S)
        H = q.shape[1]
        T = lambda x: torch.tensor(np.ascontiguousarray(x[:, :, sl]), dtype=torch.bfloat16, device="cuda")  # noqa: E731
        tq, tk, tv = T(q), T(k), T(v)
        mods = {"causal": ax.causal_mod(), "none": None,
                "window_alibi": ax.compose_score_mods(ax.sliding_window_mod(S // 2 + 5), ax.alibi_mod(H))}
        lines = []
        with torch.no_grad():
            for name, mod in mods.items():
                out = ax.ring_attention(tq, tk, tv, score_mod=mod, axis_name="sp")
                mx, rel = errors(out.float().cpu().numpy(), want[name][:, :, sl])
                lines.append(f"{name} {mx} {rel}")
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write("\n".join(lines))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="ring over NCCL needs two GPUs")
def test_ring_two_gpus_matches_global_attention(tmp_path):
    import torch.multiprocessing as mp

    rng = np.random.default_rng(0)
    B, Hq, Hkv, S, D = 1, 8, 2, 2048, 128
    q = O.bf16_round(rng.standard_normal((B, Hq, S, D), dtype=np.float32))
    k = O.bf16_round(rng.standard_normal((B, Hkv, S, D), dtype=np.float32))
    v = O.bf16_round(rng.standard_normal((B, Hkv, S, D), dtype=np.float32))
    want = {"causal": O.gqa_attention(q, k, v, score_mod=O.causal_mod()), "none": O.gqa_attention(q, k, v),
            "window_alibi": O.gqa_attention(q, k, v, score_mod=O.compose_score_mods(
                O.sliding_window_mod(S // 4 + 5), O.alibi_mod(Hq)))}
    mp.spawn(_worker, args=(2, _free_port(), q, k, v, want, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        for line in (tmp_path / f"rank{r}.txt").read_text().splitlines():
            name, mx, rel = line.split()
            assert float(mx) <= BF16_MAX_ABS and float(rel) <= BF16_MEAN_REL, f"rank {r} {line}"


def _bwd_worker(rank, world, port, q, k, v, do, want, result_dir):
    import datetime

    import torch.distributed as dist

    import attnax_b200 as ax
    from attnax_b200.ring import bind_axis

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        bind_axis("sp")
        S = q.shape[2] // world
        sl = slice(rank * S, (rank + 1) * S)
        H = q.shape[1]
        mods = {"causal": ax.causal_mod(),
                "window_alibi": ax.compose_score_mods(ax.sliding_window_mod(S // 2 + 5), ax.alibi_mod(H))}
        lines = []
        for name, mod in mods.items():
            tq, tk, tv = (torch.tensor(np.ascontiguousarray(x[:, :, sl]), dtype=torch.bfloat16, device="cuda",
                                       requires_grad=True) for x in (q, k, v))
            out = ax.ring_attention(tq, tk, tv, score_mod=mod, axis_name="sp")
            out.backward(torch.tensor(np.ascontiguousarray(do[:, :, sl]), dtype=torch.bfloat16, device="cuda"))
            for gname, g, w in zip(("dq", "dk", "dv"), (tq.grad, tk.grad, tv.grad), want[name]):
                got, ref = g.float().cpu().numpy().astype(np.float64), w[:, :, sl].astype(np.float64)
                _, rel = errors(got, ref)
                excess = float(np.max(np.abs(got - ref) - BF16_STORE_REL * np.abs(ref)))
                lines.append(f"{name}_{gname} {excess} {rel}")
        with open(os.path.join(result_dir, f"bwd_rank{rank}.txt"), "w") as f:
            f.write("\n".join(lines))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="ring over NCCL needs two GPUs")
def test_ring_two_gpus_backward_matches_global_gradients(tmp_path):
    """The ring backward (K/V and dK/dV rotation, per-pair tcgen05 backward
    with the global LSE) against the gradients of global attention."""
    import torch.multiprocessing as mp

    rng = np.random.default_rng(1)
    B, Hq, Hkv, S, D = 1, 8, 2, 1024, 128
    q, k, v, do = (O.bf16_round(rng.standard_normal((B, h, S, D), dtype=np.float32)) for h in (Hq, Hkv, Hkv, Hq))
    want = {"causal": O.gqa_attention_bwd(q, k, v, do, score_mod=O.causal_mod()),
            "window_alibi": O.gqa_attention_bwd(q, k, v, do, score_mod=O.compose_score_mods(
                O.sliding_window_mod(S // 4 + 5), O.alibi_mod(Hq)))}
    mp.spawn(_bwd_worker, args=(2, _free_port(), q, k, v, do, want, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        for line in (tmp_path / f"bwd_rank{r}.txt").read_text().splitlines():
            # |err| - 2^-8 |ref| (bf16 storage rounding of each gradient) within the 2e-2 bar
            name, excess, rel = line.split()
            assert float(excess) <= BF16_MAX_ABS and float(rel) <= BF16_MEAN_REL, f"rank {r} {line}"
