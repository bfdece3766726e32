"""Benchmark of the attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload flash|paged|document|fp32] [--scale full|small]

Default workload ("flash"): flash attention forward + backward, bf16,
B=4, Hq=32, Hkv=8, S=8192, D=128, compose(sliding_window_mod(4096),
alibi_mod(32)), q/k/v/dO ~ N(0,1).  One step = one forward and one backward
pass over that batch.  ``value`` is algorithmic TFLOP/s (only kept (q, kv)
pairs count; forward 4*D flops per pair and head, backward 2.5x forward)
summed over all ranks; inputs (>L2) are resident in HBM.  ``e2e`` is the same
step through the public API with the inputs copied from pinned host memory
and the scalar result read back every step.  At N>1 every rank runs its own
replica of the batch (independent (batch, head) units, no collective):
weak scaling.  The secondary workloads (paged decode, document mask, fp32)
run on rank 0 at the end and are reported under ``secondary``.

``--impl reference`` times the CPU restatement of the reference
(``oracle/``) on this host's cores, on a bounded sample of the same
workload, and prints the same metric.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(PEAKS_FALLBACK), "fallback"


# ----------------------------------------------------------------- configs --

def flash_cfg(scale):
    if scale == "small":  # same kernel, one batch (inputs still > L2): for ncu captures
        return dict(B=1, Hq=32, Hkv=8, S=8192, D=128, W=4096)
    return dict(B=4, Hq=32, Hkv=8, S=8192, D=128, W=4096)


def window_pairs(S, W):
    """Kept (q, kv) pairs of causal sliding window W over S positions."""
    if W >= S:
        return S * (S + 1) // 2
    return W * (W + 1) // 2 + (S - W) * W


def doc_lengths(S, seed=0):
    rng = np.random.default_rng(seed)
    lens = []
    while sum(lens) < S:
        lens.append(max(64, int(rng.geometric(1 / 2048))))
    lens[-1] -= sum(lens) - S
    if lens[-1] <= 0:
        lens.pop()
    return lens


def paged_setup(scale, seed=0):
    rng = np.random.default_rng(seed)
    nseq = 64 if scale == "full" else 16
    ctx = rng.integers(512, 32769, size=nseq)
    bs = 16
    pages = (ctx + bs - 1) // bs
    nb = int(math.ceil(1.2 * pages.sum()))
    perm = rng.permutation(nb)
    table = np.full((nseq, int(pages.max())), -1, np.int32)
    o = 0
    for s, n in enumerate(pages):
        table[s, :n] = perm[o:o + n]
        o += n
    return dict(nseq=nseq, ctx=ctx.astype(np.int32), bs=bs, nb=nb, table=table, Hq=32, Hkv=8, D=128)


def paged_tensors(c, dev):
    """Pools (N(0,1), bf16) and one decode query per sequence for ``paged_setup``."""
    import torch

    g = torch.Generator(device=dev).manual_seed(7)
    kp = torch.randn(c["nb"], c["bs"], c["Hkv"], c["D"], generator=g, device=dev).to(torch.bfloat16)
    vp = torch.randn(c["nb"], c["bs"], c["Hkv"], c["D"], generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(c["nseq"], c["Hq"], 1, c["D"], generator=g, device=dev).to(torch.bfloat16)
    return kp, vp, q


# ------------------------------------------------------------------ timing --

class Clocks:
    """Samples nvidia-smi clocks/throttle reasons while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        # Start timing only once the sampler is producing rows.
        t0 = time.time()
        while self.proc is not None and time.time() - t0 < 3.0:
            self.f.flush()
            if os.path.getsize(self.f.name) > 0:
                break
            time.sleep(0.02)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        try:
            rows = [r.split(",") for r in open(self.f.name).read().strip().splitlines() if r.strip()]
            os.unlink(self.f.name)
        except OSError:
            rows = []
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm, smax = float(r[1]), float(r[2])
            except (ValueError, IndexError):
                continue
            mhz.append(sm)
            mx = smax
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        load = [m for m in mhz if mx and m > 0.3 * mx] or mhz
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(mhz)}


class Timer:
    """CUDA-event timing on the current stream, max over ranks."""

    def __init__(self, torch, dist, world):
        self.torch, self.dist, self.world = torch, dist, world

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def run(self, step, steps, warmup, phases=None):
        torch = self.torch
        for _ in range(warmup):
            step(None)
        self.barrier()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        marks = {k: [] for k in (phases or [])}
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(steps):
            step(marks)
        end.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end)
        self.barrier()
        if self.world > 1:
            t = torch.tensor([ms], device="cuda")
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
            ms = float(t.item())
        phase_ms = {k: sum(a.elapsed_time(b) for a, b in v) / max(1, len(v)) for k, v in marks.items()}
        return ms / steps, phase_ms


def phase(torch, marks, name):
    """Context for per-phase CUDA events inside a timed step."""

    class _P:
        def __enter__(self_):
            if marks is not None:
                self_.a = torch.cuda.Event(enable_timing=True)
                self_.a.record()

        def __exit__(self_, *exc):
            if marks is not None:
                b = torch.cuda.Event(enable_timing=True)
                b.record()
                marks[name].append((self_.a, b))

    return _P()


# ------------------------------------------------------------- workloads --

def run_flash(args, torch, dist, rank, world, peaks):
    import attnax_b200 as ax
    from attnax_b200 import _lib
    from attnax_b200._spec import build_spec
    from attnax_b200.flash import bwd_raw, fwd_raw

    c = flash_cfg(args.scale)
    B, Hq, Hkv, S, D, W = c["B"], c["Hq"], c["Hkv"], c["S"], c["D"], c["W"]
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator().manual_seed(1000 * rank)
    mk = lambda *shape: torch.randn(*shape, generator=g).to(torch.bfloat16).pin_memory()  # noqa: E731
    hq, hk, hv, hdo = mk(B, Hq, S, D), mk(B, Hkv, S, D), mk(B, Hkv, S, D), mk(B, Hq, S, D)
    q, k, v, do = (t.to(dev) for t in (hq, hk, hv, hdo))
    mod = ax.compose_score_mods(ax.sliding_window_mod(W), ax.alibi_mod(Hq))
    spec = build_spec(mod, None, batch=B, heads_q=Hq, seq_q=S, seq_kv=S, device=dev)
    pairs = window_pairs(S, W)
    fwd_flops = 4.0 * D * Hq * B * pairs
    bwd_flops = 2.5 * fwd_flops
    tm = Timer(torch, dist, world)
    lib = _lib.load()

    state = {}

    def step(marks):
        with phase(torch, marks, "fwd"):
            out, lse = fwd_raw(q, k, v, spec, out=state.get("out"), lse=state.get("lse"))
        state["out"], state["lse"] = out, lse
        with phase(torch, marks, "bwd"):
            bwd_raw(q, k, v, out, lse, do, spec)

    with Clocks(torch.cuda.current_device()) as clk:
        n0 = lib.attn_launch_count()
        ms, ph = tm.run(step, args.steps, args.warmup, phases=["fwd", "bwd"])
        launches = lib.attn_launch_count() - n0
    # launches counted over warmup + timed steps; report the timed share
    launches = launches * args.steps // (args.steps + args.warmup)
    value = world * (fwd_flops + bwd_flops) / (ms * 1e-3) / 1e12

    # e2e: public API (autograd flash_attention); every step copies q, k, v
    # and dO from pinned host memory and copies the output and dQ, dK, dV
    # back to pinned host memory.  Uploads run one step ahead on a side
    # stream and downloads on another, so PCIe overlaps the kernels.
    def e2e_step(tq, tk, tv, tdo):
        tq, tk, tv = (t.detach().requires_grad_() for t in (tq, tk, tv))
        o = ax.flash_attention(tq, tk, tv, score_mod=mod)
        o.backward(tdo)
        return o.detach(), tq.grad, tk.grad, tv.grad

    host_res = [torch.empty_like(t).pin_memory() for t in (hq, hq, hk, hv)]  # out, dq, dk, dv
    e2e_steps = max(2, min(args.steps, 8))
    e2e_ms = e2e_pipelined(torch, dist, world, dev, (hq, hk, hv, hdo), host_res, e2e_step, e2e_steps, warmup=2)
    h2d, d2h = nbytes((hq, hk, hv, hdo)), nbytes(host_res)
    e2e_value = world * (fwd_flops + bwd_flops) / (e2e_ms * 1e-3) / 1e12

    peak_b, peak_s = peaks["bf16_tflops"], peaks["bf16_tflops_sustained"]
    kern = {}
    for name, fl in (("fwd", fwd_flops), ("bwd", bwd_flops)):
        a = fl / (ph[name] * 1e-3) / 1e12
        kern[name] = {"ms": round(ph[name], 4), "tflops": round(a, 2), "frac": round(a / peak_b, 4),
                      "frac_sustained": round(a / peak_s, 4)}
    dom = max(kern, key=lambda n: kern[n]["ms"])
    kernel_names = {"fwd": "fwd2::flash_fwd2_kernel<128,bf16> (tcgen05)",
                    "bwd": "attn_bwd: bwd::prep_rows_kernel + bwd::dkdv_kernel<128,bf16,fused dQ> "
                           "+ bwd::dq_convert_kernel (tcgen05)"}
    roof = {"kernel": kernel_names[dom], "bound": "tensor", "achieved": kern[dom]["tflops"],
            "peak": peak_b, "unit": "TFLOP/s", "frac": kern[dom]["frac"],
            "peak_sustained": peak_s, "frac_sustained": kern[dom]["frac_sustained"],
            "traffic": TRAFFIC.get(dom), "algorithmic_per_launch": (fwd_flops if dom == "fwd" else bwd_flops)}
    line = {
        "metric": "flash attention fwd+bwd TFLOP/s (algorithmic)", "value": round(value, 2),
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded torch.Generator",
        "config": {"workload": f"flash fwd+bwd B{B} Hq{Hq} Hkv{Hkv} S{S} D{D} "
                               f"sliding_window({W})+alibi({Hq})",
                   "batch": B, "heads_q": Hq, "heads_kv": Hkv, "seq_len": S, "head_dim": D, "window": W,
                   "pairs_per_head": pairs, "flops_fwd": fwd_flops, "flops_bwd": bwd_flops,
                   "parallelism": f"replica x{world} (independent batch/head units)",
                   "l2": "inputs larger than L2 (q 256 MiB, k/v 64 MiB each)"},
        "fwd_tflops": kern["fwd"]["tflops"], "bwd_tflops": kern["bwd"]["tflops"], "kernels": kern,
        "roofline": roof,
        "e2e": {"value": round(e2e_value, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
                "returned": "output, dQ, dK, dV to pinned host memory every step"},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "peaks_source": PEAKS_SRC,
    }
    return line


# Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of each
# phase at the B4 bench size: ncu capture of the B1 case of the same workload
# (profiles/flash_fwd2_kernel_small.md, profiles/flash_bwd_kernels_small.md) x 4
# batches.  fwd: flash_fwd2_kernel 134.5 MB; bwd: prep_rows 222.7 MB + fused dkdv
# 428.2 MB + dq_convert 176.3 MB.
TRAFFIC = {"fwd": 4 * 134.5e6, "bwd": 4 * (222.7e6 + 428.2e6 + 176.3e6)}
# Paged decode: DRAM bytes / algorithmic bytes of the 16-sequence capture
# (profiles/paged_decode_kernel_small.md); traffic scales with the tokens read.
PAGED_TRAFFIC_RATIO = (1.100622e9 + 6.36672e6) / 1.1001e9


def e2e_pipelined(torch, dist, world, dev, host_in, host_out, compute, steps, warmup):
    """ms per step of ``compute`` through the public API, end to end.

    Every step's inputs are copied from the pinned ``host_in`` buffers (on an
    upload stream, one step ahead, into two device buffer sets) and every
    step's results -- the tuple ``compute`` returns -- are copied back into
    the pinned ``host_out`` buffers (on a download stream).  The timed region
    ends when the last step's results have reached the host.
    """
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    comp = torch.cuda.current_stream()
    bufs = [[torch.empty_like(h, device=dev) for h in host_in] for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    for e in free:
        e.record(comp)

    def upload(slot):
        with torch.cuda.stream(up):
            up.wait_event(free[slot])
            for d, h in zip(bufs[slot], host_in):
                d.copy_(h, non_blocking=True)
            copied[slot].record(up)

    def run(n):
        upload(0)
        for i in range(n):
            slot = i % 2
            if i + 1 < n:
                upload((i + 1) % 2)
            comp.wait_event(copied[slot])
            res = compute(*bufs[slot])
            free[slot].record(comp)
            done = torch.cuda.Event()
            done.record(comp)
            with torch.cuda.stream(down):
                down.wait_event(done)
                for h, d in zip(host_out, res):
                    h.copy_(d, non_blocking=True)
                    d.record_stream(down)
        comp.wait_stream(down)

    run(warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(comp)
    run(steps)
    end.record(comp)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms / steps


def nbytes(ts):
    return sum(t.numel() * t.element_size() for t in ts)


def run_paged(args, torch, peaks):
    import attnax_b200 as ax
    from attnax_b200 import _lib
    from attnax_b200.paged import paged_decode_raw

    c = paged_setup(args.scale)
    dev = torch.device("cuda", torch.cuda.current_device())
    kp, vp, q = paged_tensors(c, dev)
    cache = ax.PagedKVCache(kp, vp, torch.tensor(c["table"], device=dev), torch.tensor(c["ctx"], device=dev))
    out = torch.empty_like(q)
    maxc = int(c["ctx"].max())
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)
    tm = Timer(torch, None, 1)
    lib = _lib.load()

    def step(marks):
        paged_decode_raw(q, cache, max_context=maxc, out=out, workspace=ws)

    n0 = lib.attn_launch_count()
    ms, _ = tm.run(step, args.steps * 5, args.warmup)
    launches = (lib.attn_launch_count() - n0) * args.steps * 5 // (args.steps * 5 + args.warmup)
    tokens = int(c["ctx"].sum())
    pages = int(((c["ctx"] + c["bs"] - 1) // c["bs"]).sum())
    alg_bytes = tokens * 2 * c["Hkv"] * c["D"] * 2 + pages * 4 + 2 * q.numel() * 2
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    return {"metric": "paged decode HBM GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "ms_per_step": round(ms, 4), "algorithmic_bytes": alg_bytes, "tokens": tokens,
            "config": f"{c['nseq']} seqs, ctx U[512,32768], page {c['bs']}, Hq{c['Hq']} Hkv{c['Hkv']} D{c['D']} bf16",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4),
                         "traffic": round(PAGED_TRAFFIC_RATIO * alg_bytes)},
            "gpu_launches": int(launches)}


def run_kv_cache(args, torch, peaks):
    """Decode step over the contiguous per-layer KV cache: batch 32, Hq32 Hkv8
    D128 bf16, 16000 of 16384 positions filled, one query position."""
    import attnax_b200 as ax
    from attnax_b200 import _lib

    B, Hq, Hkv, D = (32, 32, 8, 128) if args.scale == "full" else (8, 32, 8, 128)
    L, n = 16384, 16000
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(9)
    cache = ax.init_kv_layer_cache(B, Hkv, D, L, torch.bfloat16)
    cache = ax.update_kv_layer_cache(cache, torch.randn(B, Hkv, n, D, generator=g, device=dev).to(torch.bfloat16),
                                     torch.randn(B, Hkv, n, D, generator=g, device=dev).to(torch.bfloat16), 0)
    q = torch.randn(B, Hq, 1, D, generator=g, device=dev).to(torch.bfloat16)
    tm = Timer(torch, None, 1)
    lib = _lib.load()
    n0 = lib.attn_launch_count()
    ms, _ = tm.run(lambda m: ax.kv_cache_attention(q, cache), args.steps * 5, args.warmup)
    launches = (lib.attn_launch_count() - n0) * args.steps * 5 // (args.steps * 5 + args.warmup)
    alg_bytes = 2 * B * Hkv * n * D * 2 + 2 * q.numel() * 2
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    return {"metric": "KV-cache decode HBM GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "ms_per_step": round(ms, 4), "algorithmic_bytes": alg_bytes,
            "config": f"B{B} Hq{Hq} Hkv{Hkv} D{D} bf16, {n} of {L} cached positions, one query position",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4)},
            "gpu_launches": int(launches)}


def run_document(args, torch, peaks):
    import attnax_b200 as ax
    from attnax_b200._spec import build_spec
    from attnax_b200.flash import bwd_raw, fwd_raw

    S = 32768 if args.scale == "full" else 8192
    H, D = 16, 128
    lens = doc_lengths(S)
    ids = np.repeat(np.arange(len(lens)), lens)[None].astype(np.int32)
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(3)
    q, k, v = (torch.randn(1, H, S, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
    mod = ax.compose_score_mods(ax.document_mask_mod(ids), ax.causal_mod())
    spec = build_spec(mod, None, batch=1, heads_q=H, seq_q=S, seq_kv=S, device=dev)
    out = torch.empty_like(q)
    tm = Timer(torch, None, 1)
    ms, _ = tm.run(lambda m: fwd_raw(q, k, v, spec, out=out, want_lse=False), args.steps, args.warmup)
    pairs = sum(L * (L + 1) // 2 for L in lens)
    fl = 4.0 * D * H * pairs
    tf = fl / (ms * 1e-3) / 1e12
    # backward of the same call (P recomputed from the forward LSE)
    do = torch.randn(1, H, S, D, generator=g, device=dev).to(torch.bfloat16)
    o2, lse = fwd_raw(q, k, v, spec)
    ms_b, _ = tm.run(lambda m: bwd_raw(q, k, v, o2, lse, do, spec), args.steps, args.warmup)
    tf_b = 2.5 * fl / (ms_b * 1e-3) / 1e12
    return {"metric": "document-mask flash fwd TFLOP/s (algorithmic)", "value": round(tf, 2),
            "unit": "TFLOP/s", "ms_per_step": round(ms, 4), "docs": len(lens), "pairs": pairs,
            "bwd_tflops": round(tf_b, 2), "bwd_ms": round(ms_b, 4),
            "config": f"B1 S{S} H{H} D{D} bf16 document_mask+causal",
            "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": round(tf / peaks["bf16_tflops"], 4)}}


RING = dict(S=131072, Hq=32, Hkv=8, D=128)


def ring_shard(kind, rank, world, S, dtype=np.float32):
    """Rank ``rank``'s contiguous shard of the ring workload's q, k or v:
    N(0,1) drawn in fp32 from default_rng((seed, rank)), B1, (heads, S/P, D)."""
    heads = RING["Hq"] if kind == "q" else RING["Hkv"]
    seed = {"q": 31, "k": 32, "v": 33}[kind]
    Sl = S // world
    return np.random.default_rng((seed, rank)).standard_normal((1, heads, Sl, RING["D"]), dtype=dtype)


def run_ring(args, torch, dist, rank, world, peaks, headline=False):
    """Ring attention, B1 Hq32 Hkv8 D128 causal, global S split over the ranks (strong scaling).

    One step = one ring forward over the whole sequence (every rank its S/P
    shard).  At N>1 this is the headline line: it also carries the
    end-to-end number through ``ring_attention`` (host shards in, host
    output shard out), clocks, the launch count, and an in-run parity check
    of sampled output rows of every shard against the oracle.
    """
    import attnax_b200 as ax
    from attnax_b200 import _lib
    from attnax_b200.ring import bind_axis, ring_forward

    S = RING["S"] if args.scale == "full" else 16384
    Hq, Hkv, D = RING["Hq"], RING["Hkv"], RING["D"]
    Sl = S // world
    dev = torch.device("cuda", torch.cuda.current_device())
    if world > 1:
        # host shards from the seeded generator (the parity check regenerates them)
        hq, hk, hv = (torch.from_numpy(ring_shard(x, rank, world, S)).to(torch.bfloat16).pin_memory()
                      for x in ("q", "k", "v"))
        q, k, v = (t.to(dev) for t in (hq, hk, hv))
    else:
        g = torch.Generator(device=dev).manual_seed(11)
        q = torch.randn(1, Hq, Sl, D, generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn(1, Hkv, Sl, D, generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn(1, Hkv, Sl, D, generator=g, device=dev).to(torch.bfloat16)
    mod = ax.causal_mod()
    grp = dist.group.WORLD if world > 1 else None
    tm = Timer(torch, dist, world)
    state = {}

    def step(marks):
        with torch.no_grad():
            if world > 1:
                state["out"] = ring_forward(q, k, v, score_mod=mod, group=grp)
            else:
                state["out"] = ax.flash_attention(q, k, v, score_mod=mod)

    steps = max(2, min(args.steps, 5))
    lib = _lib.load()
    with Clocks(torch.cuda.current_device()) as clk:
        n0 = lib.attn_launch_count()
        ms, _ = tm.run(step, steps, 3)
        launches = (lib.attn_launch_count() - n0) * steps // (steps + 3)
    fl = 4.0 * D * Hq * S * (S + 1) / 2
    tf = fl / (ms * 1e-3) / 1e12
    line = {"metric": "ring attention tokens/s", "value": round(S / (ms * 1e-3), 1), "unit": "tokens/s",
            "n_gpus": world, "ms_per_step": round(ms, 3), "tflops_total": round(tf, 2),
            "tflops_per_gpu": round(tf / world, 2), "scaling": "strong",
            "config": f"B1 S{S} (S/P={Sl}) Hq{Hq} Hkv{Hkv} D{D} bf16 causal, "
                      f"{'zig-zag ring over NCCL' if world > 1 else 'one GPU, flash kernel'}"}
    if world == 1:
        return line
    # Per-GPU reference for the ring: one GPU's causal flash forward on a
    # sequence of the shard length S/P (same heads), no exchange.
    base = None
    if rank == 0:
        t1 = Timer(torch, None, 1)
        with torch.no_grad():
            b_ms, _ = t1.run(lambda m: ax.flash_attention(q, k, v, score_mod=mod), steps, 3)
        base = round(4.0 * D * Hq * Sl * (Sl + 1) / 2 / (b_ms * 1e-3) / 1e12, 2)
    dist.barrier()
    line["one_gpu_causal_tflops_at_shard_len"] = base
    if not headline:
        return line

    # e2e through the public API: this rank's q/k/v shard from pinned host
    # memory in, its output shard back to pinned host memory, every step.
    bind_axis("bench_sp", grp)

    def e2e_step(tq, tk, tv):
        with torch.no_grad():
            return (ax.ring_attention(tq, tk, tv, score_mod=mod, axis_name="bench_sp"),)

    host_out = [torch.empty_like(hq).pin_memory()]
    e2e_ms = e2e_pipelined(torch, dist, world, dev, (hq, hk, hv), host_out, e2e_step, steps, warmup=2)

    # In-run parity: sampled output rows of this rank's shard against the
    # oracle over the whole global sequence (all ranks' K/V regenerated here).
    import oracle as O

    out = state["out"].float().cpu().numpy()
    kg = np.concatenate([ring_shard("k", r, world, S) for r in range(world)], axis=2)
    vg = np.concatenate([ring_shard("v", r, world, S) for r in range(world)], axis=2)
    kg, vg = O.bf16_round(kg), O.bf16_round(vg)
    qn = hq.float().numpy()
    rows = np.unique(np.concatenate([[0, 1, Sl // 2, Sl - 1],
                                     np.random.default_rng(rank).choice(Sl, 12, replace=False)])) + rank * Sl
    diff = np.zeros(3)  # max-abs, sum |got - want|, sum |want|
    for h in (0, 13, 31):
        o, _ = O.gqa_attention_rows(qn, kg, vg, 0, [h], rows, score_mod=O.causal_mod(), q_offset=rank * Sl)
        got = out[0, h, rows - rank * Sl]
        d = np.abs(got.astype(np.float64) - o[0])
        diff += [0.0, d.sum(), np.abs(o[0]).sum()]
        diff[0] = max(diff[0], d.max())
    t = torch.tensor(diff, dtype=torch.float64, device=dev)
    mx = t[:1].clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    dist.all_reduce(t)
    parity = {"max_abs": float(mx.item()), "mean_rel": float(t[1].item() / max(t[2].item(), 1e-30)),
              "rows_checked": int(len(rows) * 3 * world), "oracle": "O.gqa_attention_rows over the global sequence",
              "bars": {"max_abs": 2e-2, "mean_rel": 1e-2}}
    parity["ok"] = parity["max_abs"] <= 2e-2 and parity["mean_rel"] <= 1e-2

    peak_b = peaks["bf16_tflops"]
    per_gpu = tf / world
    line.update({
        "steps": steps, "warmup": 3, "higher_is_better": True, "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1) per shard, seeded numpy default_rng",
        "config": {"workload": line["config"], "batch": 1, "seq_len": S, "seq_per_rank": Sl, "heads_q": Hq,
                   "heads_kv": Hkv, "head_dim": D, "mask": "causal_mod()",
                   "parallelism": f"sequence-parallel ring x{world} (zig-zag chunks, NCCL send/recv of K/V)",
                   "l2": "inputs larger than L2 (q shard >= 128 MiB)"},
        "roofline": {"kernel": "attn_ring_fwd: fwd2::flash_fwd2_kernel<128,bf16> per chunk pair, LSE merge in its epilogue",
                     "bound": "tensor", "achieved": round(per_gpu, 2), "peak": peak_b, "unit": "TFLOP/s",
                     "frac": round(per_gpu / peak_b, 4), "traffic": None,
                     "algorithmic_per_step_per_gpu": fl / world},
        "e2e": {"value": round(S / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": nbytes((hq, hk, hv)) * world, "d2h_bytes_per_step": nbytes(host_out) * world,
                "returned": "every rank's output shard to pinned host memory every step"},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "parity": parity,
        "peaks_source": PEAKS_SRC,
    })
    if base:
        line["scaling_efficiency_vs_one_gpu_at_shard_len"] = round(per_gpu / base, 4)
    return line


def run_fp32(args, torch, peaks):
    import attnax_b200 as ax
    from attnax_b200._spec import build_spec
    from attnax_b200.flash import fwd_raw

    B, H, S, D = 2, 8, 1024, 64
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(5)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device=dev) for _ in range(3))
    spec = build_spec(ax.causal_mod(), None, batch=B, heads_q=H, seq_q=S, seq_kv=S, device=dev)
    out = torch.empty_like(q)
    tm = Timer(torch, None, 1)
    ms, _ = tm.run(lambda m: fwd_raw(q, k, v, spec, out=out, want_lse=False), args.steps * 5, args.warmup)
    fl = 4.0 * D * H * B * S * (S + 1) // 2
    return {"metric": "fp32 causal flash fwd TFLOP/s (CUDA-core FFMA)", "value": round(fl / (ms * 1e-3) / 1e12, 3),
            "unit": "TFLOP/s", "ms_per_step": round(ms, 4), "config": f"B{B} H{H} S{S} D{D} fp32 causal"}


# ----------------------------------------------------------- CPU baseline --

def cpu_sample_flash(kind):
    """Bounded sample of the flash workload for the oracle on host cores.

    "baseline" (beside our line, ~15 s): 2 heads at S=4096;
    "arm" (one step of --impl reference, ~2 s): 1 head at S=2048.
    """
    c = flash_cfg("full")
    if kind == "baseline":
        return dict(S=4096, D=c["D"], W=c["W"], heads=2, Hq=c["Hq"])
    return dict(S=2048, D=c["D"], W=c["W"], heads=1, Hq=c["Hq"])


def run_cpu_flash(kind, reps=1):
    import oracle as O

    sm = cpu_sample_flash(kind)
    S, D, W, nh, Hq = sm["S"], sm["D"], sm["W"], sm["heads"], sm["Hq"]
    rng = np.random.default_rng(0)
    q = O.bf16_round(rng.standard_normal((1, nh, S, D), dtype=np.float32))
    k = O.bf16_round(rng.standard_normal((1, nh, S, D), dtype=np.float32))
    v = O.bf16_round(rng.standard_normal((1, nh, S, D), dtype=np.float32))
    do = O.bf16_round(rng.standard_normal((1, nh, S, D), dtype=np.float32))

    sl = O.alibi_slopes(Hq)[:nh]  # ALiBi of the first `nh` heads of a Hq-head model

    def alibi(scores, b, h, qi, kvi):
        dt = scores.dtype
        return scores - sl.astype(dt)[None, :, None, None] * np.abs(qi.astype(dt) - kvi.astype(dt))

    mod = O.compose_score_mods(O.sliding_window_mod(W), alibi)
    t0 = time.perf_counter()
    for _ in range(reps):
        O.memory_efficient_attention(q, k, v, score_mod=mod, block_size=512)
        O.standard_attention_bwd(q, k, v, do, score_mod=mod)
    dt = (time.perf_counter() - t0) / reps
    pairs = window_pairs(S, W)
    fl = 3.5 * 4.0 * D * nh * pairs
    return fl / dt / 1e12, dt, f"fwd (memory_efficient_attention) + bwd (closed form) of {nh} heads at S={S}, window {W}+ALiBi, fp32 on bf16 values"


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count()


def run_cpu_ring(world, S_sample=2048):
    """The oracle's ring recurrence (the reference's per-shard scan, every
    block computed) over ``world`` shards of a 1-head causal sample; returns
    algorithmic FLOP/s and the seconds it took."""
    import oracle as O

    rng = np.random.default_rng(0)
    q, k, v = (O.bf16_round(rng.standard_normal((1, 1, S_sample, RING["D"]), dtype=np.float32)) for _ in range(3))
    t0 = time.perf_counter()
    O.ring_attention_partitioned(q, k, v, world, score_mod=O.causal_mod())
    dt = time.perf_counter() - t0
    return 4.0 * RING["D"] * S_sample * (S_sample + 1) / 2 / dt, dt


def reference_line(args, world):
    """``--impl reference``: the CPU restatement of the reference on this
    host's cores, on bounded samples of the workload our arm reports at this
    N (the flash step at N=1, the ring at N>1), in the same metric."""
    common = {"impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
              "higher_is_better": True, "vs_baseline": None, "dtype": "f32",
              "data": "synthetic N(0,1), seeded numpy default_rng"}
    if world > 1 and args.workload in ("default", "ring"):
        S = RING["S"] if args.scale == "full" else 16384
        run_cpu_ring(world, 512)  # untimed warm-up
        per = [run_cpu_ring(world) for _ in range(args.steps)]
        rate = statistics.median(x[0] for x in per)
        full = 4.0 * RING["D"] * RING["Hq"] * S * (S + 1) / 2
        v = S / (full / rate)
        sample = (f"oracle ring_attention_partitioned over {world} shards, 1 head, S=2048 causal, D=128, fp32; "
                  f"tokens/s of the full config at the sample's algorithmic FLOP rate")
        line = dict(common, metric="ring attention tokens/s", value=round(v, 4), unit="tokens/s",
                    ms_per_step=round(statistics.median(x[1] for x in per) * 1e3, 2), scaling="strong",
                    config={"workload": f"B1 S{S} (S/P={S // world}) Hq{RING['Hq']} Hkv{RING['Hkv']} "
                                        f"D{RING['D']} bf16 causal, zig-zag ring over NCCL"})
        unit = "tokens/s"
    else:
        run_cpu_flash("arm")  # one untimed warm-up sample
        per = [run_cpu_flash("arm") for _ in range(args.steps)]
        v = statistics.median(x[0] for x in per)
        sample = per[0][2]
        c = flash_cfg(args.scale)
        line = dict(common, metric="flash attention fwd+bwd TFLOP/s (algorithmic)", value=round(v, 5),
                    unit="TFLOP/s", ms_per_step=round(statistics.median(x[1] for x in per) * 1e3, 2),
                    scaling="weak",
                    config={"workload": f"flash fwd+bwd B{c['B']} Hq{c['Hq']} Hkv{c['Hkv']} S{c['S']} D{c['D']} "
                                        f"sliding_window({c['W']})+alibi({c['Hq']})"})
        unit = "TFLOP/s"
    line["cpu_baseline"] = {"value": line["value"], "unit": unit, "cores": cpu_cores(), "kind": "port",
                            "sample": sample}
    line["e2e"] = {"value": line["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    return line


# -------------------------------------------------------------------- main --

PEAKS_SRC = "measured"


def main():
    global PEAKS_SRC
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["default", "flash", "paged", "kv_cache", "document", "fp32", "ring"],
                    default="default")
    ap.add_argument("--scale", choices=["full", "small"], default="full")
    ap.add_argument("--no-secondary", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    peaks, PEAKS_SRC = load_peaks()

    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(reference_line(args, world)))
        return 0

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        if args.workload == "default" and world > 1:
            # Multi-GPU headline: the sequence-parallel ring (strong scaling).
            line = run_ring(args, torch, dist, rank, world, peaks, headline=True)
            if not args.no_secondary:
                fl = run_flash(args, torch, dist, rank, world, peaks)
                if rank == 0:
                    line["secondary"] = {"flash_replicas": {k: fl[k] for k in (
                        "metric", "value", "unit", "ms_per_step", "fwd_tflops", "bwd_tflops", "scaling", "config")}}
        elif args.workload in ("default", "flash"):
            line = run_flash(args, torch, dist, rank, world, peaks)
            if rank == 0 and world == 1:
                v, dt, sample = run_cpu_flash("baseline")
                line["cpu_baseline"] = {"value": round(v, 5), "unit": "TFLOP/s", "cores": cpu_cores(),
                                        "kind": "port", "sample": sample, "seconds": round(dt, 2)}
            if world == 1 and not args.no_secondary:
                line["secondary"] = {"ring": run_ring(args, torch, dist, rank, world, peaks),
                                     "paged": run_paged(args, torch, peaks),
                                     "kv_cache": run_kv_cache(args, torch, peaks),
                                     "document": run_document(args, torch, peaks),
                                     "fp32": run_fp32(args, torch, peaks)}
            if world > 1:
                dist.barrier()
        elif args.workload == "paged":
            line = run_paged(args, torch, peaks)
        elif args.workload == "kv_cache":
            line = run_kv_cache(args, torch, peaks)
        elif args.workload == "document":
            line = run_document(args, torch, peaks)
        elif args.workload == "ring":
            line = run_ring(args, torch, dist, rank, world, peaks, headline=world > 1)
        else:
            line = run_fp32(args, torch, peaks)
        if rank == 0:
            print(json.dumps(line))
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
