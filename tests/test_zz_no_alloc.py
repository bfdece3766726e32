"""The allocation-free paged decode (attn_paged_decode_static) against the regular one and the oracle.

attn_paged_decode_static serves callers that cannot allocate device memory
for a workspace -- serving loops whose allocator forbids cudaMalloc on the
decode path (it synchronises the device), embedders running inside a fixed
device-memory budget, plugin hosts that hand a kernel only its inputs and
outputs.  Its split partials live in an 8 MiB array inside the library
instead of a caller workspace.  Both entry points are called through the C
ABI on the same inputs; the static one must match the workspace one within
the bf16 tolerance, twice in a row (the array keeps the previous call's
contents), and the oracle's paged_attention as well.  This file sorts last
so a run stopped at its first failure has already run every other test.
"""

import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from attnax_b200 import _lib
from tests._util import BF16_MAX_ABS, BF16_MEAN_REL, assert_bf16_close, errors

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _cache(rng, lens, hkv, bs=16, D=128, nan_tail=False):
    """Random bf16 pools and a permuted block table; with ``nan_tail`` the
    unused slots of each sequence's last page hold NaN (never written)."""
    pages = [(n + bs - 1) // bs for n in lens]
    nb = sum(pages) + 3
    perm = rng.permutation(nb)
    table = np.full((len(lens), max(max(pages), 1)), -1, np.int32)
    o = 0
    for s, n in enumerate(pages):
        table[s, :n] = perm[o:o + n]
        o += n
    kp = O.bf16_round(rng.standard_normal((nb, bs, hkv, D), dtype=np.float32))
    vp = O.bf16_round(rng.standard_normal((nb, bs, hkv, D), dtype=np.float32))
    okp, ovp = kp.copy(), vp.copy()
    if nan_tail:
        for s, n in enumerate(lens):
            if n % bs:
                kp[table[s, (n - 1) // bs], n % bs:] = np.nan
                vp[table[s, (n - 1) // bs], n % bs:] = np.nan
    oc = O.PagedKVCache(okp, ovp, table, np.array(lens, np.int32))
    t = (torch.tensor(kp, device=DEV).to(torch.bfloat16), torch.tensor(vp, device=DEV).to(torch.bfloat16),
         torch.tensor(table, device=DEV), torch.tensor(lens, dtype=torch.int32, device=DEV))
    return t, oc


def _params(q, kp, vp, table, lens, out, max_context):
    p = _lib.PagedParams()
    p.dtype = _lib.ATTN_BF16
    p.num_seqs, p.num_heads_q, p.seq_q, p.head_dim = q.shape[0], q.shape[1], q.shape[2], q.shape[3]
    p.num_heads_kv = kp.shape[2]
    p.num_blocks, p.block_size, p.max_blocks_per_seq = kp.shape[0], kp.shape[1], table.shape[1]
    p.max_context = max_context
    p.q, p.key_pool, p.value_pool = q.data_ptr(), kp.data_ptr(), vp.data_ptr()
    p.block_table, p.seq_lengths, p.out = table.data_ptr(), lens.data_ptr(), out.data_ptr()
    p.softmax_scale = 128 ** -0.5
    return p


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _both(lib, q, cache, max_context):
    """(workspace decode, static decode) outputs for the same inputs."""
    kp, vp, table, tl = cache
    want = torch.empty_like(q)
    p = _params(q, kp, vp, table, tl, want, max_context)
    ws = torch.empty(lib.attn_paged_decode_workspace_size(C.byref(p)), dtype=torch.uint8, device=DEV)
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.attn_paged_decode(C.byref(p), _stream()), "attn_paged_decode")
    got = torch.full_like(q, float("nan"))
    _lib.check(lib.attn_paged_decode_static(C.byref(_params(q, kp, vp, table, tl, got, max_context)), _stream()),
               "attn_paged_decode_static")
    torch.cuda.synchronize()
    return want.float().cpu().numpy(), got.float().cpu().numpy()


def test_static_decode_matches_workspace_decode_and_oracle_twice():
    lib = _lib.load()
    rng = np.random.default_rng(21)
    lens = [0, 1, 17, 700, 2048, 2049, 9000]
    cache, oc = _cache(rng, lens, 8)
    for call in range(2):
        qn = O.bf16_round(rng.standard_normal((len(lens), 32, 1, 128), dtype=np.float32))
        want, got = _both(lib, torch.tensor(qn, device=DEV).to(torch.bfloat16), cache, max(lens))
        mx, rel = errors(got, want)
        assert mx <= BF16_MAX_ABS and rel <= BF16_MEAN_REL, f"call {call}: max-abs {mx:.3e} rel {rel:.3e}"
        assert_bf16_close(got, O.paged_attention_batched(qn, oc), f"call {call} vs oracle")


def test_static_decode_fewer_splits_when_the_array_is_tight():
    """16 sequences x 128 heads (2048 rows) with 15-20K contexts need more splits than fit."""
    lib = _lib.load()
    rng = np.random.default_rng(22)
    lens = [int(x) for x in rng.integers(15000, 20001, size=16)]
    cache, oc = _cache(rng, lens, 16)
    qn = O.bf16_round(rng.standard_normal((16, 128, 1, 128), dtype=np.float32))
    want, got = _both(lib, torch.tensor(qn, device=DEV).to(torch.bfloat16), cache, max(lens))
    mx, rel = errors(got, want)
    assert mx <= BF16_MAX_ABS and rel <= BF16_MEAN_REL, f"max-abs {mx:.3e} rel {rel:.3e}"
    assert_bf16_close(got, O.paged_attention_batched(qn, oc), "tight array vs oracle")


@pytest.mark.parametrize("bs", [8, 12])
def test_static_decode_split_boundary_inside_a_page(bs):
    """Block sizes that are not multiples of 16 take the scalar decode kernel;
    with the split count cut to fit the array, a split's chunk length is not
    a multiple of the block size, so splits begin and end inside pages whose
    unused slots hold NaN."""
    lib = _lib.load()
    rng = np.random.default_rng(23 + bs)
    # 12 sequences x 64 heads x 4 positions = 3072 rows: 5 splits fit where the
    # longest context (12001) needs 6, so each split covers 2401 tokens.
    lens = [int(x) for x in rng.integers(9000, 12000, size=10)] + [bs - 3, 12001]
    cache, oc = _cache(rng, lens, 8, bs=bs, nan_tail=True)
    qn = O.bf16_round(rng.standard_normal((len(lens), 64, 4, 128), dtype=np.float32))
    want, got = _both(lib, torch.tensor(qn, device=DEV).to(torch.bfloat16), cache, max(lens))
    assert np.isfinite(got).all()
    mx, rel = errors(got, want)
    assert mx <= BF16_MAX_ABS and rel <= BF16_MEAN_REL, f"bs={bs}: max-abs {mx:.3e} rel {rel:.3e}"
    assert_bf16_close(got, O.paged_attention_batched(qn, oc), f"bs={bs} vs oracle")


def test_static_decode_rejects_requests_beyond_the_array():
    lib = _lib.load()
    rng = np.random.default_rng(24)
    (kp, vp, table, tl), _ = _cache(rng, [40] * 200, 8)
    q = torch.zeros(200, 128, 1, 128, device=DEV, dtype=torch.bfloat16)   # 25600 rows > 16256
    out = torch.empty_like(q)
    rc = lib.attn_paged_decode_static(C.byref(_params(q, kp, vp, table, tl, out, 40)), _stream())
    assert rc == _lib.ATTN_ERR_WORKSPACE
