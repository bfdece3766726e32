"""The allocation-free paged decode (attn_paged_decode_static) against the regular one.

attn_paged_decode_static is for callers that cannot allocate device memory
(code running under CUDA graph capture, serving loops whose allocator forbids
cudaMalloc on the hot path, fixed-budget embedders): its split partials live
in an 8 MiB array inside the library instead of a caller workspace.  Both
entry points are called through the C ABI on the same inputs and must agree
within the bf16 tolerance, twice in a row (the array keeps the previous
call's contents).  This file sorts last so a run stopped at its first failure
has already run every other test.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from attnax_b200 import _lib
from tests._util import BF16_MAX_ABS, BF16_MEAN_REL, errors

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _cache(rng, lens, hkv, bs=16, D=128):
    pages = [(n + bs - 1) // bs for n in lens]
    nb = sum(pages) + 3
    perm = rng.permutation(nb)
    table = np.full((len(lens), max(max(pages), 1)), -1, np.int32)
    o = 0
    for s, n in enumerate(pages):
        table[s, :n] = perm[o:o + n]
        o += n
    kp = torch.randn(nb, bs, hkv, D, device=DEV).to(torch.bfloat16)
    vp = torch.randn(nb, bs, hkv, D, device=DEV).to(torch.bfloat16)
    return kp, vp, torch.tensor(table, device=DEV), torch.tensor(lens, dtype=torch.int32, device=DEV)


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


def test_static_decode_matches_workspace_decode_twice():
    lib = _lib.load()
    rng = np.random.default_rng(21)
    torch.manual_seed(21)
    lens = [0, 1, 17, 700, 2048, 2049, 9000]
    kp, vp, table, tl = _cache(rng, lens, 8)
    for call in range(2):
        q = torch.randn(len(lens), 32, 1, 128, device=DEV).to(torch.bfloat16)
        want = torch.empty_like(q)
        p = _params(q, kp, vp, table, tl, want, max(lens))
        ws = torch.empty(lib.attn_paged_decode_workspace_size(C.byref(p)), dtype=torch.uint8, device=DEV)
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
        _lib.check(lib.attn_paged_decode(C.byref(p), _stream()), "attn_paged_decode")
        got = torch.full_like(q, float("nan"))
        p2 = _params(q, kp, vp, table, tl, got, max(lens))
        _lib.check(lib.attn_paged_decode_static(C.byref(p2), _stream()), "attn_paged_decode_static")
        torch.cuda.synchronize()
        mx, rel = errors(got.float().cpu().numpy(), want.float().cpu().numpy())
        assert mx <= BF16_MAX_ABS and rel <= BF16_MEAN_REL, f"call {call}: max-abs {mx:.3e} rel {rel:.3e}"


def test_static_decode_fewer_splits_when_the_array_is_tight():
    """16 sequences x 128 heads (2048 rows) with 15-20K contexts need more splits than fit."""
    lib = _lib.load()
    rng = np.random.default_rng(22)
    torch.manual_seed(22)
    lens = [int(x) for x in rng.integers(15000, 20001, size=16)]
    kp, vp, table, tl = _cache(rng, lens, 16)
    q = torch.randn(16, 128, 1, 128, device=DEV).to(torch.bfloat16)
    want = torch.empty_like(q)
    p = _params(q, kp, vp, table, tl, want, max(lens))
    ws = torch.empty(lib.attn_paged_decode_workspace_size(C.byref(p)), dtype=torch.uint8, device=DEV)
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.attn_paged_decode(C.byref(p), _stream()), "attn_paged_decode")
    got = torch.empty_like(q)
    _lib.check(lib.attn_paged_decode_static(C.byref(_params(q, kp, vp, table, tl, got, max(lens))), _stream()),
               "attn_paged_decode_static")
    torch.cuda.synchronize()
    mx, rel = errors(got.float().cpu().numpy(), want.float().cpu().numpy())
    assert mx <= BF16_MAX_ABS and rel <= BF16_MEAN_REL, f"max-abs {mx:.3e} rel {rel:.3e}"


def test_static_decode_rejects_requests_beyond_the_array():
    lib = _lib.load()
    rng = np.random.default_rng(23)
    kp, vp, table, tl = _cache(rng, [40] * 200, 8)
    q = torch.zeros(200, 128, 1, 128, device=DEV, dtype=torch.bfloat16)   # 25600 rows > 16256
    out = torch.empty_like(q)
    rc = lib.attn_paged_decode_static(C.byref(_params(q, kp, vp, table, tl, out, 40)), _stream())
    assert rc == _lib.ATTN_ERR_WORKSPACE
