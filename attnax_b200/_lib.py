"""ctypes binding of ``libattnb200.so`` (the C ABI in ``include/attnb200.h``).

The library is built in-tree (``attnax_b200/libattnb200.so``); there is no
fallback: if it is missing or fails to load, every kernel call raises.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libattnb200.so")

ATTN_OK, ATTN_ERR_INVALID, ATTN_ERR_UNSUPPORTED, ATTN_ERR_CUDA, ATTN_ERR_NCCL, \
    ATTN_ERR_WORKSPACE, ATTN_ERR_TIMEOUT = range(7)
ATTN_F32, ATTN_BF16, ATTN_F16 = 0, 1, 2
# Device status codes (attn_device_status): bounded-wait timeouts and notices.
STATUS_TIMEOUTS = (0x101, 0x102, 0x103, 0x104)
NOTICE_CONTEXT_OVERRUN = 0x201   # a paged decode met a length above max_context
NOTICE_TABLE_OVERRUN = 0x202     # a paged decode met a length past its block-table row

i32, i64, f32, vp, szt = C.c_int32, C.c_int64, C.c_float, C.c_void_p, C.c_size_t


class AttnMask(C.Structure):
    _fields_ = [
        ("has_band", i32), ("band_lo", i64), ("band_hi", i64),
        ("prefix_len", vp), ("doc_q", vp), ("doc_kv", vp),
        ("doc_q_bstride", i64), ("doc_kv_bstride", i64),
        ("alibi_slopes", vp), ("bias", vp), ("bias_dtype", C.c_int),
        ("bias_strides", i64 * 4), ("bool_mask", vp), ("mask_strides", i64 * 4),
        ("q_offset", i64), ("kv_offset", i64),
    ]


class FwdParams(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("batch", i32), ("num_heads_q", i32), ("num_heads_kv", i32),
        ("seq_q", i32), ("seq_kv", i32), ("head_dim", i32),
        ("q", vp), ("k", vp), ("v", vp), ("out", vp),
        ("q_strides", i64 * 3), ("k_strides", i64 * 3), ("v_strides", i64 * 3),
        ("o_strides", i64 * 3), ("lse", vp), ("softmax_scale", f32),
        ("fix_masked_rows", i32), ("mask", AttnMask), ("workspace", vp),
        ("workspace_bytes", szt),
    ]


class BwdParams(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("batch", i32), ("num_heads_q", i32), ("num_heads_kv", i32),
        ("seq_q", i32), ("seq_kv", i32), ("head_dim", i32),
        ("q", vp), ("k", vp), ("v", vp), ("out", vp), ("d_out", vp), ("lse", vp),
        ("dq", vp), ("dk", vp), ("dv", vp),
        ("q_strides", i64 * 3), ("k_strides", i64 * 3), ("v_strides", i64 * 3),
        ("o_strides", i64 * 3), ("do_strides", i64 * 3), ("dq_strides", i64 * 3),
        ("dk_strides", i64 * 3), ("dv_strides", i64 * 3), ("softmax_scale", f32),
        ("fix_masked_rows", i32), ("mask", AttnMask), ("workspace", vp),
        ("workspace_bytes", szt),
    ]


class PagedParams(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("num_seqs", i32), ("num_heads_q", i32), ("num_heads_kv", i32),
        ("head_dim", i32), ("seq_q", i32), ("num_blocks", i32), ("block_size", i32),
        ("max_blocks_per_seq", i32), ("max_context", i32),
        ("q", vp), ("key_pool", vp), ("value_pool", vp), ("block_table", vp),
        ("seq_lengths", vp), ("out", vp), ("softmax_scale", f32),
        ("workspace", vp), ("workspace_bytes", szt),
    ]


class RopeParams(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("batch", i32), ("heads", i32), ("seq", i32), ("head_dim", i32),
        ("x_strides", i64 * 3), ("out_strides", i64 * 3),
        ("x", vp), ("out", vp), ("cos", vp), ("sin", vp), ("table_len", i32), ("positions", vp),
    ]


class RingParams(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("batch", i32), ("num_heads_q", i32), ("num_heads_kv", i32),
        ("seq_local", i32), ("head_dim", i32), ("q", vp), ("k", vp), ("v", vp), ("out", vp),
        ("lse", vp), ("softmax_scale", f32), ("has_band", i32), ("band_lo", i64), ("band_hi", i64),
        ("alibi_slopes", vp), ("zigzag", i32), ("workspace", vp), ("workspace_bytes", szt),
    ]


class RingBwdParams(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("batch", i32), ("num_heads_q", i32), ("num_heads_kv", i32),
        ("seq_local", i32), ("head_dim", i32), ("q", vp), ("k", vp), ("v", vp), ("out", vp),
        ("lse", vp), ("d_out", vp), ("dq", vp), ("dk", vp), ("dv", vp), ("softmax_scale", f32),
        ("has_band", i32), ("band_lo", i64), ("band_hi", i64), ("alibi_slopes", vp), ("zigzag", i32),
        ("workspace", vp), ("workspace_bytes", szt),
    ]


COMM_ID_BYTES = 128
RING_PLAN_FIELDS = ("hop", "q_slot", "q_chunks", "kv_slot", "kv_chunks", "q_start", "kv_start", "masked",
                    "final_from", "local")

# Every symbol the header declares, with its ctypes signature.
SIGNATURES = {
    "attn_fwd_workspace_size": (szt, [C.POINTER(FwdParams)]),
    "attn_fwd": (C.c_int, [C.POINTER(FwdParams), vp]),
    "attn_bwd_workspace_size": (szt, [C.POINTER(BwdParams)]),
    "attn_bwd": (C.c_int, [C.POINTER(BwdParams), vp]),
    "attn_paged_decode_workspace_size": (szt, [C.POINTER(PagedParams)]),
    "attn_paged_decode": (C.c_int, [C.POINTER(PagedParams), vp]),
    "attn_paged_decode_static": (C.c_int, [C.POINTER(PagedParams), vp]),
    "attn_paged_gather": (C.c_int, [C.c_int, vp, vp, i32, i32, i32, i32, vp, i32, i32, vp, vp, vp]),
    "attn_paged_append": (C.c_int, [C.c_int, vp, vp, i32, i32, i32, i32, vp, i32, i32, i32, vp, vp, vp, vp]),
    "attn_paged_physical_page": (i64, [i32, i32]),
    "attn_lse_merge": (C.c_int, [C.c_int, i64, i32, vp, vp, vp, vp, vp, vp]),
    "attn_rope": (C.c_int, [C.POINTER(RopeParams), vp]),
    "attn_comm_unique_id": (C.c_int, [vp, szt]),
    "attn_comm_init": (C.c_int, [C.POINTER(vp), i32, i32, vp, szt]),
    "attn_comm_destroy": (C.c_int, [vp]),
    "attn_ring_plan": (C.c_int, [i32, i32, i32, i32, i32, i64, i64, i32, C.POINTER(i64), i32]),
    "attn_ring_fwd_workspace_size": (szt, [C.POINTER(RingParams), i32]),
    "attn_ring_fwd": (C.c_int, [C.POINTER(RingParams), vp, vp, vp]),
    "attn_ring_bwd_workspace_size": (szt, [C.POINTER(RingBwdParams), i32]),
    "attn_ring_bwd": (C.c_int, [C.POINTER(RingBwdParams), vp, vp, vp]),
    "attn_device_status": (C.c_int, [C.POINTER(i32)]),
    "attn_status_string": (C.c_char_p, [C.c_int]),
    "attn_version": (C.c_int, []),
    "attn_launch_count": (C.c_uint64, []),
}

_lock = threading.Lock()
_lib = None


def load():
    """Loads the library once; raises ``RuntimeError`` if it is not built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"attnax_b200 CUDA library not built ({LIB_PATH}); run "
                    "`python -c 'import __graft_entry__ as g; g.build()'` or `make -C attnax_b200/csrc`")
            lib = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


class KernelError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def check(status: int, what: str):
    if status == ATTN_OK:
        return
    msg = load().attn_status_string(status).decode()
    if status == ATTN_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    if status == ATTN_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise KernelError(f"{what}: {msg} (status {status})")


def device_status() -> int:
    """Reads and clears the device status word (non-zero after a timed-out wait)."""
    v = i32(0)
    check(load().attn_device_status(C.byref(v)), "attn_device_status")
    return int(v.value)
