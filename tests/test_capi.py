"""The C-ABI library loads and exports every symbol the public header declares (no GPU)."""

import ctypes
import pathlib
import re

import pytest

from attnax_b200 import _lib

ROOT = pathlib.Path(__file__).resolve().parent.parent


def header_functions():
    text = (ROOT / "include" / "attnb200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(attn_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    names = header_functions()
    for n in ("attn_fwd", "attn_bwd", "attn_paged_decode", "attn_paged_gather", "attn_paged_append",
              "attn_lse_merge"):
        assert n in names


def test_library_loads_and_exports_every_header_symbol():
    if not pathlib.Path(_lib.LIB_PATH).exists():
        pytest.fail("libattnb200.so is not built; run __graft_entry__.build()")
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for n in header_functions():
        assert hasattr(lib, n), f"{n} missing from {_lib.LIB_PATH}"
    assert set(header_functions()) == set(_lib.SIGNATURES), "ctypes signatures out of sync with header"
    assert _lib.load().attn_version() >= 1
    assert _lib.load().attn_status_string(2) == b"unsupported configuration"


def test_struct_sizes_are_stable():
    # The ctypes mirrors must match the C layout the library was compiled with.
    assert ctypes.sizeof(_lib.AttnMask) % 8 == 0
    assert ctypes.sizeof(_lib.FwdParams) > ctypes.sizeof(_lib.AttnMask)


def test_ctypes_layout_matches_c_compiler(tmp_path):
    """Offsets and sizes of the ctypes mirrors equal what gcc computes from the header."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    structs = {"attn_mask_t": _lib.AttnMask, "attn_fwd_params_t": _lib.FwdParams,
               "attn_bwd_params_t": _lib.BwdParams, "attn_paged_params_t": _lib.PagedParams,
               "attn_rope_params_t": _lib.RopeParams, "attn_ring_params_t": _lib.RingParams,
               "attn_ring_bwd_params_t": _lib.RingBwdParams}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{ROOT}/include/attnb200.h"',
             "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                 check=True).stdout.splitlines())
    for cname, py in structs.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(py, fname).offset, f"{cname}.{fname}"


def test_block_table_entries_are_read_like_jax_indexing():
    """The page rule shared by the gather, append and decode kernels (host copy
    of the same inline function): a negative entry counts from the end of the
    pool, then the index is clamped into the pool -- what JAX's pool[block_ids]
    does in the reference's gather_kv (attnax/paged_cache.py:222-230)."""
    if not pathlib.Path(_lib.LIB_PATH).exists():
        pytest.fail("libattnb200.so is not built; run __graft_entry__.build()")
    page = _lib.load().attn_paged_physical_page
    nb = 10
    for entry, want in [(0, 0), (5, 5), (9, 9), (10, 9), (2**31 - 1, 9), (-1, 9), (-10, 0), (-11, 0),
                        (-(2**31), 0)]:
        assert page(entry, nb) == want, entry
    assert page(3, 0) == -1


def test_ring_communicator_entry_points_validate_and_fail_cleanly():
    """attn_comm_*: a unique id is 128 opaque bytes made without a GPU; bad
    arguments are ATTN_ERR_INVALID; without a GPU, init reports an error and
    hands back no communicator (the GPU path runs in tests/test_ring_gpu.py)."""
    import torch

    if not pathlib.Path(_lib.LIB_PATH).exists():
        pytest.fail("libattnb200.so is not built; run __graft_entry__.build()")
    lib = _lib.load()
    raw = (ctypes.c_char * _lib.COMM_ID_BYTES)()
    rc = lib.attn_comm_unique_id(raw, _lib.COMM_ID_BYTES)
    if rc == _lib.ATTN_ERR_NCCL:
        pytest.skip("NCCL is not installed on this host")
    assert rc == _lib.ATTN_OK and any(raw.raw)
    assert lib.attn_comm_unique_id(raw, 16) == _lib.ATTN_ERR_INVALID
    c = ctypes.c_void_p()
    assert lib.attn_comm_init(ctypes.byref(c), 2, 5, raw, _lib.COMM_ID_BYTES) == _lib.ATTN_ERR_INVALID
    assert lib.attn_comm_init(ctypes.byref(c), 1, 0, raw, 8) == _lib.ATTN_ERR_INVALID
    assert lib.attn_comm_destroy(None) == _lib.ATTN_ERR_INVALID
    if not torch.cuda.is_available():
        assert lib.attn_comm_init(ctypes.byref(c), 1, 0, raw, _lib.COMM_ID_BYTES) != _lib.ATTN_OK
        assert c.value is None
    p = _lib.RingParams()
    assert lib.attn_ring_fwd(ctypes.byref(p), None, None, None) == _lib.ATTN_ERR_INVALID
