"""JAX front-end of the attnb200 kernels: ``jax.ffi`` targets with ``custom_vjp``.

The functions here keep the reference's ``AttentionFn`` signature
(attnax/kernels/_api.py:75-112) so that ``MultiHeadAttention`` can take
``flash_attention`` from this module in place of attnax's.  Forward and
backward are XLA custom calls into ``libattnax_ffi.so`` (``attnax_ffi.cc``),
which forwards to the C ABI of ``libattnb200.so``:

* ``flash_attention`` -- target ``attnb200_fwd``; its VJP is
  ``attnb200_bwd`` on the saved output and LSE (the reference differentiates
  with JAX autodiff);
* ``paged_attention_batched`` -- ``attnb200_paged_decode``;
* ``ring_attention`` -- ``attnb200_ring_fwd`` with the process's ring
  communicator (``make_ring_comm``).

Masks travel as attributes, so the score mods must be the tagged ones of this
module (``causal_mod``, ``sliding_window_mod``, ``alibi_mod`` and
``compose_score_mods`` of those); each is also a plain ``ScoreMod`` with the
reference's semantics.  An untagged callable raises ``NotImplementedError``,
as the kernels have no general score-mod path.

Nothing here runs without jax and jaxlib: the imports are local so the mask
flattening can be checked anywhere.
"""

from __future__ import annotations

import ctypes
import functools
import math
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
FFI_LIB = os.path.join(_HERE, "libattnax_ffi.so")
BAND_INF = 1 << 62


# ------------------------------------------------------------ score mods --
class _Tagged:
    kind = ""

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        raise NotImplementedError


class causal_mod(_Tagged):  # noqa: N801 - the reference's constructor name
    """Keep ``kv <= q`` (attnax/kernels/score_mods.py:84-104)."""

    kind = "causal"

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        import jax.numpy as jnp

        return jnp.where(kv_idx <= q_idx, scores, jnp.finfo(scores.dtype).min)


class sliding_window_mod(_Tagged):  # noqa: N801
    """Window of ``window_size`` (attnax/kernels/score_mods.py:107-145)."""

    kind = "window"

    def __init__(self, window_size: int, *, causal: bool = True):
        if window_size <= 0:
            raise ValueError(f"window_size must be positive, got {window_size}")
        self.window_size, self.causal = int(window_size), bool(causal)

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        import jax.numpy as jnp

        if self.causal:
            keep = (kv_idx <= q_idx) & (q_idx - kv_idx < self.window_size)
        else:
            keep = jnp.abs(q_idx - kv_idx) < self.window_size
        return jnp.where(keep, scores, jnp.finfo(scores.dtype).min)


class alibi_mod(_Tagged):  # noqa: N801
    """``s - slope[h] |q - kv|`` (attnax/kernels/score_mods.py:48-81)."""

    kind = "alibi"

    def __init__(self, num_heads: int):
        self.num_heads = int(num_heads)

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        import jax.numpy as jnp

        slopes = jnp.asarray(alibi_slopes(self.num_heads), scores.dtype)[None, :, None, None]
        return scores - slopes * jnp.abs(q_idx.astype(scores.dtype) - kv_idx.astype(scores.dtype))


class _Composed(_Tagged):
    kind = "compose"

    def __init__(self, mods):
        self.mods = mods

    def __call__(self, scores, b_idx, h_idx, q_idx, kv_idx):
        for m in self.mods:
            scores = m(scores, b_idx, h_idx, q_idx, kv_idx)
        return scores


def compose_score_mods(*score_mods):
    """Left to right, ``None`` skipped, a single mod returned as itself (_api.py:166-196)."""
    active = [m for m in score_mods if m is not None]
    if not active:
        return None
    return active[0] if len(active) == 1 else _Composed(active)


def alibi_slopes(num_heads: int):
    """Per-head slopes (attnax/kernels/score_mods.py:14-45): the published ALiBi schedule."""

    def pow2(n):
        start = 2.0 ** (-(2.0 ** -(math.log2(n) - 3)))
        return [start * start ** i for i in range(n)]

    if num_heads & (num_heads - 1) == 0:
        return pow2(num_heads)
    closest = 2 ** math.floor(math.log2(num_heads))
    return pow2(closest) + pow2(2 * closest)[0::2][: num_heads - closest]


def mask_attrs(score_mod, num_heads):
    """FFI attributes of a tagged mod chain: band (causal / window) and ALiBi."""
    mods = []

    def walk(m):
        if m is None:
            return
        if isinstance(m, _Composed):
            for x in m.mods:
                walk(x)
        elif isinstance(m, _Tagged):
            mods.append(m)
        else:
            raise NotImplementedError(f"score_mod {m!r} is not one of this module's tagged ScoreMods")

    walk(score_mod)
    lo, hi, has, alibi = -BAND_INF, BAND_INF, False, False
    for m in mods:
        if m.kind == "causal":
            lo, has = max(lo, 0), True
        elif m.kind == "window":
            lo = max(lo, 0 if m.causal else -(m.window_size - 1))
            hi, has = min(hi, m.window_size - 1), True
        elif m.kind == "alibi":
            if m.num_heads != num_heads:
                raise ValueError(f"alibi_mod({m.num_heads}) used with {num_heads} query heads")
            if alibi:
                raise NotImplementedError("two alibi_mod terms in one chain")
            alibi = True
    return {"has_band": int(has), "band_lo": int(lo), "band_hi": int(hi), "alibi": bool(alibi)}


# ------------------------------------------------------------- targets --
@functools.lru_cache(maxsize=None)
def _register():
    import jax

    lib = ctypes.cdll.LoadLibrary(FFI_LIB)
    for name, sym in (("attnb200_fwd", "AttnFwd"), ("attnb200_bwd", "AttnBwd"),
                      ("attnb200_paged_decode", "PagedDecode"), ("attnb200_ring_fwd", "RingFwd")):
        jax.ffi.register_ffi_target(name, jax.ffi.pycapsule(getattr(lib, sym)), platform="CUDA")
    return True


def _attrs(attrs, scale):
    import numpy as np

    out = {k: (np.int64(v) if isinstance(v, int) and not isinstance(v, bool) else v) for k, v in attrs.items()}
    out["softmax_scale"] = np.float32(scale)
    return out


def _scale(head_dim):
    import numpy as np

    return float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))


def _fwd_call(q, k, v, attrs):
    import jax
    import jax.numpy as jnp

    _register()
    out_t = jax.ShapeDtypeStruct(q.shape, q.dtype)
    lse_t = jax.ShapeDtypeStruct(q.shape[:3], jnp.float32)
    return jax.ffi.ffi_call("attnb200_fwd", (out_t, lse_t))(q, k, v, **_attrs(attrs, _scale(q.shape[-1])))


def _bwd_call(q, k, v, out, lse, dout, attrs):
    import jax

    _register()
    shapes = tuple(jax.ShapeDtypeStruct(x.shape, x.dtype) for x in (q, k, v))
    return jax.ffi.ffi_call("attnb200_bwd", shapes)(q, k, v, out, lse, dout, **_attrs(attrs, _scale(q.shape[-1])))


def _make_attention():
    import jax

    @functools.partial(jax.custom_vjp, nondiff_argnums=(3,))
    def attend(q, k, v, attrs_key):
        return _fwd_call(q, k, v, dict(attrs_key))[0]

    def fwd(q, k, v, attrs_key):
        out, lse = _fwd_call(q, k, v, dict(attrs_key))
        return out, (q, k, v, out, lse)

    def bwd(attrs_key, res, dout):
        q, k, v, out, lse = res
        return _bwd_call(q, k, v, out, lse, dout, dict(attrs_key))

    attend.defvjp(fwd, bwd)
    return attend


_attend = None


def flash_attention(query, key, value, *, mask=None, score_mod=None, dropout_rng=None, dropout_rate: float = 0.0,
                    deterministic: bool = True, block_size: int = 512):
    """``flash_attention`` (attnax/kernels/attention.py:209-283) on the sm_100a kernels.

    K/V may have fewer heads than Q.  ``mask=`` tensors are not carried by the
    custom call (use the band mods); output dropout follows the reference.
    """
    global _attend
    import jax

    if mask is not None:
        raise NotImplementedError("mask= is not carried by the attnb200 custom call; use the tagged mods")
    if _attend is None:
        _attend = _make_attention()
    attrs = tuple(sorted(mask_attrs(score_mod, query.shape[1]).items()))
    out = _attend(query, key, value, attrs)
    if not deterministic and dropout_rate > 0.0 and dropout_rng is not None:
        keep = jax.random.bernoulli(dropout_rng, 1.0 - dropout_rate, out.shape)
        out = jax.numpy.where(keep, out / (1.0 - dropout_rate), 0.0).astype(out.dtype)
    return out


def paged_attention_batched(query, key_pool, value_pool, block_table, seq_lengths, *, max_context):
    """Decode of every sequence of a PagedKVCache (attnax/kernels/paged.py:17-84), one launch."""
    import jax
    import numpy as np

    _register()
    return jax.ffi.ffi_call("attnb200_paged_decode", jax.ShapeDtypeStruct(query.shape, query.dtype))(
        query, key_pool, value_pool, block_table, seq_lengths, max_context=np.int64(max_context),
        softmax_scale=np.float32(_scale(query.shape[-1])))


def make_ring_comm(world: int, rank: int, exchange_id):
    """This process's ring communicator.  ``exchange_id(bytes_or_None) -> bytes``
    broadcasts rank 0's id (e.g. through jax.distributed's key-value store)."""
    from attnax_b200 import _lib

    lib = _lib.load()
    ident = None
    if rank == 0:
        raw = (ctypes.c_char * _lib.COMM_ID_BYTES)()
        _lib.check(lib.attn_comm_unique_id(raw, _lib.COMM_ID_BYTES), "attn_comm_unique_id")
        ident = raw.raw
    ident = exchange_id(ident)
    comm = ctypes.c_void_p()
    _lib.check(lib.attn_comm_init(ctypes.byref(comm), world, rank, ident, _lib.COMM_ID_BYTES), "attn_comm_init")
    return comm.value


def ring_attention(query, key, value, *, comm, world, score_mod=None, zigzag=None):
    """Forward of ``ring_attention`` (attention.py:540-691) for this process's
    contiguous shard, through the library's ring (``attn_ring_fwd``)."""
    import jax
    import jax.numpy as jnp
    import numpy as np

    _register()
    attrs = mask_attrs(score_mod, query.shape[1])
    if zigzag is None:
        zigzag = attrs["has_band"] and attrs["band_lo"] >= 0 and world > 1 and query.shape[2] % 2 == 0
    out_t = jax.ShapeDtypeStruct(query.shape, query.dtype)
    lse_t = jax.ShapeDtypeStruct(query.shape[:3], jnp.float32)
    out, _ = jax.ffi.ffi_call("attnb200_ring_fwd", (out_t, lse_t))(
        query, key, value, comm=np.int64(comm), world=np.int64(world), zigzag=np.int64(int(bool(zigzag))),
        **_attrs(attrs, _scale(query.shape[-1])))
    return out
