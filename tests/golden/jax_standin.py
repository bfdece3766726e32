"""A numpy stand-in for the few ``jax``/``flax`` names attnax's hot path calls.

JAX is not installed where the golden vectors are made, so
``make_golden.py`` installs these modules under the names ``jax``,
``jax.numpy``, ``jax.lax``, ``jax.nn``, ``jax.random``, ``flax`` and
``flax.nnx`` and then imports the reference's own, unmodified source files.
Only what those files touch is provided: array creation with JAX's 32-bit
defaults, ``einsum``/``where``/reductions, ``x.at[i].set/add``,
``jax.nn.softmax``, ``jax.lax.rsqrt``/``scan``, and a thread-based emulation
of a named device axis (``axis_size``/``axis_index``/``ppermute``) so that
``ring_attention`` runs with a bound axis.  Anything else raises.
"""

from __future__ import annotations

import sys
import threading
import types

import numpy as np


class Array(np.ndarray):
    """ndarray with JAX's functional ``.at[idx].set/add`` update syntax."""

    @property
    def at(self):
        return _At(self)


class _At:
    def __init__(self, a):
        self._a = a

    def __getitem__(self, idx):
        return _AtIndex(self._a, idx)


class _AtIndex:
    def __init__(self, a, idx):
        self._a, self._idx = a, idx

    def set(self, v):
        out = np.array(self._a, copy=True).view(Array)
        out[self._idx] = np.asarray(v)
        return out

    def add(self, v):
        out = np.array(self._a, copy=True).view(Array)
        out[self._idx] += np.asarray(v)
        return out


def _w(x):
    if isinstance(x, np.ndarray):
        return x.view(Array)
    return x


def _default_dtype(x, dtype):
    if dtype is not None:
        return np.dtype(dtype)
    a = np.asarray(x)
    if a.dtype == np.float64:
        return np.dtype(np.float32)
    if a.dtype == np.int64:
        return np.dtype(np.int32)
    return a.dtype


def _wrap_fn(fn):
    def inner(*a, **k):
        return _w(fn(*a, **k))
    inner.__name__ = getattr(fn, "__name__", "fn")
    return inner


def _make_jnp():
    m = types.ModuleType("jax.numpy")
    m.ndarray = np.ndarray
    m.float32, m.float16, m.int32, m.bool_ = np.float32, np.float16, np.int32, np.bool_
    m.dtype = np.dtype
    m.finfo = np.finfo
    for name in ("where", "transpose", "sum", "exp", "broadcast_to", "maximum", "max",
                 "abs", "tril", "repeat", "concatenate", "minimum", "outer", "cos", "sin"):
        setattr(m, name, _wrap_fn(getattr(np, name)))
    m.einsum = lambda spec, *ops: _w(np.einsum(spec, *ops, optimize=True))
    m.dot = lambda a, b: _w(np.dot(a, b))

    def asarray(x, dtype=None):
        return _w(np.asarray(x, dtype=_default_dtype(x, dtype)))

    def arange(*args, dtype=None):
        return _w(np.arange(*args, dtype=dtype or np.int32))

    def zeros(shape, dtype=None):
        return _w(np.zeros(shape, dtype=dtype or np.float32))

    def ones(shape, dtype=None):
        return _w(np.ones(shape, dtype=dtype or np.float32))

    def full(shape, fill, dtype=None):
        return _w(np.full(shape, fill, dtype=dtype or np.float32))

    m.asarray, m.array, m.arange, m.zeros, m.ones, m.full = asarray, asarray, arange, zeros, ones, full
    m.zeros_like = lambda x, dtype=None: _w(np.zeros_like(x, dtype=dtype))
    m.ones_like = lambda x, dtype=None: _w(np.ones_like(x, dtype=dtype))
    return m


class _AxisEnv(threading.local):
    """Per-thread binding of a named axis: (name, size, index, exchange)."""

    binding = None


_AXIS = _AxisEnv()


class RingExchange:
    """Shared mailbox + barrier that plays the role of a device ring."""

    def __init__(self, size):
        self.size = size
        self.slots = [None] * size
        self.barrier = threading.Barrier(size)


def _make_lax():
    m = types.ModuleType("jax.lax")
    m.rsqrt = lambda x: _w(np.asarray(1.0, dtype=np.asarray(x).dtype) / np.sqrt(x))

    def scan(f, init, xs):
        carry, ys = init, []
        for x in xs:
            carry, y = f(carry, x)
            ys.append(y)
        if all(y is None for y in ys):
            return carry, None
        return carry, _w(np.stack(ys))

    def fori_loop(lo, hi, body, init):
        val = init
        for i in range(lo, hi):
            val = body(i, val)
        return val

    def _binding(name):
        b = _AXIS.binding
        if b is None or b[0] != name:
            raise NameError(f"unbound axis name: {name}")
        return b

    def axis_size(name):
        return _binding(name)[1]

    def axis_index(name):
        return np.int32(_binding(name)[2])

    def ppermute(x, axis_name, perm):
        _, size, idx, ex = _binding(axis_name)
        dest = dict(perm)[idx]
        ex.barrier.wait()
        ex.slots[dest] = np.array(x, copy=True)
        ex.barrier.wait()
        got = ex.slots[idx]
        ex.barrier.wait()
        return _w(got)

    m.scan, m.fori_loop, m.axis_size, m.axis_index, m.ppermute = (
        scan, fori_loop, axis_size, axis_index, ppermute)
    return m


def run_on_ring(fn, per_rank_args, axis_name):
    """Runs ``fn(*args_r)`` on one thread per rank with ``axis_name`` bound."""
    size = len(per_rank_args)
    ex = RingExchange(size)
    out = [None] * size
    err = []

    def worker(r):
        _AXIS.binding = (axis_name, size, r, ex)
        try:
            out[r] = fn(*per_rank_args[r])
        except BaseException as e:  # surface worker failures in the caller
            err.append(e)
            ex.barrier.abort()

    threads = [threading.Thread(target=worker, args=(r,)) for r in range(size)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if err:
        raise err[0]
    return out


def _make_nn():
    m = types.ModuleType("jax.nn")

    def softmax(x, axis=-1):
        e = np.exp(x - np.max(x, axis=axis, keepdims=True))
        return _w(e / np.sum(e, axis=axis, keepdims=True))

    m.softmax = softmax
    m.elu = lambda x: _w(np.where(x > 0, x, np.expm1(x)))
    return m


def install():
    """Registers the stand-in modules in ``sys.modules``."""
    jax = types.ModuleType("jax")
    jax.numpy = _make_jnp()
    jax.lax = _make_lax()
    jax.nn = _make_nn()
    jax.random = types.ModuleType("jax.random")
    jax.Array = np.ndarray
    jax.default_backend = lambda: "cpu"
    flax = types.ModuleType("flax")
    nnx = types.ModuleType("flax.nnx")

    class _Stub:
        def __init__(self, *a, **k):
            raise NotImplementedError("flax is not available in the stand-in")

    nnx.Linear = nnx.Module = nnx.Rngs = _Stub
    flax.nnx = nnx
    sys.modules.update({"jax": jax, "jax.numpy": jax.numpy, "jax.lax": jax.lax,
                        "jax.nn": jax.nn, "jax.random": jax.random,
                        "flax": flax, "flax.nnx": nnx})


def as_array(x):
    """Wraps a numpy array as the stand-in's array type."""
    return _w(np.asarray(x))
