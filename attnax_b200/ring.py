"""Sequence-parallel ring attention (attnax/kernels/attention.py:540-721).

In the reference, ``axis_name`` names a JAX mesh axis bound by
``shard_map``/``pmap``; an unbound name falls back to the local kernel
(:590-616).  Here an axis is a ``torch.distributed`` process group (one
process per GPU) registered under a name with :func:`bind_axis`; unbound
names fall back to the local flash kernel the same way.
"""

from __future__ import annotations

from .flash import attention, _output_dropout

_AXES = {}


def bind_axis(name: str, process_group=None):
    """Binds ``name`` to a process group (the default group when ``None``)."""
    import torch.distributed as dist

    if not dist.is_initialized():
        raise RuntimeError("torch.distributed is not initialised")
    _AXES[name] = process_group if process_group is not None else dist.group.WORLD


def unbind_axis(name: str):
    _AXES.pop(name, None)


def ring_attention(query, key, value, *, mask=None, score_mod=None, dropout_rng=None,
                   dropout_rate: float = 0.0, deterministic: bool = True, axis_name=None,
                   block_size: int = 512):
    """Ring attention over the ranks bound to ``axis_name``; local when unbound."""
    if axis_name is None or axis_name not in _AXES:
        out = attention(query, key, value, mask=mask, score_mod=score_mod)
        return _output_dropout(out, dropout_rng, dropout_rate, deterministic)
    from ._ring_impl import ring_forward

    out = ring_forward(query, key, value, mask=mask, score_mod=score_mod, group=_AXES[axis_name])
    return _output_dropout(out, dropout_rng, dropout_rate, deterministic)


def ring_attention_reference(query, key, value, *, mask=None, score_mod=None):
    """Single-device equivalent of the ring on the global sequence (attention.py:694-721)."""
    return attention(query, key, value, mask=mask, score_mod=score_mod)
