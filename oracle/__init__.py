"""CPU oracle for the attention hot path (test infrastructure only).

This package restates, in numpy, the reference implementation of attnax's
attention hot path.  It is the checker: only ``tests/``, ``__graft_entry__.smoke``
and the CPU-baseline leg of ``bench.py`` may import it.  The product package
``attnax_b200`` never imports it and has no CPU fallback.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference's own
source files (``attnax/kernels/*.py``, ``attnax/paged_cache.py``,
``attnax/masking.py``) unmodified under a small numpy stand-in for the
``jax.numpy`` primitives they call, and ``tests/test_oracle_golden.py``
checks this restatement against those vectors and against the known-answer
assertions in the reference's test suite.
"""

from .attention_oracle import *  # noqa: F401,F403
