"""CPU oracle for the Redshift attention / gated-DeltaNet hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product library imports this package;
only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` use it, and only as the checker (or as the timed CPU baseline).

The arithmetic restates the reference's scalar float64 oracle
``tests/cpu_reference.py`` (cristianku/redshift) in vectorised numpy float64.
Parity of this restatement with the reference is pinned by golden vectors that
were produced by running the reference oracle itself (``tests/golden/``), and
by the reference's closed-form long-context known-answer test
(``tests/test_cuda.py:237-273``), restated in ``oracle.closed_form``.
"""
from .hotpath import (attention, delta, delta_commit, delta_core, delta_trace,  # noqa: F401
                      prefill_attention_core, half, sigmoid, silu, softplus)
from . import inputs, closed_form  # noqa: F401
