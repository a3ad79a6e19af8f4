"""CPU oracle for the delta-attention hot path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker or as the timed
CPU reference arm.  The product path (``delta_attention_b200``) never imports
it and has no CPU fallback.

Parity status: PINNED.  ``tests/golden/make_golden.py`` runs the reference's
own CPU-runnable implementation (``delta_attention/train/flex_delta.py``
``delta_forward_train``, ``delta_attention/stride.py``, and the decode methods
of ``delta_attention/llama.py`` executed from the reference source) and stores
its outputs as fixtures; ``tests/test_oracle_golden.py`` checks this oracle
against them.
"""

from .delta_oracle import *  # noqa: F401,F403
