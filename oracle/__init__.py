"""CPU oracle for the fused selected-quant paged decode path.

TEST INFRASTRUCTURE ONLY.  This package restates, in numpy, the reference
algorithms of manishklach/intent-attention-kernel for the hot path (fake
quantisation, dense attention over selected blocks, the paged online-softmax
decode, the LSE merge and the MLA latent decode).  It is the checker, never the
thing measured or shipped: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.  The
product package (``intent-attention-kernel_b200/intent_attention``) never
imports it and has no CPU fallback.

Parity pinning: every function here is checked against golden vectors that
``tests/golden/make_golden.py`` produced by importing and running the reference
Python package itself (see ``tests/test_oracle_golden.py``).
"""

from . import quant, attention, decode, mla  # noqa: F401
