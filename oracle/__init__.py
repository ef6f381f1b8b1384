"""CPU oracle for the GMM EM hot path (test infrastructure only).

This package restates, in numpy, the soft-EM algorithm of the reference's
PyTorch implementation (``gmmxx/torch_fallback.py``).  It is the checker that
the CUDA engine is compared against; it is never imported by the product code
path.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (the
``cpu_baseline`` leg and ``--impl reference``) may use it.

Parity pin: ``tests/test_oracle_golden.py`` checks this restatement against
golden vectors produced by the reference itself (``tests/golden/make_golden.py``
imports the reference read-only and records its outputs).
"""

from .gmm_oracle import *  # noqa: F401,F403
