"""CPU oracle for the tensor-parallel decoder-layer forward.

TEST INFRASTRUCTURE ONLY.  This package restates, in numpy, the algorithm of the
reference engine (kmadasamy212-tech/pythonintern) for the decoder-layer hot path so
that the CUDA path in ``pythonintern_b200`` can be checked against it.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it, and only as the checker or as the timed CPU stand-in for the reference.
The product path never calls into this package.

Parity of this oracle is pinned by ``tests/test_oracle_golden.py`` against golden
vectors produced by running the reference itself (``tests/golden/make_golden.py``).
"""

from oracle.decoder import *  # noqa: F401,F403
