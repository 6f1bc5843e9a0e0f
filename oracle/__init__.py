"""CPU oracle for the AR-aware 3D block-sparse attention path.

TEST INFRASTRUCTURE ONLY. This package is the checker that the CUDA path is
compared against. It may be imported only by ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``. The product package never imports it, and the product
path raises when its CUDA library is missing instead of falling back here.

Parity pinning: the reference ships no tests, golden vectors or known-answer
tests. The oracle is pinned against the reference's own code, run unchanged on
CPU in the build container (its Triton kernels under ``TRITON_INTERPRET=1``,
its selection functions in plain torch). ``tests/golden/make_golden.py``
records those outputs as fixtures, and ``tests/test_oracle_golden.py`` checks
the oracle against them.
"""

from .li_oracle import *  # noqa: F401,F403
from .inputs import det_normal, det_normal_like  # noqa: F401
