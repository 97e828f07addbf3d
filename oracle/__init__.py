"""CPU oracle for the UltraQuant quantization hot path.

TEST INFRASTRUCTURE ONLY.  This package is a plain numpy / torch-CPU
restatement of the reference algorithm (qlab.py, trellis.py, qat.py of
hackerbbrine/UltraQuant).  It exists to check the CUDA path and to time the
reference-style CPU baseline.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py`` (its CPU-baseline / reference arm) may import it; the product
package ``ultraquant_b200`` never does, and has no CPU fallback.

Pinning: every function here is checked against golden vectors produced by
running the reference modules themselves (``tests/golden/make_golden.py``,
fixtures in ``tests/golden/*.npz``), see ``tests/test_oracle_golden.py``.
"""
from .uq_oracle import *  # noqa: F401,F403
