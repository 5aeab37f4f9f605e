"""CPU oracle for the Qwen3 decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the golden (CPU reference) functions of the
IRON operators on the Qwen3 decode path.  Each function cites the reference
file:line it follows.  It is the *checker* for the CUDA kernels in
``iron_b200``: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / reference arm may import it.  The product path (``iron_b200``)
never imports or calls anything here and has no CPU fallback.

Pinning: ``tests/golden/*.npz`` hold vectors produced by running the
reference's own golden functions (``tests/golden/make_golden.py``, run in a
container where the reference source is present).  ``tests/test_oracle_golden.py``
checks every function here against those vectors.
"""

from . import bf16, ops, qwen3  # noqa: F401
