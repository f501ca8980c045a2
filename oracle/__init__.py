"""CPU oracle for the quaternion SSM hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the ``mambaqc_b200`` package imports this
package; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline / reference arm use it, and only as the checker or the timed CPU
baseline, never as the product path.

``oracle.ref`` restates, in plain PyTorch on the CPU, the reference
implementation of polux06/mambaqc for the functions on the hot path. Each
function cites the reference file:line it follows. Parity of this restatement is
pinned by golden fixtures generated from the reference itself
(``tests/golden/make_golden.py``) and checked by ``tests/test_oracle_golden.py``.
"""

from . import ref  # noqa: F401
