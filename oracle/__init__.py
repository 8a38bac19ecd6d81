"""CPU oracle for Daiza's hybrid-attention hot path.

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.  Only
tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs may import this
package; the product library (``daiza_b200``) never does.

Parity status: unpinned by the reference's own tests (the Rust reference cannot
be built here and ships no golden vectors for this path).  The C++ restatement
in ``dz_oracle.cpp`` follows the reference op for op and is cross-checked
against the independent float64 restatement in ``f64_ref.py``.
"""
from .oracle import *  # noqa: F401,F403
