"""CPU oracle for the exact-kNN / PQ-ADC hot path (test infrastructure only).

The oracle restates the reference's CPU arithmetic bit for bit
(crates/core/src/distance.rs, flat.rs, pq.rs; see oracle.cpp). It is used by
tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
as the checker and the timed CPU baseline. The product package
``proxima_b200`` never imports it.

Parity status: pinned by the reference's own known-answer and property tests
(restated in tests/test_oracle.py); the reference ships no golden vectors and
its Rust crate cannot be built in this image.
"""

from .oracle import *  # noqa: F401,F403
