"""CPU oracle for the exact-kNN / PQ-ADC hot path (test infrastructure only).

The oracle restates the reference's CPU arithmetic bit for bit
(crates/core/src/distance.rs, flat.rs, pq.rs; see oracle.cpp). It is used by
tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
as the checker and the timed CPU baseline. The product package
``proxima_b200`` never imports it.

Parity status: the flat search is pinned against outputs of the reference's
own CUDA kernel (crates/core/cuda/knn.cu, compiled unchanged into
_ref/libknn_ref.so and run on a B200; fixtures in
tests/golden/knn_ref_golden.npz, made by tests/golden/make_knn_ref_golden.py)
and by the reference's known-answer and property tests (restated in
tests/test_oracle.py). The PQ restatement is pinned by those tests only: the
reference has no PQ code outside its Rust crate, which cannot be built here.
"""

from .oracle import *  # noqa: F401,F403
