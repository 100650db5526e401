"""Generates tests/golden/knn_ref_golden.npz from the REFERENCE's own code.

The reference's CUDA satellite (crates/core/cuda/knn.cu, knn_gpu_create /
knn_gpu_search, k <= 46) is compiled unchanged into oracle/_ref/libknn_ref.so
(`make -C oracle _ref/libknn_ref.so`) and run on a GPU host. Its key-space
top-k (squared L2, or -inner product) on seeded inputs are stored here, so
that the CPU test suite can check the oracle's restatement of
FlatIndex::search_batch (crates/core/src/flat.rs:150-191) against output of
the reference itself:

  * "sift": config 2's integer-valued SIFT-like mixture (values 0..255,
    d = 128). Every squared-L2 and inner-product partial sum is an integer
    below 2^24, so the kernel's sequential sums and the CPU's 8-lane sums are
    exactly equal: keys must match bit for bit, ids except at exact ties.
  * "unit": config 1/4's unit-norm N(0,1) rows (d = 96), inner product. The
    kernel sums in another order than the CPU path, so keys agree to rounding
    (1e-5 relative) and ids except at near-ties.

Usage (needs a CUDA device and oracle/_ref/libknn_ref.so):
  python tests/golden/make_knn_ref_golden.py [out.npz]
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402
from tests import _data  # noqa: E402

# name: (generator, n, dim, nq, seed, metrics)
CASES = {
    "sift": ("sift", 20000, 128, 40, 21, (O.L2, O.IP)),
    "unit": ("unit", 20000, 96, 40, 22, (O.IP,)),
}
KS = (10, 46)


def case_data(name):
    gen, n, dim, nq, seed, _ = CASES[name]
    if gen == "sift":
        return _data.sift_like(n, nq, d=dim, centres=100, seed=seed)
    return _data.unit_gaussian(n, dim, seed), _data.unit_gaussian(nq, dim, seed + 1000)


def main():
    out_path = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "knn_ref_golden.npz")
    if not O.ref_knn_available():
        raise SystemExit("oracle/_ref/libknn_ref.so is missing: make -C oracle _ref/libknn_ref.so")
    out = {}
    for name in CASES:
        base, queries = case_data(name)
        ref = O.RefKnn(base)
        for metric in CASES[name][5]:
            for k in KS:
                ids, keys = ref.search(queries, k, metric)
                out[f"{name}_m{metric}_k{k}_ids"] = ids
                out[f"{name}_m{metric}_k{k}_keys"] = keys
        ref.close()
    np.savez_compressed(out_path, **out)
    print(out_path, os.path.getsize(out_path), "bytes")


if __name__ == "__main__":
    main()
