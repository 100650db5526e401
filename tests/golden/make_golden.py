"""Generates tests/golden/flat_pq_golden.npz from the CPU oracle.

The reference ships no golden vectors (its Rust crate cannot be built or run
in this image), so these fixtures are regression pins of the oracle on the
reference tests' own SplitMix data generator (crates/core/src/flat.rs:238):
exact Flat top-k for L2 and inner product, and a PQ index trained, encoded
and searched as pq.rs does it. The GPU parity tests compare against them too.

Usage: python tests/golden/make_golden.py
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402


def main():
    n, dim, nq, k, m = 600, 24, 20, 10, 4
    seed_base, seed_query, pq_seed = 7, 999, 0x5EED
    data = O.gen_uniform(n, dim, seed_base)
    queries = O.gen_uniform(nq, dim, seed_query)
    out = dict(n=n, dim=dim, nq=nq, k=k, m=m, seed_base=seed_base, seed_query=seed_query,
               pq_seed=pq_seed)
    for metric, name in ((O.L2, "l2"), (O.IP, "ip")):
        ids, d = O.flat_search_batch(data, metric, queries, k)
        out[f"flat_{name}_ids"] = ids
        out[f"flat_{name}_dists"] = d
    books = O.pq_train(data, m, train_iters=10, train_sample=0, seed=pq_seed)
    codes = O.pq_encode(books, data)
    ids, d = O.pq_search_batch(books, O.L2, codes, queries, k)
    out.update(pq_books=books, pq_codes=codes, pq_ids=ids, pq_dists=d)
    path = os.path.join(HERE, "flat_pq_golden.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
