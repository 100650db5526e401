"""Tie-aware parity checks shared by the GPU tests.

Rule (from the north star): returned ids must equal the oracle's except where
distances tie, and distances must agree. Here distances must agree bit for
bit, because every GPU path ends in the reference's exact arithmetic:

  1. the k reported distances equal the oracle's, rank by rank, bitwise;
  2. padding (-1 ids) sits at the same ranks;
  3. the ids of a row are distinct, pass the filter, and each id's own exact
     distance (recomputed by the oracle) equals the distance reported beside
     it;
  4. an id may differ from the oracle's only at a rank whose distance occurs
     more than once in the row or equals the k-th distance (an exact tie).
"""

import numpy as np

import oracle as O


def check(ids, dists, ref_ids, ref_dists, natural_of, filter_=None):
    """natural_of(q, id_array) -> the exact natural distances of those ids."""
    ids = np.asarray(ids)
    dists = np.asarray(dists, dtype=np.float32)
    assert ids.shape == ref_ids.shape, (ids.shape, ref_ids.shape)
    du, ru = dists.view(np.uint32), ref_dists.view(np.uint32)
    if not np.array_equal(du, ru):
        bad = np.argwhere(du != ru)
        q, j = bad[0]
        raise AssertionError(
            f"distance mismatch at query {q} rank {j}: got {dists[q, j]!r} want {ref_dists[q, j]!r}"
            f" ({len(bad)} positions differ); ids {ids[q]} vs {ref_ids[q]}")
    n_tie = 0
    for q in range(ids.shape[0]):
        row = ids[q]
        valid = row >= 0
        assert np.array_equal(valid, ref_ids[q] >= 0), f"padding differs at query {q}"
        got = row[valid]
        assert len(set(got.tolist())) == got.size, f"duplicate ids at query {q}: {row}"
        if filter_ is not None:
            assert np.all(np.asarray(filter_)[got]), f"filtered-out id at query {q}"
        if got.size:
            nat = np.asarray(natural_of(q, got), dtype=np.float32)
            assert np.array_equal(nat.view(np.uint32), dists[q][valid].view(np.uint32)), \
                f"reported distances are not the ids' own distances at query {q}"
        for j in np.nonzero(row != ref_ids[q])[0]:
            d = dists[q, j]
            tied = np.count_nonzero(dists[q] == d) > 1 or d == dists[q, -1]
            assert tied, f"id differs without a tie at query {q} rank {j}: {row} vs {ref_ids[q]}"
            n_tie += 1
    return n_tie


def flat_natural(data, metric, queries):
    def f(q, idx):
        keys = O.flat_keys(data, metric, queries[q], idx)
        return np.sqrt(keys) if metric == O.L2 else -keys
    return f


def pq_natural(books, metric, codes, queries):
    tables = {}

    def f(q, idx):
        if q not in tables:
            tables[q] = O.pq_adc_table(books, metric, queries[q])
        t = tables[q]
        m = codes.shape[1]
        out = []
        for i in idx:
            key = np.float32(0.0)
            for sub in range(m):
                key = np.float32(key + t[sub, codes[i, sub]])
            out.append(key)
        keys = np.array(out, dtype=np.float32)
        return np.sqrt(keys) if metric == O.L2 else -keys
    return f


def check_flat(data, metric, queries, ids, dists, k, filter_=None):
    ref_ids, ref_d = O.flat_search_batch(data, metric, queries, k, filter_)
    return check(ids, dists, ref_ids, ref_d, flat_natural(data, metric, queries), filter_)


def check_pq(books, metric, codes, queries, ids, dists, k, filter_=None):
    ref_ids, ref_d = O.pq_search_batch(books, metric, codes, queries, k, filter_)
    return check(ids, dists, ref_ids, ref_d, pq_natural(books, metric, codes, queries), filter_)
