"""The tensor-core path's certificate (k_rescore.cu) on inputs built to break it.

The bf16 / tf32 candidate pass ranks rows by approximate keys; the exact
rescoring is only trusted when the certificate proves that no row outside the
candidates can beat the k-th. These tests target the two assumptions the
proof rests on:

1. the representation bound |q.x - q~.x~| <= ||q - q~|| max||x|| +
   ||q~|| max||x - x~||: data whose bf16 rounding error is as large as it can
   be (components 1 + 2^-8, exactly halfway between two bf16 values) and
   parallel to the query, so Cauchy-Schwarz is tight, with competitors that
   the bf16 pass ranks above the true neighbour. A bound that is too small
   certifies a wrong answer; the correct one sends the query to a more
   precise tier, and the answer must equal the oracle's
   (FlatIndex::scan, crates/core/src/flat.rs:106-148);
2. the accumulation model (at most 3 * 2^-23 * sum|q~_i x~_i| lost per
   product, whatever grouping the tensor core uses): the approximate keys of
   the first pass, read through px_flat_debug_candidates, are compared with
   the exact sums of the rounded products on mixed-magnitude data (one large
   product and many below the accumulator's last place in every K step).
"""

import ctypes
import math

import numpy as np
import pytest

import oracle as O
from tests import _parity

pytestmark = pytest.mark.gpu

U8 = 2.0 ** -8  # half a bf16 unit in the last place at 1.0


@pytest.fixture(scope="module")
def pxm(px, oracle_lib):
    assert px.device_count() > 0, "GPU tests need a CUDA device"
    return px


def _index(pxm, data, metric, path="tensor"):
    m = pxm.Metric.L2 if metric == O.L2 else pxm.Metric.InnerProduct
    idx = pxm.FlatIndex(data.shape[1], m)
    idx.add(data)
    idx.set_search_path(path)
    return idx


def _adversarial_ip(d=768, n=4096):
    """Row 200 (every component 1 + 2^-8) is the query's true best match,
    but its bf16 copy is all ones; rows 0..199 (ones with j+1 components at
    1 + 2^-7, exact in bf16) score higher in bf16 and fill the candidate
    lists of every split that could hold row 200."""
    data = np.zeros((n, d), dtype=np.float32)
    for j in range(200):
        data[j] = 1.0
        data[j, : j + 1] = 1.0 + 2 * U8
    data[200] = 1.0 + U8
    queries = np.full((16, d), 1.0 + U8, dtype=np.float32)
    return data, queries


def _adversarial_folded_l2(d=96, n=4096):
    """L2 with d <= 256: the bf16 pass multiplies 2q with rows that carry
    their norms (folded). The row equal to the query (distance 0) is ranked
    behind 200 rows of ones with one component at 1.5 .. 1.75 (distance
    >= 0.246), because every 1 + 2^-8 rounds to 1 in bf16."""
    data = np.zeros((n, d), dtype=np.float32)
    for j in range(200):
        data[j] = 1.0
        data[j, j % d] = 1.5 + (j % 33) * 2.0 ** -7
    data[200] = 1.0 + U8
    queries = np.full((16, d), 1.0 + U8, dtype=np.float32)
    return data, queries


@pytest.mark.parametrize("k", [1, 10])
def test_tensor_path_certificate_adversarial_ip(pxm, k):
    data, queries = _adversarial_ip()
    idx = _index(pxm, data, O.IP)
    ids, d = idx.search_batch(queries, k=k)
    prof = idx.last_search_profile()
    assert prof["path"] == "tensor" and prof["first_pass"] == "bf16", prof
    # No query may be certified from the bf16 candidates alone.
    assert prof["fallback_queries"] + prof["refined_queries"] == len(queries), prof
    assert np.all(ids[:, 0] == 200), ids[:, :3]
    _parity.check_flat(data, O.IP, queries, ids, d, k)


@pytest.mark.parametrize("k", [1, 10])
def test_tensor_path_certificate_adversarial_folded_l2(pxm, k):
    data, queries = _adversarial_folded_l2()
    idx = _index(pxm, data, O.L2)
    ids, d = idx.search_batch(queries, k=k)
    prof = idx.last_search_profile()
    assert prof["path"] == "tensor" and prof["first_pass"] == "bf16", prof
    assert prof["fallback_queries"] + prof["refined_queries"] == len(queries), prof
    assert np.all(ids[:, 0] == 200), ids[:, :3]
    _parity.check_flat(data, O.L2, queries, ids, d, k)


def test_tensor_path_certificate_adversarial_mixed_batch(pxm):
    # Adversarial queries among ordinary ones: only they leave the bf16 tier.
    data, adv = _adversarial_ip()
    rng = np.random.default_rng(5)
    data[300:] = rng.standard_normal((data.shape[0] - 300, data.shape[1])).astype(np.float32)
    normal = rng.standard_normal((48, data.shape[1])).astype(np.float32)
    queries = np.concatenate([normal[:24], adv[:4], normal[24:]])
    idx = _index(pxm, data, O.IP)
    ids, d = idx.search_batch(queries, k=10)
    prof = idx.last_search_profile()
    assert prof["fallback_queries"] + prof["refined_queries"] >= 4, prof
    assert np.all(ids[24:28, 0] == 200)
    _parity.check_flat(data, O.IP, queries, ids, d, 10)


@pytest.mark.parametrize("metric", [O.IP, O.L2])
def test_tensor_path_certificate_adversarial_sample_pass(pxm, metric):
    """The same decoys on a shard long enough for the sample pass (160
    tiles; the sample is tiles 0, 5, ..., 155). The decoys sit in sample tile
    0, so every query starts from the 64th decoy's bf16 key (64 candidates
    are rescored for k = 10), and the true best row (in tile 3, outside the
    sample) scores above it in bf16: the main pass never offers it. The
    certificate's bound is then the starting key itself, which the decoys'
    exact keys do not clear, so the query must leave the bf16 tier, and the
    answer must still be the oracle's."""
    n = 40960
    if metric == O.IP:
        small, queries = _adversarial_ip()
    else:
        small, queries = _adversarial_folded_l2()
    d = small.shape[1]
    data = np.zeros((n, d), dtype=np.float32)
    data[:200] = small[:200]
    true_row = 3 * 256 + 7
    data[true_row] = small[200]
    idx = _index(pxm, data, metric)
    idx.set_sample_pass("on")
    ids, dd = idx.search_batch(queries, k=10)
    prof = idx.last_search_profile()
    assert prof["first_pass"] == "bf16" and prof["sample_tiles"] == 32, prof
    assert prof["fallback_queries"] + prof["refined_queries"] == len(queries), prof
    assert np.all(ids[:, 0] == true_row), ids[:, :3]
    _parity.check_flat(data, metric, queries, ids, dd, 10)


# ---- the accumulation model --------------------------------------------------

def _bf16_exact(rng, shape, lo, hi):
    """Positive values 2^-e * (1 + m/128), e in [lo, hi], m in [0, 127]:
    exactly representable in bf16 (and so in tf32 and fp32)."""
    e = rng.integers(lo, hi + 1, size=shape)
    m = rng.integers(0, 128, size=shape)
    return (np.ldexp(1.0 + m / 128.0, -e)).astype(np.float32)


def _mixed_magnitude_rows(rng, groups, per_group, d):
    """Per group g a sign pattern s_g (the group's query) and rows s_g * p with
    p a magnitude pattern: one large product and many far below the running
    sum's last place in each 16- or 8-value K step, in every position of the
    step, all one sign (so truncation errors add up) or mixed."""
    signs = rng.choice(np.array([-1.0, 1.0], dtype=np.float32), size=(groups, d))
    rows = []
    for g in range(groups):
        for r in range(per_group):
            kind = r % 8
            if kind in (0, 1, 5, 6):
                p = _bf16_exact(rng, d, 17, 26)  # small: 2^-17 .. 2^-26
                step = 16
                pos = {0: 0, 1: 15, 5: 7, 6: 0}[kind]
                p[pos::step] = 1.0 + rng.integers(0, 128, size=len(p[pos::step])) / 128.0
                if kind == 6:  # the small ones alternate in sign
                    p[1::2] *= -1.0
            elif kind == 2:  # large value at the head of every 8-value step
                p = _bf16_exact(rng, d, 14, 24)
                p[0::8] = 2.0
            elif kind == 3:  # random exponents over 24 binades
                p = _bf16_exact(rng, d, 0, 24)
            elif kind == 4:  # geometric decay along the row, repeating
                p = np.ldexp(np.float32(1.5), -(np.arange(d) % 24)).astype(np.float32)
            else:  # kind 7: a few large values, the rest just below them
                p = _bf16_exact(rng, d, 8, 12)
                p[rng.integers(0, d, size=4)] = 4.0
            rows.append((signs[g] * p).astype(np.float32))
    return signs.astype(np.float32), np.stack(rows)


def _bf16_round(x):
    """Round-to-nearest-even to bf16, as the device conversion does."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("metric,d,k,path", [
    (O.IP, 768, 10, "tensor"),          # bf16 pass, CTA pairs, kind::f16
    (O.IP, 768, 150, "tensor"),         # tf32 hi pass, kind::tf32
    (O.IP, 768, 10, "tensor_3xtf32"),   # three-pass tf32 (lo planes zero here)
    (O.IP, 96, 10, "tensor"),           # short rows: two K slices
    (O.L2, 96, 10, "tensor"),           # folded norms: 2q.x - ||x||^2
    (O.L2, 768, 10, "tensor"),          # L2 epilogue: ||x||^2 - 2 q.x
])
def test_tensor_accumulation_within_model(pxm, metric, d, k, path):
    rng = np.random.default_rng(1000 + d + k)
    groups, per_group = 32, 64
    qsign, data = _mixed_magnitude_rows(rng, groups, per_group, d)
    queries = qsign.copy()
    if metric == O.L2:
        queries *= np.float32(0.5)  # a query that is not a row
    assert np.array_equal(_bf16_round(data), data) and np.array_equal(_bf16_round(queries), queries)
    idx = _index(pxm, data, metric, path)
    lib = pxm._lib.load()
    nq = queries.shape[0]
    maxc = 256
    ids = np.empty((nq, maxc), dtype=np.int64)
    keys = np.empty((nq, maxc), dtype=np.float32)
    cands, kind = ctypes.c_int32(0), ctypes.c_int32(0)
    pxm._lib.check(lib.px_flat_debug_candidates(
        idx.handle, queries.ctypes.data_as(pxm._lib._f32p), nq, k, maxc,
        ids.ctypes.data_as(pxm._lib._i64p), keys.ctypes.data_as(pxm._lib._f32p),
        ctypes.byref(cands), ctypes.byref(kind)))
    want_kind = {("tensor", 10): 2, ("tensor", 150): 1, ("tensor_3xtf32", 10): 0}[(path, k)]
    assert kind.value == want_kind
    folded = metric == O.L2 and d <= 256
    norms = None
    if metric == O.L2:
        # The rows' fp32 squared norms in the reference's 8-lane order.
        zero = np.zeros(d, dtype=np.float32)
        norms = O.flat_keys(data, O.L2, zero, np.arange(data.shape[0]))
    worst = 0.0
    measured = 0
    for q in range(nq):
        qd = queries[q].astype(np.float64)
        for j in range(cands.value):
            r = int(ids[q, j])
            if r < 0:
                continue
            prods = qd * data[r].astype(np.float64)  # exact: bf16 x bf16 fits in a double
            dot = math.fsum(prods.tolist())
            mag = math.fsum(np.abs(prods).tolist())
            nprod = int(np.count_nonzero(prods))
            key = float(keys[q, j])
            if metric == O.IP:
                exact, m_acc, extra = -dot, mag, 0.0
            else:
                s = float(norms[r])
                exact = s - 2.0 * dot
                # Folded: 2q.x - ||x||^2 accumulates three more products of
                # the norm's pieces; otherwise the epilogue's fma rounds once.
                m_acc = 2.0 * mag + s if folded else 2.0 * mag
                nprod += 3 if folded else 0
                extra = 0.0 if folded else abs(key) * 2.0 ** -23
            bound = 3.0 * 2.0 ** -23 * (nprod + 2) * m_acc + extra + 1e-30
            err = abs(key - exact)
            worst = max(worst, err / bound)
            measured += 1
            assert err <= bound, (q, r, key, exact, err, bound)
    assert measured >= nq * min(cands.value, 32)
    # And the full search on the same data is exact.
    ids2, d2 = idx.search_batch(queries, k=k)
    _parity.check_flat(data, metric, queries, ids2, d2, k)
    print(f"accumulation error / model bound: max {worst:.4f} over {measured} products sums "
          f"(metric {metric}, d {d}, pass {kind.value})")
