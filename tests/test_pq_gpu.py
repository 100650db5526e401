"""GPU parity of PqIndex (training, encoding, ADC scan) against the oracle.

Training (k-means), encoding and the ADC keys are all bit-exact
restatements of crates/core/src/pq.rs, so codebooks and codes must be
identical and search results must pass the tie-aware rule of
tests/_parity.py.
"""

import os

import numpy as np
import pytest

import oracle as O
from tests import _data, _parity

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "flat_pq_golden.npz")


@pytest.fixture(scope="module")
def pxm(px, oracle_lib):
    assert px.device_count() > 0, "GPU tests need a CUDA device"
    return px


def _metric(pxm, m):
    return pxm.Metric.L2 if m == O.L2 else pxm.Metric.InnerProduct


def test_golden_fixture(pxm):
    g = np.load(GOLDEN)
    data = O.gen_uniform(int(g["n"]), int(g["dim"]), int(g["seed_base"]))
    queries = O.gen_uniform(int(g["nq"]), int(g["dim"]), int(g["seed_query"]))
    pq = pxm.PqIndex(int(g["dim"]), pxm.Metric.L2, m=int(g["m"]), train_iters=10, train_sample=0,
                     seed=int(g["pq_seed"]))
    pq.train(data)
    assert np.array_equal(pq.codebooks.view(np.uint32), g["pq_books"].view(np.uint32))
    pq.add(data)
    assert np.array_equal(pq.encode(data), g["pq_codes"])
    ids, d = pq.search_batch(queries, k=int(g["k"]))
    _parity.check(ids, d, g["pq_ids"], g["pq_dists"],
                  _parity.pq_natural(g["pq_books"], O.L2, g["pq_codes"], queries))


@pytest.mark.parametrize("metric", [O.L2, O.IP])
@pytest.mark.parametrize("dim,m,nbits,sample", [(64, 8, 8, 50000), (64, 16, 8, 2000),
                                                 (48, 16, 4, 0), (30, 5, 6, 50)])
def test_training_and_encoding_bit_exact(pxm, metric, dim, m, nbits, sample):
    rng = np.random.default_rng(dim + m)
    data = rng.standard_normal((4000, dim)).astype(np.float32)
    pq = pxm.PqIndex(dim, _metric(pxm, metric), m=m, nbits=nbits, train_iters=8,
                     train_sample=sample, seed=24301)
    pq.train(data)
    books = O.pq_train(data, m, nbits=nbits, train_iters=8, train_sample=sample, seed=24301)
    assert np.array_equal(pq.codebooks.view(np.uint32), books.view(np.uint32))
    codes = O.pq_encode(books, data)
    assert np.array_equal(pq.encode(data), codes)
    pq.add(data)
    queries = rng.standard_normal((23, dim)).astype(np.float32)
    for k in (1, 10, 100):
        ids, d = pq.search_batch(queries, k=k)
        _parity.check_pq(books, metric, codes, queries, ids, d, k)


def test_config3_shape(pxm):
    # Config 3's shape (d=128, m=16, 256 centroids, SIFT-like data), scaled down.
    base, queries = _data.sift_like(60000, 40, seed=7, centres=200)
    pq = pxm.PqIndex(128, pxm.Metric.L2, m=16, train_iters=6, train_sample=20000, seed=3)
    pq.train(base)
    books = pq.codebooks
    pq.add(base)
    codes = pq.encode(base)
    ids, d = pq.search_batch(queries, k=10)
    _parity.check_pq(books, O.L2, codes, queries, ids, d, 10)
    ids1, d1 = pq.search(queries[3], k=10)
    assert ids1.tolist() == ids[3].tolist()


@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_search_device_matches_host_search(pxm, metric):
    # px_pq_search_device: queries and results in device memory on the
    # caller's stream; natural distances equal px_pq_search's bit for bit,
    # key space is squared L2 / -IP.
    import ctypes

    import torch

    base, queries = _data.sift_like(20000, 19, seed=11, centres=50)
    pq = pxm.PqIndex(128, _metric(pxm, metric), m=16, train_iters=4, seed=9)
    pq.train(base)
    pq.add(base)
    k = 10
    want_ids, want_d = pq.search_batch(queries, k=k)
    dev = torch.device("cuda", 0)
    d_q = torch.from_numpy(queries).to(dev)
    lib = pxm._lib.load()
    sp = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for key_space in (0, 1):
        ids = torch.empty((len(queries), k), dtype=torch.int64, device=dev)
        d = torch.empty((len(queries), k), dtype=torch.float32, device=dev)
        pxm._lib.check(lib.px_pq_search_device(pq.handle, ctypes.c_void_p(d_q.data_ptr()), len(queries), k,
                                               key_space, ctypes.c_void_p(ids.data_ptr()),
                                               ctypes.c_void_p(d.data_ptr()), sp))
        torch.cuda.synchronize()
        got_ids, got_d = ids.cpu().numpy(), d.cpu().numpy()
        assert np.array_equal(got_ids, want_ids)
        if key_space == 0:
            assert np.array_equal(got_d.view(np.uint32), want_d.view(np.uint32))
        else:
            nat = np.sqrt(got_d) if metric == O.L2 else -got_d
            assert np.array_equal(nat.astype(np.float32).view(np.uint32), want_d.view(np.uint32))


@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_m16_scan_edges(pxm, metric):
    # m = 16 with 256 centroids and 8-query groups is the scan's skewed path:
    # a ragged row count over several CTAs and iterations, a partial last
    # group, a filter, and an all-zero query (inner-product entries -0.0,
    # whose sums must still start from +0.0).
    rng = np.random.default_rng(16)
    data = rng.standard_normal((3000, 32)).astype(np.float32)
    pq = pxm.PqIndex(32, _metric(pxm, metric), m=16, train_iters=4, seed=5)
    pq.train(data)
    books = pq.codebooks
    codes = rng.integers(0, 256, size=(70001, 16), dtype=np.uint8)
    codes[:40] = codes[40]  # a run of identical rows (exact key ties)
    pq.add_codes(codes)
    queries = rng.standard_normal((21, 32)).astype(np.float32)
    queries[4] = 0.0
    for k in (1, 10, 50):
        ids, d = pq.search_batch(queries, k=k)
        _parity.check_pq(books, metric, codes, queries, ids, d, k)
    mask = rng.random(len(codes)) < 0.3
    ids, d = pq.search_batch_filtered(queries, mask, k=10)
    _parity.check_pq(books, metric, codes, queries, ids, d, 10, filter_=mask)


def test_add_codes_and_filters(pxm):
    rng = np.random.default_rng(4)
    data = rng.standard_normal((3000, 32)).astype(np.float32)
    pq = pxm.PqIndex(32, pxm.Metric.L2, m=8, train_iters=5)
    pq.train(data)
    books = pq.codebooks
    codes = O.pq_encode(books, data)
    pq.add_codes(codes[:1000])
    pq.add_codes(codes[1000:])
    queries = rng.standard_normal((7, 32)).astype(np.float32)
    for mask in (rng.random(3000) < 0.25, np.zeros(3000, bool)):
        ids, d = pq.search_batch_filtered(queries, mask, k=10)
        _parity.check_pq(books, O.L2, codes, queries, ids, d, 10, filter_=mask)
        sid, sd = pq.search_filtered(queries[0], mask, k=10)
        assert sid.tolist() == ids[0].tolist()


# ---- the reference's tests/test_pq.py, run against this package ----------

def _recall(approx, gt, k):
    hits = sum(len({int(x) for x in a if x >= 0} & {int(x) for x in g}) for a, g in zip(approx, gt))
    return hits / (len(approx) * k)


@pytest.fixture(scope="module")
def pq_data():
    return np.random.default_rng(0).standard_normal((4000, 64)).astype(np.float32)


@pytest.fixture(scope="module")
def pq_queries():
    return np.random.default_rng(9).standard_normal((200, 64)).astype(np.float32)


def test_lifecycle_and_recall(pxm, pq_data, pq_queries):
    flat = pxm.FlatIndex(dim=64, metric=pxm.Metric.L2)
    flat.add(pq_data)
    gt, _ = flat.search_batch(pq_queries, k=10)
    pq = pxm.PqIndex(dim=64, metric=pxm.Metric.L2, m=8)
    assert not pq.is_trained
    pq.train(pq_data)
    assert pq.is_trained
    pq.add(pq_data)
    assert pq.size == len(pq_data) == len(pq)
    approx, _ = pq.search_batch(pq_queries, k=10)
    assert _recall(approx, gt, 10) > 0.25


def test_recall_at_100_high(pxm, pq_data, pq_queries):
    flat = pxm.FlatIndex(dim=64, metric=pxm.Metric.L2)
    flat.add(pq_data)
    gt, _ = flat.search_batch(pq_queries, k=100)
    pq = pxm.PqIndex(dim=64, metric=pxm.Metric.L2, m=16)
    pq.train(pq_data)
    pq.add(pq_data)
    approx, _ = pq.search_batch(pq_queries, k=100)
    assert _recall(approx, gt, 100) > 0.55


def test_compression_ratio(pxm):
    base = np.random.default_rng(0).standard_normal((40000, 64)).astype(np.float32)
    pq = pxm.PqIndex(dim=64, metric=pxm.Metric.L2, m=8)
    pq.train(base)
    pq.add(base)
    assert pq.raw_bytes == len(base) * 64 * 4
    assert pq.compression_ratio > 20


def test_small_train_sample_not_degenerate(pxm, pq_data, pq_queries):
    flat = pxm.FlatIndex(dim=64, metric=pxm.Metric.L2)
    flat.add(pq_data)
    gt, _ = flat.search_batch(pq_queries, k=10)
    pq = pxm.PqIndex(dim=64, metric=pxm.Metric.L2, m=8, train_sample=50)
    pq.train(pq_data)
    pq.add(pq_data)
    assert pq.is_trained and pq.size == len(pq_data)
    approx, _ = pq.search_batch(pq_queries, k=10)
    assert _recall(approx, gt, 10) > 0.15


def test_inner_product_metric(pxm, pq_queries):
    rng = np.random.default_rng(1)
    data = rng.standard_normal((4000, 64)).astype(np.float32)
    data /= np.linalg.norm(data, axis=1, keepdims=True)
    q = pq_queries / np.linalg.norm(pq_queries, axis=1, keepdims=True)
    flat = pxm.FlatIndex(dim=64, metric=pxm.Metric.InnerProduct)
    flat.add(data)
    gt, _ = flat.search_batch(q, k=10)
    pq = pxm.PqIndex(dim=64, metric=pxm.Metric.InnerProduct, m=16)
    pq.train(data)
    pq.add(data)
    approx, _ = pq.search_batch(q, k=10)
    assert _recall(approx, gt, 10) > 0.3


def test_train_rejects_bad_input(pxm):
    pq = pxm.PqIndex(dim=16, metric=pxm.Metric.L2, m=4)
    with pytest.raises(ValueError, match="too small"):
        pq.train(np.zeros((100, 16), np.float32))
    bad = np.random.default_rng(0).standard_normal((300, 16)).astype(np.float32)
    bad[5, 3] = np.nan
    with pytest.raises(ValueError, match="NaN"):
        pq.train(bad)
