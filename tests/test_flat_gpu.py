"""GPU parity of FlatIndex (exact kNN) against the CPU oracle.

Every case compares the sm_100a path, called through the C ABI, with the
oracle's restatement of FlatIndex::search_batch (crates/core/src/flat.rs)
using the tie-aware, bit-exact rule of tests/_parity.py.
"""

import ctypes
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


def _run(pxm, data, metric, queries, k, adds=1, filter_=None):
    idx = pxm.FlatIndex(data.shape[1], _metric(pxm, metric))
    for part in np.array_split(data, adds):
        idx.add(np.ascontiguousarray(part))
    if filter_ is None:
        return idx.search_batch(queries, k=k)
    return idx.search_batch_filtered(queries, filter_, k=k)


@pytest.mark.parametrize("metric", [O.L2, O.IP])
@pytest.mark.parametrize("n,dim,nq,k", [
    (1000, 24, 1, 10), (1000, 24, 7, 10), (5000, 64, 33, 5), (2000, 12, 9, 1),
    (3000, 7, 5, 17), (777, 3, 4, 100), (4000, 128, 64, 10), (300, 16, 2, 300),
])
def test_uniform_parity(pxm, metric, n, dim, nq, k):
    data = O.gen_uniform(n, dim, 7 + n)
    queries = O.gen_uniform(nq, dim, 999 + dim)
    ids, d = _run(pxm, data, metric, queries, k)
    _parity.check_flat(data, metric, queries, ids, d, k)


def test_golden_fixture(pxm):
    g = np.load(GOLDEN)
    data = O.gen_uniform(int(g["n"]), int(g["dim"]), int(g["seed_base"]))
    queries = O.gen_uniform(int(g["nq"]), int(g["dim"]), int(g["seed_query"]))
    k = int(g["k"])
    for metric, name in ((O.L2, "l2"), (O.IP, "ip")):
        ids, d = _run(pxm, data, metric, queries, k)
        _parity.check(ids, d, g[f"flat_{name}_ids"], g[f"flat_{name}_dists"],
                      _parity.flat_natural(data, metric, queries))


def test_config1_shape_ip(pxm):
    # Config 1's distribution (unit-norm N(0,1), d=384, IP), fewer rows.
    data = _data.unit_gaussian(20000, 384, 1)
    queries = _data.unit_gaussian(16, 384, 2)
    ids, d = _run(pxm, data, O.IP, queries, 10)
    _parity.check_flat(data, O.IP, queries, ids, d, 10)


def test_config2_shape_l2_with_ties(pxm):
    # Config 2's distribution (integer-valued SIFT-like mixture, L2).
    data, queries = _data.sift_like(50000, 24, seed=3, centres=100)
    ids, d = _run(pxm, data, O.L2, queries, 10)
    _parity.check_flat(data, O.L2, queries, ids, d, 10)
    # Duplicated rows force exact ties at every rank.
    dup = np.repeat(data[:500], 3, axis=0)
    ids, d = _run(pxm, dup, O.L2, dup[:8] + 1.0, 10)
    _parity.check_flat(dup, O.L2, dup[:8] + 1.0, ids, d, 10)


def test_config5_shape_l2(pxm):
    data, queries = _data.gaussian_mixture(30000, 12, centres=300, seed=5)
    ids, d = _run(pxm, data, O.L2, queries, 10)
    _parity.check_flat(data, O.L2, queries, ids, d, 10)


def test_incremental_adds_keep_global_ids(pxm):
    data = O.gen_uniform(4000, 32, 21)
    queries = O.gen_uniform(9, 32, 22)
    ids, d = _run(pxm, data, O.L2, queries, 10, adds=5)
    _parity.check_flat(data, O.L2, queries, ids, d, 10)


@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_filtered_parity(pxm, metric):
    data = O.gen_uniform(3000, 48, 31)
    queries = O.gen_uniform(6, 48, 32)
    rng = np.random.default_rng(1)
    for mask in (rng.random(3000) < 0.2, np.zeros(3000, bool), np.arange(3000) == 17):
        ids, d = _run(pxm, data, metric, queries, 10, filter_=mask)
        _parity.check_flat(data, metric, queries, ids, d, 10, filter_=mask)


def test_empty_and_small_index(pxm):
    idx = pxm.FlatIndex(4, pxm.Metric.L2)
    ids, d = idx.search(np.zeros(4, np.float32), k=3)
    assert ids.tolist() == [-1, -1, -1]
    assert d.tolist() == [np.finfo(np.float32).max] * 3
    idx.add(np.array([[0, 0, 0, 0], [1, 1, 1, 1]], np.float32))
    ids, d = idx.search(np.zeros(4, np.float32), k=5)
    assert ids.tolist() == [0, 1, -1, -1, -1]
    assert d.tolist()[:2] == [0.0, 2.0]
    ids, d = idx.search(np.zeros(4, np.float32), k=0)
    assert ids.shape == (0,) and d.shape == (0,)
    ipx = pxm.FlatIndex(4, pxm.Metric.InnerProduct)
    ipx.add(np.ones((1, 4), np.float32))
    ids, d = ipx.search(np.ones(4, np.float32), k=3)
    assert ids.tolist() == [0, -1, -1]
    assert d.tolist()[1:] == [-np.finfo(np.float32).max] * 2


def test_errors_are_reported(pxm):
    idx = pxm.FlatIndex(8, pxm.Metric.L2)
    with pytest.raises(ValueError):
        idx.add(np.zeros((10, 9), np.float32))
    with pytest.raises(ValueError, match="NaN"):
        idx.add(np.full((1, 8), np.nan, np.float32))
    idx.add(np.zeros((10, 8), np.float32))
    with pytest.raises(ValueError):
        idx.search(np.zeros(7, np.float32), k=3)
    with pytest.raises(ValueError, match="NaN"):
        idx.search(np.full(8, np.inf, np.float32), k=3)
    with pytest.raises(ValueError):
        idx.search(np.zeros(8, np.float32), k=pxm.PX_MAX_K + 1)
    with pytest.raises(ValueError, match="mask length"):
        idx.search_filtered(np.zeros(8, np.float32), np.zeros(9, bool), k=3)
    with pytest.raises(TypeError):
        idx.add(np.zeros((10, 8), np.float64))


# ---- the reference's tests/test_engine.py, run against this package ------

def _normalize(x):
    return x / np.linalg.norm(x, axis=-1, keepdims=True)


@pytest.fixture(scope="module")
def engine_data():
    rng = np.random.default_rng(0)
    return _normalize(rng.standard_normal((3000, 64)).astype(np.float32))


def test_engine_inner_product_matches_numpy(pxm, engine_data):
    idx = pxm.FlatIndex(dim=64, metric=pxm.Metric.InnerProduct)
    idx.add(engine_data)
    q = _normalize(np.random.default_rng(1).standard_normal(64).astype(np.float32))
    ids, sims = idx.search(q, k=10)
    ref = np.argsort(-(engine_data @ q))[:10]
    assert set(ids.tolist()) == set(ref.tolist())
    for i, s in zip(ids.tolist(), sims.tolist()):
        assert abs(s - float(engine_data[i] @ q)) < 1e-4


def test_engine_l2_matches_numpy(pxm, engine_data):
    idx = pxm.FlatIndex(dim=64, metric=pxm.Metric.L2)
    idx.add(engine_data)
    q = _normalize(np.random.default_rng(2).standard_normal(64).astype(np.float32))
    ids, dists = idx.search(q, k=10)
    d_all = np.linalg.norm(engine_data - q, axis=1)
    ref = np.argsort(d_all)[:10]
    assert set(ids.tolist()) == set(ref.tolist())
    assert np.all(np.diff(dists) >= -1e-4)
    assert abs(dists[0] - d_all[ref[0]]) < 1e-3


def test_engine_self_is_nearest(pxm, engine_data):
    idx = pxm.FlatIndex(dim=64, metric=pxm.Metric.InnerProduct)
    idx.add(engine_data)
    for i in (0, 100, 2999):
        ids, sims = idx.search(engine_data[i].copy(), k=1)
        assert ids[0] == i
        assert sims[0] == pytest.approx(1.0, abs=1e-3)


def test_engine_batch_equals_single(pxm, engine_data):
    idx = pxm.FlatIndex(dim=64, metric=pxm.Metric.InnerProduct)
    idx.add(engine_data)
    queries = _normalize(np.random.default_rng(3).standard_normal((50, 64)).astype(np.float32))
    bids, _ = idx.search_batch(queries, k=8, num_threads=4)
    for qi in range(len(queries)):
        sids, _ = idx.search(queries[qi], k=8)
        assert bids[qi].tolist() == sids.tolist()


def test_engine_padding_and_metadata(pxm):
    idx = pxm.FlatIndex(dim=4, metric=pxm.Metric.L2)
    idx.add(np.eye(3, 4, dtype=np.float32))
    ids, _ = idx.search(np.zeros(4, dtype=np.float32), k=5)
    assert (ids[3:] == -1).all()
    assert sorted(ids[:3].tolist()) == [0, 1, 2]
    m = pxm.FlatIndex(dim=16, metric=pxm.Metric.L2)
    assert m.metric == pxm.Metric.L2 and m.dim == 16
    m.add(np.zeros((4, 16), dtype=np.float32))
    assert m.memory_bytes == 4 * 16 * 4 and len(m) == m.size == 4


def test_engine_non_contiguous_input_not_corrupted(pxm, engine_data):
    for metric in (pxm.Metric.InnerProduct, pxm.Metric.L2):
        idx = pxm.FlatIndex(dim=64, metric=metric)
        idx.add(np.asfortranarray(engine_data))
        for i in (0, 123, 2999):
            ids, _ = idx.search(np.ascontiguousarray(engine_data[i]), k=1)
            assert ids[0] == i
    idx = pxm.FlatIndex(dim=64, metric=pxm.Metric.L2)
    idx.add(engine_data)
    strided = np.zeros(128, dtype=np.float32)[::2]
    strided[:] = engine_data[42]
    ids, _ = idx.search(strided, k=1)
    assert ids[0] == 42


# ---- the reference's C ABI (knn.cu / gpu.rs), called as gpu.rs does -------

@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_knn_gpu_abi_key_space(pxm, metric):
    lib = pxm._lib.load()
    n, dim, nq, k = 5000, 40, 11, 12
    data = O.gen_uniform(n, dim, 1)
    queries = O.gen_uniform(nq, dim, 2)
    f32p = ctypes.POINTER(ctypes.c_float)
    h = lib.knn_gpu_create(data.ctypes.data_as(f32p), n, dim)
    assert h
    try:
        ids = np.zeros(nq * k, np.int64)
        keys = np.zeros(nq * k, np.float32)
        rc = lib.knn_gpu_search(h, queries.ctypes.data_as(f32p), nq, k, metric,
                                ids.ctypes.data_as(ctypes.POINTER(ctypes.c_longlong)),
                                keys.ctypes.data_as(f32p))
        assert rc == 0
        assert lib.knn_gpu_search(h, queries.ctypes.data_as(f32p), nq, 0, metric, None, None) == -1
    finally:
        lib.knn_gpu_free(h)
    # gpu.rs:80-93 turns keys into natural distances.
    nat = np.sqrt(keys) if metric == O.L2 else -keys
    _parity.check_flat(data, metric, queries, ids.reshape(nq, k), nat.reshape(nq, k), k)


def test_multi_device_handle_if_available(pxm):
    ndev = pxm.device_count()
    if ndev < 2:
        pytest.skip("one GPU visible")
    data = O.gen_uniform(9001, 32, 41)
    queries = O.gen_uniform(13, 32, 42)
    idx = pxm.FlatIndex(32, pxm.Metric.L2, devices=list(range(min(ndev, 4))))
    idx.add(data[:5000])
    idx.add(data[5000:])
    ids, d = idx.search_batch(queries, k=10)
    _parity.check_flat(data, O.L2, queries, ids, d, 10)


# ---- the tensor-core path (K1 tcgen05 3xTF32 + K5 exact rescoring) --------

def _run_path(pxm, data, metric, queries, k, path):
    idx = pxm.FlatIndex(data.shape[1], _metric(pxm, metric))
    idx.add(data)
    idx.set_search_path(path)
    ids, d = idx.search_batch(queries, k=k)
    return ids, d, idx.last_search_profile()


@pytest.mark.parametrize("path", ["tensor", "tensor_3xtf32"])
@pytest.mark.parametrize("metric", [O.L2, O.IP])
@pytest.mark.parametrize("n,dim,nq,k", [
    (5000, 32, 16, 10), (20000, 64, 128, 10), (9000, 128, 300, 16), (12345, 24, 77, 1),
    (30000, 96, 200, 40), (8192, 768, 130, 10), (4096, 384, 129, 5),
    (20000, 64, 140, 100), (9000, 48, 33, 224), (12000, 128, 260, 41),
])
def test_tensor_path_parity(pxm, metric, n, dim, nq, k, path):
    data = _data.unit_gaussian(n, dim, n + dim) if metric == O.IP else \
        _data.gaussian_mixture(n, nq, d=dim, centres=50, seed=dim)[0]
    queries = _data.unit_gaussian(nq, dim, 7 * dim) if metric == O.IP else \
        _data.gaussian_mixture(10, nq, d=dim, centres=50, seed=dim)[1]
    ids, d, prof = _run_path(pxm, data, metric, queries, k, path)
    assert prof["path"] == "tensor"
    expected = "3xtf32" if path == "tensor_3xtf32" else ("bf16" if k <= 100 else "tf32")
    assert prof["first_pass"] == expected, prof
    _parity.check_flat(data, metric, queries, ids, d, k)
    # Exact-scan fallbacks are legal but must stay rare on generic data
    # (clustered L2 data leaves a few percent uncertified by the one-pass
    # candidates when too few fail for the three-pass refinement to pay).
    assert prof["fallback_queries"] <= max(4, nq // 10), prof


@pytest.mark.parametrize("dim", [96, 100, 29, 128, 62])
def test_tensor_path_l2_folded_norms(pxm, dim):
    # L2 at dim <= 256: the bf16 rows carry ||x||^2 after the dim columns
    # (in the padding, or in one more 64-column slice when the padding is
    # too short, as for 128 and 62) and the bf16 pass runs as an inner
    # product of 2q with them. Config 5's distribution certifies nearly
    # every query; rows far from the origin (norms ~1e8 against distances
    # ~1e2) make the folded sums large, and whatever the bound cannot
    # certify must come out exact through the fallback.
    data, queries = _data.gaussian_mixture(30000, 96, d=dim, centres=300, seed=dim)
    ids, d, prof = _run_path(pxm, data, O.L2, queries, 10, "tensor")
    assert prof["first_pass"] == "bf16"
    _parity.check_flat(data, O.L2, queries, ids, d, 10)
    assert prof["fallback_queries"] + prof["refined_queries"] <= max(4, len(queries) // 10), prof
    far = (data + np.float32(1000.0)).astype(np.float32)
    qfar = (queries + np.float32(1000.0)).astype(np.float32)
    ids, d, prof = _run_path(pxm, far, O.L2, qfar, 10, "tensor")
    _parity.check_flat(far, O.L2, qfar, ids, d, 10)


def test_tensor_path_integer_data_single_pass(pxm):
    # Config 2's integer data: the tf32 lo planes are zero, one MMA pass is exact.
    data, queries = _data.sift_like(40000, 64, seed=11, centres=100)
    ids, d, prof = _run_path(pxm, data, O.L2, queries, 10, "tensor")
    _parity.check_flat(data, O.L2, queries, ids, d, 10)


def test_tensor_path_certificate_fallback_on_ties(pxm):
    # Every row appears 40 times: ties exceed the candidate capacity, the
    # certificate cannot hold, and the exact scan must take over.
    base = _data.unit_gaussian(300, 64, 3)
    data = np.repeat(base, 40, axis=0)
    queries = _data.unit_gaussian(32, 64, 4)
    ids, d, prof = _run_path(pxm, data, O.IP, queries, 10, "tensor")
    assert prof["fallback_queries"] > 0
    _parity.check_flat(data, O.IP, queries, ids, d, 10)


def test_auto_path_uses_tensor_cores_for_batches(pxm):
    data = _data.unit_gaussian(20000, 128, 9)
    queries = _data.unit_gaussian(64, 128, 10)
    idx = pxm.FlatIndex(128, pxm.Metric.InnerProduct)
    idx.add(data)
    ids, d = idx.search_batch(queries, k=10)
    assert idx.last_search_profile()["path"] == "tensor"
    _parity.check_flat(data, O.IP, queries, ids, d, 10)
    ids1, d1 = idx.search(queries[5], k=10)
    assert idx.last_search_profile()["path"] == "exact"
    assert ids1.tolist() == ids[5].tolist()


def test_tensor_path_rejects_what_it_cannot_serve(pxm):
    idx = pxm.FlatIndex(16, pxm.Metric.L2)
    idx.add(O.gen_uniform(5000, 16, 1))
    idx.set_search_path("tensor")
    with pytest.raises(pxm.PxError):
        idx.search_batch(O.gen_uniform(32, 16, 2), k=225)


@pytest.mark.parametrize("metric", [O.L2, O.IP])
@pytest.mark.parametrize("k", [10, 100])
def test_tensor_path_filtered_parity(pxm, metric, k):
    n, dim, nq = 20000, 64, 48
    data = _data.unit_gaussian(n, dim, 17)
    queries = _data.unit_gaussian(nq, dim, 18)
    idx = pxm.FlatIndex(dim, _metric(pxm, metric))
    idx.add(data)
    idx.set_search_path("tensor")
    rng = np.random.default_rng(k)
    masks = [rng.random(n) < 0.3,                 # ordinary filter
             np.arange(n) < 50,                   # all admitted rows in one split
             (np.arange(n) % 997) == 0,           # fewer than k admitted rows for k=100
             np.zeros(n, bool)]                   # nothing admitted
    for mask in masks:
        ids, d = idx.search_batch_filtered(queries, mask, k=k)
        assert idx.last_search_profile()["path"] == "tensor"
        _parity.check_flat(data, metric, queries, ids, d, k, filter_=mask)


@pytest.mark.parametrize("path", ["exact", "tensor"])
@pytest.mark.parametrize("side_stream", [False, True])
def test_device_search_is_ordered_on_the_callers_stream(pxm, path, side_stream):
    # The queries are rewritten on the caller's stream behind a ~20 ms spin;
    # a search that ran on any other stream would read the stale queries.
    # torch's default stream has a null handle, which must mean CUDA's
    # default stream (not a private stream of the handle).
    import torch
    from proxima_b200 import _lib
    n, dim, nq, k = 20000, 64, 64, 10
    data = _data.unit_gaussian(n, dim, 31)
    q_old = _data.unit_gaussian(nq, dim, 32)
    q_new = _data.unit_gaussian(nq, dim, 33)
    idx = pxm.FlatIndex(dim, pxm.Metric.InnerProduct)
    idx.add(data)
    idx.set_search_path(path)
    dev = torch.device("cuda", 0)
    dq = torch.from_numpy(q_old).to(dev)
    src = torch.from_numpy(q_new).to(dev)
    ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
    dists = torch.empty((nq, k), dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.Stream(dev) if side_stream else torch.cuda.default_stream(dev)
    assert side_stream or stream.cuda_stream == 0
    with torch.cuda.stream(stream):
        torch.cuda._sleep(40_000_000)
        dq.copy_(src)
        _lib.check(_lib.load().px_flat_search_device(
            idx.handle, ctypes.c_void_p(dq.data_ptr()), nq, k, 0, ctypes.c_void_p(ids.data_ptr()),
            ctypes.c_void_p(dists.data_ptr()), ctypes.c_void_p(stream.cuda_stream)))
    stream.synchronize()
    assert idx.last_search_profile()["path"] == path
    _parity.check_flat(data, O.IP, q_new, ids.cpu().numpy(), dists.cpu().numpy(), k)


@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_tensor_path_three_tiers(pxm, metric):
    # Every row comes in 48 copies perturbed by 2e-4 per coordinate, so more
    # than the 32 candidates a list keeps sit within ~3e-4 of each other:
    # the one-pass bound (~1e-3) cannot certify them, the three-pass bound
    # (~2e-5) can. With 256 queries the three-pass refinement pays, and the
    # exact scan sees at most the few queries that are still uncertified.
    rng = np.random.default_rng(5)
    base = _data.unit_gaussian(800, 96, 6)
    data = np.repeat(base, 48, axis=0)
    data = (data + rng.standard_normal(data.shape).astype(np.float32) * np.float32(2e-4)).astype(np.float32)
    queries = _data.unit_gaussian(256, 96, 7)
    ids, d, prof = _run_path(pxm, data, metric, queries, 10, "tensor")
    _parity.check_flat(data, metric, queries, ids, d, 10)
    assert prof["refined_queries"] >= 200, prof
    assert prof["fallback_queries"] <= prof["refined_queries"] // 4, prof
    # Few uncertified queries go straight to the exact scan.
    ids, d, prof = _run_path(pxm, data, metric, queries[:20], 10, "tensor")
    _parity.check_flat(data, metric, queries[:20], ids, d, 10)
    assert prof["refined_queries"] == 0 and prof["fallback_queries"] > 0, prof


@pytest.mark.parametrize("metric", [O.L2, O.IP])
@pytest.mark.parametrize("n,nq,k", [(100, 300, 10), (257, 64, 16), (513, 257, 40), (1000, 513, 100)])
def test_tensor_path_tile_edges(pxm, metric, n, nq, k):
    # Shards shorter than one 256-row pair tile or one row past a tile, and
    # query counts one past a 256-query group: the tiles' tails, the padded
    # query rows and the (few) split lists all stay exact.
    dim = 64
    data = _data.unit_gaussian(n, dim, n + 11)
    queries = _data.unit_gaussian(nq, dim, nq + 13)
    ids, d, prof = _run_path(pxm, data, metric, queries, k, "tensor")
    assert prof["path"] == "tensor" and prof["first_pass"] == "bf16"
    _parity.check_flat(data, metric, queries, ids, d, k)


@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_tensor_path_filtered_large_k(pxm, metric):
    # k = 100 on the bf16 pass (32-candidate lists, 256 rescored) with filters.
    n, dim, nq, k = 30000, 96, 64, 100
    data = _data.unit_gaussian(n, dim, 41)
    queries = _data.unit_gaussian(nq, dim, 42)
    idx = pxm.FlatIndex(dim, _metric(pxm, metric))
    idx.add(data)
    idx.set_search_path("tensor")
    rng = np.random.default_rng(43)
    for mask in (rng.random(n) < 0.5, np.arange(n) % 7 == 0, np.arange(n) < 150):
        ids, d = idx.search_batch_filtered(queries, mask, k=k)
        assert idx.last_search_profile()["first_pass"] == "bf16"
        _parity.check_flat(data, metric, queries, ids, d, k, filter_=mask)


def test_small_batch_graph_replay(pxm):
    # Small batches on one device run as a replayed CUDA graph: new query
    # values, alternating shapes and k (several cached graphs), an add that
    # grows the index (the graph must be rebuilt) and the launch count.
    from proxima_b200 import _lib
    dim = 48
    data = _data.unit_gaussian(6000, dim, 71)
    idx = pxm.FlatIndex(dim, pxm.Metric.L2)
    idx.add(data[:4000])
    rng = np.random.default_rng(72)
    for step in range(6):
        nq, k = ((1, 10), (3, 5), (1, 10), (7, 32))[step % 4]
        q = rng.standard_normal((nq, dim)).astype(np.float32)
        before = _lib.launch_count()
        ids, d = idx.search_batch(q, k=k)
        assert idx.last_search_profile()["path"] == "exact"
        assert _lib.launch_count() - before == 3
        _parity.check_flat(data[:4000], O.L2, q, ids, d, k)
    idx.add(data[4000:])
    for _ in range(3):
        q = rng.standard_normal((1, dim)).astype(np.float32)
        ids, d = idx.search(q[0], k=10)
        _parity.check_flat(data, O.L2, q, ids[None, :], d[None, :], 10)
    # A query equal to a base row finds it at distance 0 in the grown index.
    ids, d = idx.search(data[4321], k=3)
    assert ids[0] == 4321 and d[0] == 0.0


# ---- the bf16 pass's sample pass ----------------------------------------------
# The bf16 pass can first run over 32 single tiles spread evenly over the
# shard; the 64th (k <= 16), 128th or 256th best key each query finds there is
# where its lists start, and rows above it are never offered. By default only
# shards with splits of 512+ tiles (millions of rows) take it; these tests
# force it on shards of 128+ tiles.

def _run_sampled(pxm, data, metric, queries, k, mode="on"):
    idx = pxm.FlatIndex(data.shape[1], _metric(pxm, metric))
    idx.add(data)
    idx.set_search_path("tensor")
    idx.set_sample_pass(mode)
    ids, d = idx.search_batch(queries, k=k)
    return ids, d, idx.last_search_profile()


@pytest.mark.parametrize("metric,dim,nq,k", [
    (O.IP, 64, 300, 10),    # two 8-entry lists per thread
    (O.L2, 96, 257, 10),    # folded norms in the padding
    (O.L2, 128, 64, 16),    # folded norms in one more K slice
    (O.IP, 384, 130, 1),
    (O.L2, 320, 100, 40),   # norm epilogue (dim > 256), 16-entry lists
    (O.IP, 48, 48, 100),    # the largest k of the bf16 pass
])
def test_tensor_path_sample_pass_parity(pxm, metric, dim, nq, k):
    n = 40000
    if metric == O.IP:
        data, queries = _data.unit_gaussian(n, dim, dim + 1), _data.unit_gaussian(nq, dim, dim + 2)
    else:
        data, queries = _data.gaussian_mixture(n, nq, d=dim, centres=200, seed=dim)
    ids, d, prof = _run_sampled(pxm, data, metric, queries, k)
    assert prof["first_pass"] == "bf16" and prof["sample_tiles"] == 32, prof
    _parity.check_flat(data, metric, queries, ids, d, k)
    # The clustered L2 cases leave some queries to the exact scan whether
    # or not the sample pass runs (11 of 64 and 11 of 100 here both ways:
    # the lists start from the sample's 64th or 128th key, above the merged
    # candidates' own bound).
    assert prof["fallback_queries"] <= max(4, nq // (10 if metric == O.IP else 5)), prof


def test_tensor_path_sample_pass_modes(pxm):
    short = _data.unit_gaussian(127 * 256, 32, 3)  # one tile short of the sample pass
    queries = _data.unit_gaussian(40, 32, 4)
    ids, d, prof = _run_sampled(pxm, short, O.IP, queries, 10, "on")
    assert prof["sample_tiles"] == 0, prof
    _parity.check_flat(short, O.IP, queries, ids, d, 10)
    data = _data.unit_gaussian(40000, 32, 5)  # 157 tiles in splits of a few tiles
    for mode, tiles in (("auto", 0), ("off", 0), ("on", 32)):
        ids, d, prof = _run_sampled(pxm, data, O.IP, queries, 10, mode)
        assert prof["sample_tiles"] == tiles, (mode, prof)
        _parity.check_flat(data, O.IP, queries, ids, d, 10)
    idx = pxm.FlatIndex(32)
    with pytest.raises(pxm.PxError, match="sample pass mode"):
        pxm._lib.check(pxm._lib.load().px_flat_set_sample_pass(idx.handle, 7))


@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_tensor_path_sample_pass_filtered(pxm, metric):
    # 160 tiles: the sample is tiles 0, 5, 10, ..., 155. The filter applies
    # to both passes: admitted rows only inside the sample, only outside it,
    # fewer than k, or none (a query whose sample holds fewer than k rows
    # starts with open lists).
    n, dim, nq, k = 40960, 64, 64, 10
    data = _data.unit_gaussian(n, dim, 51)
    queries = _data.unit_gaussian(nq, dim, 52)
    idx = pxm.FlatIndex(dim, _metric(pxm, metric))
    idx.add(data)
    idx.set_search_path("tensor")
    idx.set_sample_pass("on")
    tile = np.arange(n) // 256
    rng = np.random.default_rng(53)
    masks = [rng.random(n) < 0.3,
             np.arange(n) < 256,                      # sample tile 0 only
             tile % 5 != 0,                           # every tile but the sample's
             (tile % 5 == 3) & (rng.random(n) < 0.01),
             np.isin(np.arange(n), [7, 20000, 40959]),
             np.zeros(n, bool)]
    for mask in masks:
        ids, d = idx.search_batch_filtered(queries, mask, k=k)
        assert idx.last_search_profile()["sample_tiles"] == 32
        _parity.check_flat(data, metric, queries, ids, d, k, filter_=mask)


def test_tensor_path_sample_pass_ties(pxm):
    # Every row 40 times over 48,000 rows: the sample's k-th key is shared by
    # rows outside the sample, which are admitted too (a key equal to the
    # starting one passes), and the ties exceed the lists.
    base = _data.unit_gaussian(1200, 64, 61)
    data = np.repeat(base, 40, axis=0)
    queries = _data.unit_gaussian(32, 64, 62)
    ids, d, prof = _run_sampled(pxm, data, O.IP, queries, 10)
    assert prof["sample_tiles"] == 32, prof
    _parity.check_flat(data, O.IP, queries, ids, d, 10)


def test_profile_totals(pxm):
    # The totals a benchmark reads once after its loop: every search counted,
    # the profiled ones' kernel times summed, and a reset.
    data = _data.unit_gaussian(20000, 64, 81)
    queries = _data.unit_gaussian(64, 64, 82)
    idx = pxm.FlatIndex(64, pxm.Metric.InnerProduct)
    idx.add(data)
    idx.set_search_path("tensor")
    idx.search_batch(queries, k=10)
    idx.profile_totals(reset=True)
    pxm.set_profiling(True)
    try:
        times = []
        for _ in range(3):
            idx.search_batch(queries, k=10)
            times.append(idx.last_search_profile()["main_kernel_ms"])
        idx.set_search_path("exact")
        idx.search(queries[0], k=10)  # a small exact batch: profiled unless it replays a graph
        last = idx.last_search_profile()["main_kernel_ms"]
        if last is not None:
            times.append(last)
    finally:
        pxm.set_profiling(False)
    t = idx.profile_totals()
    assert t["searches"] == 4 and t["profiled_searches"] == len(times), (t, times)
    assert abs(t["main_kernel_ms"] - sum(times)) <= 1e-3 * sum(times) + 1e-6, (t, times)
    assert t["fallback_queries"] == 0 and t["refined_queries"] == 0
    assert idx.profile_totals(reset=True)["searches"] == 4
    assert idx.profile_totals()["searches"] == 0


def test_tensor_path_repeated_searches(pxm):
    # Repeated tensor-core searches reuse the handle's workspace and staging:
    # new query values, another k, an add (the rows move) and certificate
    # fallbacks on every repeat all stay exact.
    data = _data.unit_gaussian(24000, 64, 91)
    idx = pxm.FlatIndex(64, pxm.Metric.InnerProduct)
    idx.add(data[:18000])
    idx.set_search_path("tensor")
    for seed in (92, 93, 94):
        queries = _data.unit_gaussian(64, 64, seed)
        ids, d = idx.search_batch(queries, k=10)
        assert idx.last_search_profile()["path"] == "tensor"
        _parity.check_flat(data[:18000], O.IP, queries, ids, d, 10)
    ids, d = idx.search_batch(queries, k=16)
    _parity.check_flat(data[:18000], O.IP, queries, ids, d, 16)
    idx.add(data[18000:])
    ids, d = idx.search_batch(queries, k=10)
    _parity.check_flat(data, O.IP, queries, ids, d, 10)
    # Certificate fallbacks still run after a replay: duplicated rows defeat it.
    dup = np.repeat(data[:400], 40, axis=0)
    idx2 = pxm.FlatIndex(64, pxm.Metric.InnerProduct)
    idx2.add(dup)
    idx2.set_search_path("tensor")
    for _ in range(2):
        ids, d = idx2.search_batch(queries[:32], k=10)
        assert idx2.last_search_profile()["fallback_queries"] > 0
        _parity.check_flat(dup, O.IP, queries[:32], ids, d, 10)
