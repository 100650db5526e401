"""ctypes bindings of the C++ oracle (test infrastructure only).

Every function here mirrors one function of oracle.cpp, which in turn cites
the reference line it restates.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

L2 = 0
IP = 1

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_u64p = ctypes.POINTER(ctypes.c_uint64)


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile if it is missing or stale."""
    src = os.path.join(_HERE, "oracle.cpp")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.ox_gen_uniform.argtypes = [ctypes.c_uint64, ctypes.c_int64, _f32p]
        L.ox_splitmix_next.argtypes = [_u64p]
        L.ox_splitmix_next.restype = ctypes.c_uint64
        L.ox_l2_sqr.argtypes = [_f32p, _f32p, ctypes.c_int64]
        L.ox_l2_sqr.restype = ctypes.c_float
        L.ox_inner_product.argtypes = [_f32p, _f32p, ctypes.c_int64]
        L.ox_inner_product.restype = ctypes.c_float
        L.ox_flat_keys.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, _f32p,
                                   _i64p, ctypes.c_int64, _f32p]
        L.ox_flat_search.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, _f32p,
                                     ctypes.c_int64, _u8p, _i64p, _f32p]
        L.ox_flat_search_batch.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                           _f32p, ctypes.c_int64, ctypes.c_int64, _u8p, _i64p,
                                           _f32p, ctypes.c_int32]
        L.ox_pq_train.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint64,
                                  _f32p]
        L.ox_kmeans.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                ctypes.c_int64, ctypes.c_uint64, _f32p]
        L.ox_pq_encode.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _f32p,
                                   ctypes.c_int64, _u8p]
        L.ox_pq_adc_table.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int32, _f32p, _f32p]
        L.ox_pq_search.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_int32, _u8p, ctypes.c_int64, _f32p, ctypes.c_int64,
                                   _u8p, _i64p, _f32p]
        L.ox_pq_search_batch.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int32, _u8p, ctypes.c_int64, _f32p,
                                         ctypes.c_int64, ctypes.c_int64, _u8p, _i64p, _f32p,
                                         ctypes.c_int32]
        L.ox_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _f(a):
    return a.ctypes.data_as(_f32p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _mask(filter_):
    if filter_ is None:
        return None, None
    m = np.ascontiguousarray(filter_, dtype=np.uint8)
    return m, m.ctypes.data_as(_u8p)


def max_threads() -> int:
    return int(lib().ox_max_threads())


def gen_uniform(n: int, dim: int, seed: int) -> np.ndarray:
    """The reference tests' SplitMix generator (flat.rs:238-250), shape (n, dim)."""
    out = np.empty(n * dim, dtype=np.float32)
    lib().ox_gen_uniform(ctypes.c_uint64(seed), out.size, _f(out))
    return out.reshape(n, dim)


def l2_sqr(a, b) -> float:
    a = _c(a, np.float32)
    b = _c(b, np.float32)
    assert a.size == b.size, "l2_sqr: mismatched vector lengths"
    return float(lib().ox_l2_sqr(_f(a), _f(b), a.size))


def inner_product(a, b) -> float:
    a = _c(a, np.float32)
    b = _c(b, np.float32)
    assert a.size == b.size, "inner_product: mismatched vector lengths"
    return float(lib().ox_inner_product(_f(a), _f(b), a.size))


def flat_keys(data, metric: int, query, ids=None) -> np.ndarray:
    """Exact reference keys (squared L2 or -IP) of query against rows `ids`."""
    data = _c(data, np.float32)
    query = _c(query, np.float32)
    n, dim = data.shape
    if ids is None:
        count, idp = n, None
    else:
        ids = _c(ids, np.int64)
        count, idp = ids.size, ids.ctypes.data_as(_i64p)
    out = np.empty(count, dtype=np.float32)
    lib().ox_flat_keys(_f(data), n, dim, metric, _f(query), idp, count, _f(out))
    return out


def flat_search(data, metric: int, query, k: int, filter_=None):
    data = _c(data, np.float32)
    query = _c(query, np.float32)
    n, dim = data.shape
    ids = np.zeros(k, dtype=np.int64)
    dists = np.zeros(k, dtype=np.float32)
    _, mp = _mask(filter_)
    lib().ox_flat_search(_f(data), n, dim, metric, _f(query), k, mp,
                         ids.ctypes.data_as(_i64p), _f(dists))
    return ids, dists


def flat_search_batch(data, metric: int, queries, k: int, filter_=None, num_threads: int = 0):
    data = _c(data, np.float32)
    queries = _c(queries, np.float32)
    n, dim = data.shape
    nq = queries.shape[0]
    ids = np.zeros((nq, k), dtype=np.int64)
    dists = np.zeros((nq, k), dtype=np.float32)
    _, mp = _mask(filter_)
    lib().ox_flat_search_batch(_f(data), n, dim, metric, _f(queries), nq, k, mp,
                               ids.ctypes.data_as(_i64p), _f(dists), num_threads)
    return ids, dists


def pq_train(training, m: int, nbits: int = 8, train_iters: int = 25, train_sample: int = 50000,
             seed: int = 0x5EED) -> np.ndarray:
    training = _c(training, np.float32)
    n, dim = training.shape
    ksub = 1 << nbits
    books = np.zeros((m, ksub, dim // m), dtype=np.float32)
    lib().ox_pq_train(_f(training), n, dim, m, nbits, train_iters, train_sample,
                      ctypes.c_uint64(seed), _f(books))
    return books


def kmeans(data, k: int, iters: int, seed: int) -> np.ndarray:
    data = _c(data, np.float32)
    n, d = data.shape
    out = np.zeros((k, d), dtype=np.float32)
    lib().ox_kmeans(_f(data), n, d, k, iters, ctypes.c_uint64(seed), _f(out))
    return out


def pq_encode(books, vectors) -> np.ndarray:
    books = _c(books, np.float32)
    vectors = _c(vectors, np.float32)
    m, ksub, dsub = books.shape
    n, dim = vectors.shape
    out = np.zeros((n, m), dtype=np.uint8)
    lib().ox_pq_encode(_f(books), dim, m, ksub, _f(vectors), n, out.ctypes.data_as(_u8p))
    return out


def pq_adc_table(books, metric: int, query) -> np.ndarray:
    books = _c(books, np.float32)
    query = _c(query, np.float32)
    m, ksub, dsub = books.shape
    out = np.zeros((m, ksub), dtype=np.float32)
    lib().ox_pq_adc_table(_f(books), m * dsub, m, ksub, metric, _f(query), _f(out))
    return out


def pq_search_batch(books, metric: int, codes, queries, k: int, filter_=None,
                    num_threads: int = 0):
    books = _c(books, np.float32)
    codes = _c(codes, np.uint8)
    queries = _c(queries, np.float32)
    m, ksub, dsub = books.shape
    n = codes.shape[0]
    nq = queries.shape[0]
    ids = np.zeros((nq, k), dtype=np.int64)
    dists = np.zeros((nq, k), dtype=np.float32)
    _, mp = _mask(filter_)
    lib().ox_pq_search_batch(_f(books), m * dsub, m, ksub, metric, codes.ctypes.data_as(_u8p), n,
                             _f(queries), nq, k, mp, ids.ctypes.data_as(_i64p), _f(dists),
                             num_threads)
    return ids, dists


def check_topk(metric: int, data, queries, ids, dists, ref_ids, ref_dists, *, filter_=None):
    """Tie-aware parity check of a top-k result against the oracle's.

    The rule (ids identical except where distances tie): the k distances must
    equal the oracle's bit for bit, rank by rank; every returned id must be a
    distinct row whose own exact distance (recomputed here) equals the
    distance reported beside it; and a rank may carry a different id than the
    oracle only where that rank's distance also occurs at another rank or at
    the k-th boundary (an exact tie). Returns the number of rank positions
    whose id differs from the oracle's (all of them ties).
    """
    ids = np.asarray(ids).reshape(ref_ids.shape)
    dists = np.asarray(dists, dtype=np.float32).reshape(ref_dists.shape)
    nq, k = ref_ids.shape
    if not np.array_equal(dists.view(np.uint32), ref_dists.view(np.uint32)):
        bad = np.argwhere(dists.view(np.uint32) != ref_dists.view(np.uint32))
        q, j = bad[0]
        raise AssertionError(
            f"distance mismatch at query {q} rank {j}: got {dists[q, j]!r} want {ref_dists[q, j]!r}"
            f" ({len(bad)} positions differ)")
    data = _c(data, np.float32)
    n_tie = 0
    for q in range(nq):
        row_ids = ids[q]
        valid = row_ids >= 0
        if not np.array_equal(valid, ref_ids[q] >= 0):
            raise AssertionError(f"padding mismatch at query {q}: {row_ids} vs {ref_ids[q]}")
        got = row_ids[valid]
        if len(set(got.tolist())) != got.size:
            raise AssertionError(f"duplicate ids at query {q}: {row_ids}")
        if filter_ is not None and not np.all(np.asarray(filter_)[got]):
            raise AssertionError(f"filtered-out id returned at query {q}")
        keys = flat_keys(data, metric, queries[q], got)
        nat = np.sqrt(keys) if metric == L2 else -keys
        if not np.array_equal(nat.astype(np.float32).view(np.uint32),
                              dists[q][valid].view(np.uint32)):
            raise AssertionError(f"reported distances do not match the ids' exact distances at query {q}")
        diff = np.nonzero(row_ids != ref_ids[q])[0]
        for j in diff:
            d = dists[q, j]
            tied = np.count_nonzero(dists[q] == d) > 1 or d == dists[q, -1]
            if not tied:
                raise AssertionError(
                    f"id mismatch at query {q} rank {j} without a tie: {row_ids[j]} vs {ref_ids[q, j]}")
        n_tie += diff.size
    return n_tie


# ---- the reference's own CUDA kernel (crates/core/cuda/knn.cu) -------------
# Built unchanged by `make -C oracle _ref/libknn_ref.so` from the reference
# tree (when it is present); the built library travels with the repository to
# a GPU host. A second, independent checker of the oracle's flat search, and
# a same-box floor. Never used by the product.

_REF_KNN_PATH = os.path.join(_HERE, "_ref", "libknn_ref.so")
_REF_SRC = os.environ.get("PX_REFERENCE_TREE", "/root/reference")
_ref_lib = None


def build_ref(force: bool = False) -> str | None:
    """Compile _ref/libknn_ref.so from the reference tree if that tree is here."""
    src = os.path.join(_REF_SRC, "crates", "core", "cuda", "knn.cu")
    if not os.path.exists(src):
        return _REF_KNN_PATH if os.path.exists(_REF_KNN_PATH) else None
    if force or not os.path.exists(_REF_KNN_PATH) or os.path.getmtime(_REF_KNN_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "_ref/libknn_ref.so", f"REF={_REF_SRC}"], check=True)
    return _REF_KNN_PATH


def ref_knn_available() -> bool:
    return os.path.exists(_REF_KNN_PATH)


def ref_knn_lib():
    """ctypes handle of the reference's knn_gpu_* (signatures of gpu.rs:10-15)."""
    global _ref_lib
    if _ref_lib is None:
        L = ctypes.CDLL(_REF_KNN_PATH)
        L.knn_gpu_create.argtypes = [_f32p, ctypes.c_int, ctypes.c_int]
        L.knn_gpu_create.restype = ctypes.c_void_p
        L.knn_gpu_search.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.POINTER(ctypes.c_longlong), _f32p]
        L.knn_gpu_search.restype = ctypes.c_int
        L.knn_gpu_free.argtypes = [ctypes.c_void_p]
        L.knn_gpu_free.restype = None
        _ref_lib = L
    return _ref_lib


class RefKnn:
    """The reference GPU index: knn_gpu_create / search / free (knn.cu:123-180).
    Returns KEY-SPACE values (squared L2, or -inner product) as the kernel
    writes them; k <= 46 (knn.cu:5)."""

    def __init__(self, base: np.ndarray):
        b = np.ascontiguousarray(base, dtype=np.float32)
        self.dim = b.shape[1]
        self.h = ref_knn_lib().knn_gpu_create(b.ctypes.data_as(_f32p), b.shape[0], self.dim)
        if not self.h:
            raise RuntimeError("knn_gpu_create failed")

    def search(self, queries: np.ndarray, k: int, metric: int):
        q = np.ascontiguousarray(queries, dtype=np.float32)
        ids = np.empty((q.shape[0], k), dtype=np.int64)
        keys = np.empty((q.shape[0], k), dtype=np.float32)
        rc = ref_knn_lib().knn_gpu_search(self.h, q.ctypes.data_as(_f32p), q.shape[0], k, metric,
                                          ids.ctypes.data_as(ctypes.POINTER(ctypes.c_longlong)),
                                          keys.ctypes.data_as(_f32p))
        if rc != 0:
            raise RuntimeError(f"knn_gpu_search returned {rc}")
        return ids, keys

    def close(self):
        if self.h:
            ref_knn_lib().knn_gpu_free(self.h)
            self.h = None

    def __del__(self):
        self.close()
