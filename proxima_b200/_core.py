"""Host-side mirror of the reference's ``proxima._core`` module.

Same classes, constructor signatures, defaults, return shapes and error types
as crates/py/src/lib.rs (``Metric`` :49-63, ``FlatIndex`` :65-230,
``PqIndex`` :440-683), but every index lives on the GPU and every search runs
the sm_100a kernels of libproxima_b200.so through its C ABI. Input handling
follows the PyO3 layer: arrays must be float32 numpy arrays of the right rank
(TypeError otherwise, as PyO3's ``PyReadonlyArray`` extraction raises), are
copied when not C-contiguous (``rows_c``/``vec_c`` :18-31), and non-finite
values raise ``ValueError`` (``check_finite`` :41-47).

Differences a user can observe: each constructor takes an optional
keyword-only ``devices`` list (CUDA ordinals the base is row-sharded across;
default: the current device), ``num_threads`` is accepted and ignored, and
``k`` above ``PX_MAX_K`` (768) raises ``ValueError``.
"""

from __future__ import annotations

import ctypes
import enum
import os
import struct

import numpy as np

from . import _lib
from ._lib import PX_MAX_K, PxError

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u8p = ctypes.POINTER(ctypes.c_uint8)


class Metric(enum.IntEnum):
    """Distance metric (crates/core/src/metric.rs:4; PyO3 enum lib.rs:49-54)."""

    L2 = 0
    InnerProduct = 1


def _metric_code(metric) -> int:
    if not isinstance(metric, Metric):
        raise TypeError(f"metric must be a Metric, got {type(metric).__name__}")
    return int(metric)


def _usize(x, name: str) -> int:
    if isinstance(x, bool) or not isinstance(x, (int, np.integer)):
        raise TypeError(f"argument '{name}': expected an integer")
    x = int(x)
    if x < 0:
        raise OverflowError(f"argument '{name}': can't convert negative int to unsigned")
    return x


def _array(a, ndim: int, dtype, name: str) -> np.ndarray:
    if not isinstance(a, np.ndarray) or a.ndim != ndim or a.dtype != dtype:
        raise TypeError(
            f"argument '{name}': expected a {ndim}-d numpy array of {np.dtype(dtype).name}")
    return np.ascontiguousarray(a)


def _check_finite(a: np.ndarray) -> None:
    if a.size and not np.isfinite(a).all():
        raise ValueError("input must not contain NaN or infinite values")


def _check_k(k: int) -> None:
    if k > PX_MAX_K:
        raise ValueError(f"k={k} exceeds the GPU limit PX_MAX_K={PX_MAX_K}")


def _devices_arg(devices):
    if devices is None:
        return None, 0
    devs = [int(d) for d in devices]
    arr = (ctypes.c_int32 * len(devs))(*devs)
    return arr, len(devs)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class FlatIndex:
    """Exact brute-force index (crates/core/src/flat.rs:35-231) on the GPU."""

    def __init__(self, dim, metric=Metric.InnerProduct, *, devices=None):
        dim = _usize(dim, "dim")
        if dim == 0:
            raise ValueError("dim must be > 0")
        self._lib = _lib.load()
        self._dim = dim
        self._metric = Metric(_metric_code(metric))
        arr, nd = _devices_arg(devices)
        h = ctypes.c_void_p()
        _lib.check(self._lib.px_flat_create(dim, int(self._metric), arr, nd, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self._lib.px_flat_destroy(h)
            self._h = None

    # -- lib.rs:81-94 ------------------------------------------------------
    def add(self, vectors) -> None:
        v = _array(vectors, 2, np.float32, "vectors")
        if v.shape[1] != self._dim:
            raise ValueError(f"vector dim {v.shape[1]} does not match index dim {self._dim}")
        _check_finite(v)
        _lib.check(self._lib.px_flat_add(self._h, _ptr(v, _f32p), v.shape[0]))

    def read_rows(self, start: int, count: int) -> np.ndarray:
        """Rows [start, start + count) in id order, copied back from the GPU."""
        out = np.empty((count, self._dim), dtype=np.float32)
        if count:
            _lib.check(self._lib.px_flat_read_rows(self._h, start, count, _ptr(out, _f32p)))
        return out

    # -- lib.rs:219-226 (bincode .sfidx files, see persist.py) -------------
    def save(self, path) -> None:
        from .persist import save_flat
        save_flat(self, os.fspath(path))

    @staticmethod
    def load(path, *, devices=None) -> "FlatIndex":
        from .persist import load_flat
        return load_flat(FlatIndex, os.fspath(path), devices=devices)

    def reserve(self, n_total: int) -> None:
        """Pre-sizes device storage for n_total rows (no reallocation on add)."""
        _lib.check(self._lib.px_flat_reserve(self._h, _usize(n_total, "n_total")))

    def _search(self, q: np.ndarray, nq: int, k: int, mask=None):
        ids = np.zeros((nq, k), dtype=np.int64)
        dists = np.zeros((nq, k), dtype=np.float32)
        if k == 0 or nq == 0:
            return ids, dists
        _check_k(k)
        if mask is None:
            st = self._lib.px_flat_search(self._h, _ptr(q, _f32p), nq, k, _ptr(ids, _i64p),
                                          _ptr(dists, _f32p))
        else:
            m = np.ascontiguousarray(mask, dtype=np.uint8)
            st = self._lib.px_flat_search_filtered(self._h, _ptr(q, _f32p), nq, k, _ptr(m, _u8p),
                                                   _ptr(ids, _i64p), _ptr(dists, _f32p))
        _lib.check(st)
        return ids, dists

    # -- lib.rs:96-112 -----------------------------------------------------
    def search(self, query, k=10):
        q = _array(query, 1, np.float32, "query")
        k = _usize(k, "k")
        if q.shape[0] != self._dim:
            raise ValueError("query dim mismatch")
        _check_finite(q)
        ids, dists = self._search(q, 1, k)
        return ids[0], dists[0]

    # -- lib.rs:114-139 ----------------------------------------------------
    def search_batch(self, queries, k=10, num_threads=0):
        q = _array(queries, 2, np.float32, "queries")
        k = _usize(k, "k")
        _usize(num_threads, "num_threads")
        if q.shape[1] != self._dim:
            raise ValueError("query dim mismatch")
        _check_finite(q)
        return self._search(q, q.shape[0], k)

    def _mask(self, mask) -> np.ndarray:
        m = _array(mask, 1, np.bool_, "mask")
        if m.shape[0] != self.size:
            raise ValueError(f"mask length {m.shape[0]} must equal index size {self.size}")
        return m

    # -- lib.rs:141-164 ----------------------------------------------------
    def search_filtered(self, query, mask, k=10):
        q = _array(query, 1, np.float32, "query")
        k = _usize(k, "k")
        if q.shape[0] != self._dim:
            raise ValueError("query dim mismatch")
        m = self._mask(mask)
        _check_finite(q)
        ids, dists = self._search(q, 1, k, m)
        return ids[0], dists[0]

    # -- lib.rs:166-198 ----------------------------------------------------
    def search_batch_filtered(self, queries, mask, k=10, num_threads=0):
        q = _array(queries, 2, np.float32, "queries")
        k = _usize(k, "k")
        _usize(num_threads, "num_threads")
        if q.shape[1] != self._dim:
            raise ValueError("query dim mismatch")
        m = self._mask(mask)
        _check_finite(q)
        return self._search(q, q.shape[0], k, m)

    # -- lib.rs:200-229 ----------------------------------------------------
    @property
    def size(self) -> int:
        return int(self._lib.px_flat_size(self._h))

    @property
    def dim(self) -> int:
        return self._dim

    @property
    def metric(self) -> Metric:
        return self._metric

    @property
    def memory_bytes(self) -> int:
        # flat.rs:60-62: the f32 payload of the stored rows.
        return self.size * self._dim * 4

    def __len__(self) -> int:
        return self.size

    @property
    def handle(self) -> ctypes.c_void_p:
        """The px_flat* handle (for callers that drive the C ABI directly)."""
        return self._h

    _PATHS = {"auto": 0, "exact": 1, "tensor": 2, "tensor_3xtf32": 3}

    def set_search_path(self, path: str) -> None:
        """Kernel path for searches: "auto" (default), "exact" (streaming
        scan), "tensor" (tcgen05 candidates -- bf16 for k <= 100, tf32 above --
        then exact rescoring) or "tensor_3xtf32" (the same with ~fp32-accurate
        3xTF32 candidates). Results are identical on every path; this only
        changes speed."""
        _lib.check(self._lib.px_flat_set_path(self._h, self._PATHS[path]))

    _SAMPLE = {"auto": 0, "off": 1, "on": 2}

    def set_sample_pass(self, mode: str) -> None:
        """The bf16 pass's sample pass: "auto" (default: shards of at least
        128 tiles whose splits are at least 512 tiles long), "on" (every
        shard of at least 128 tiles) or "off". Results are identical either
        way; this only changes speed."""
        _lib.check(self._lib.px_flat_set_sample_pass(self._h, self._SAMPLE[mode]))

    def profile_totals(self, reset: bool = False) -> dict:
        """Totals over this index's searches since the last reset: the summed
        device time of the profiled searches' dominant kernel, their count,
        all searches, and the queries sent to the refinement and the exact
        scan. reset=True zeroes them after reading."""
        t = _lib.ProfileTotals()
        _lib.check(self._lib.px_flat_profile_totals(self._h, 1 if reset else 0, ctypes.byref(t)))
        return {"main_kernel_ms": t.main_kernel_ms, "profiled_searches": t.profiled_searches,
                "searches": t.searches, "fallback_queries": t.fallback_queries,
                "refined_queries": t.refined_queries}

    def last_search_profile(self) -> dict:
        """Path, kernel launches, queries the certificate sent to the
        three-pass refinement and to the exact scan, and (when profiling is
        on, see proxima_b200.set_profiling) the dominant kernel's device time
        of the last search."""
        prof = _lib.SearchProfile()
        _lib.check(self._lib.px_flat_last_profile(self._h, ctypes.byref(prof)))
        return {"path": ("exact", "tensor")[prof.path], "launches": prof.launches,
                "fallback_queries": prof.fallback_queries, "refined_queries": prof.refined_queries,
                "first_pass": {0: "3xtf32", 1: "tf32", 2: "bf16"}.get(prof.first_pass),
                "sample_tiles": prof.sample_tiles,
                "main_kernel_ms": prof.main_kernel_ms if prof.profiled else None}


class PqIndex:
    """Product-quantized index (crates/core/src/pq.rs:218-396) on the GPU."""

    def __init__(self, dim, metric=Metric.InnerProduct, m=8, nbits=8, train_iters=25,
                 train_sample=50000, seed=24301, *, devices=None):
        dim = _usize(dim, "dim")
        m = _usize(m, "m")
        nbits = _usize(nbits, "nbits")
        train_iters = _usize(train_iters, "train_iters")
        train_sample = _usize(train_sample, "train_sample")
        seed = _usize(seed, "seed")
        # lib.rs:455-463
        if m == 0:
            raise ValueError("m must be >= 1")
        if dim == 0 or dim % m != 0:
            raise ValueError("dim must be > 0 and divisible by m")
        if not 1 <= nbits <= 8:
            raise ValueError("nbits must be in 1..=8")
        self._lib = _lib.load()
        self._dim = dim
        self._metric = Metric(_metric_code(metric))
        self._m = m
        self._nbits = nbits
        self._train_iters = train_iters
        self._train_sample = train_sample
        self._seed = seed & 0xFFFFFFFFFFFFFFFF
        self._devices = None if devices is None else [int(d) for d in devices]
        self._h = None
        self._books = None

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self._lib.px_pq_destroy(h)
            self._h = None

    @property
    def handle(self) -> ctypes.c_void_p:
        """The px_pq* handle (for callers that drive the C ABI directly);
        None until the index is trained."""
        return self._h

    # -- lib.rs:472-490 ----------------------------------------------------
    def train(self, training) -> None:
        t = _array(training, 2, np.float32, "training")
        if t.shape[1] != self._dim:
            raise ValueError("training dim mismatch")
        ksub = 1 << self._nbits
        if t.shape[0] < ksub:
            raise ValueError(
                f"training set too small: need at least {ksub} rows for nbits={self._nbits}, "
                f"got {t.shape[0]}")
        _check_finite(t)
        books = np.zeros((self._m, ksub, self._dim // self._m), dtype=np.float32)
        dev = self._devices[0] if self._devices else -1
        _lib.check(self._lib.px_pq_train(_ptr(t, _f32p), t.shape[0], self._dim, self._m,
                                         self._nbits, self._train_iters, self._train_sample,
                                         ctypes.c_uint64(self._seed), dev, _ptr(books, _f32p)))
        self._set_codebooks(books)

    def _set_codebooks(self, books: np.ndarray) -> None:
        if self._h is not None:
            self._lib.px_pq_destroy(self._h)
            self._h = None
        arr, nd = _devices_arg(self._devices)
        h = ctypes.c_void_p()
        books = np.ascontiguousarray(books, dtype=np.float32)
        _lib.check(self._lib.px_pq_create(self._dim, self._m, self._nbits, int(self._metric),
                                          _ptr(books, _f32p), arr, nd, ctypes.byref(h)))
        self._h = h
        self._books = books

    def _trained(self, msg: str):
        if self._h is None:
            raise ValueError(msg)

    # -- lib.rs:492-504 ----------------------------------------------------
    def add(self, vectors) -> None:
        self._trained("index is not trained; call train() first")
        v = _array(vectors, 2, np.float32, "vectors")
        if v.shape[1] != self._dim:
            raise ValueError("vector dim mismatch")
        _check_finite(v)
        _lib.check(self._lib.px_pq_add(self._h, _ptr(v, _f32p), v.shape[0]))

    def add_codes(self, codes) -> None:
        """Appends pre-encoded codes (n x m uint8)."""
        self._trained("index is not trained; call train() first")
        c = _array(codes, 2, np.uint8, "codes")
        if c.shape[1] != self._m:
            raise ValueError("code width must equal m")
        _lib.check(self._lib.px_pq_add_codes(self._h, _ptr(c, _u8p), c.shape[0]))

    def read_codes(self, start: int, count: int) -> np.ndarray:
        """Codes of rows [start, start + count), copied back from the GPU."""
        self._trained("index is not trained")
        out = np.empty((count, self._m), dtype=np.uint8)
        if count:
            _lib.check(self._lib.px_pq_read_codes(self._h, start, count, _ptr(out, _u8p)))
        return out

    # -- lib.rs:662-679 (bincode .sfidx files, see persist.py) -------------
    def save(self, path) -> None:
        self._trained("index is not trained")
        from .persist import save_pq
        save_pq(self, os.fspath(path))

    @staticmethod
    def load(path, *, devices=None) -> "PqIndex":
        from .persist import load_pq
        return load_pq(PqIndex, os.fspath(path), devices=devices)

    def encode(self, vectors) -> np.ndarray:
        """ProductQuantizer::encode_into for each row (pq.rs:107-121)."""
        self._trained("index is not trained")
        v = _array(vectors, 2, np.float32, "vectors")
        if v.shape[1] != self._dim:
            raise ValueError("vector dim mismatch")
        _check_finite(v)
        out = np.zeros((v.shape[0], self._m), dtype=np.uint8)
        _lib.check(self._lib.px_pq_encode(self._h, _ptr(v, _f32p), v.shape[0], _ptr(out, _u8p)))
        return out

    def _search(self, q, nq, k, mask=None):
        ids = np.zeros((nq, k), dtype=np.int64)
        dists = np.zeros((nq, k), dtype=np.float32)
        if k == 0 or nq == 0:
            return ids, dists
        _check_k(k)
        if mask is None:
            st = self._lib.px_pq_search(self._h, _ptr(q, _f32p), nq, k, _ptr(ids, _i64p),
                                        _ptr(dists, _f32p))
        else:
            m = np.ascontiguousarray(mask, dtype=np.uint8)
            st = self._lib.px_pq_search_filtered(self._h, _ptr(q, _f32p), nq, k, _ptr(m, _u8p),
                                                 _ptr(ids, _i64p), _ptr(dists, _f32p))
        _lib.check(st)
        return ids, dists

    # -- lib.rs:506-526 ----------------------------------------------------
    def search(self, query, k=10):
        self._trained("index is not trained")
        q = _array(query, 1, np.float32, "query")
        k = _usize(k, "k")
        if q.shape[0] != self._dim:
            raise ValueError("query dim mismatch")
        _check_finite(q)
        ids, dists = self._search(q, 1, k)
        return ids[0], dists[0]

    # -- lib.rs:528-555 ----------------------------------------------------
    def search_batch(self, queries, k=10, num_threads=0):
        self._trained("index is not trained")
        q = _array(queries, 2, np.float32, "queries")
        k = _usize(k, "k")
        _usize(num_threads, "num_threads")
        if q.shape[1] != self._dim:
            raise ValueError("query dim mismatch")
        _check_finite(q)
        return self._search(q, q.shape[0], k)

    def _mask(self, mask):
        m = _array(mask, 1, np.bool_, "mask")
        if m.shape[0] != self.size:
            raise ValueError(f"mask length {m.shape[0]} must equal index size {self.size}")
        return m

    # -- lib.rs:557-584 ----------------------------------------------------
    def search_filtered(self, query, mask, k=10):
        self._trained("index is not trained")
        q = _array(query, 1, np.float32, "query")
        k = _usize(k, "k")
        if q.shape[0] != self._dim:
            raise ValueError("query dim mismatch")
        m = self._mask(mask)
        _check_finite(q)
        ids, dists = self._search(q, 1, k, m)
        return ids[0], dists[0]

    # -- lib.rs:586-622 ----------------------------------------------------
    def search_batch_filtered(self, queries, mask, k=10, num_threads=0):
        self._trained("index is not trained")
        q = _array(queries, 2, np.float32, "queries")
        k = _usize(k, "k")
        _usize(num_threads, "num_threads")
        if q.shape[1] != self._dim:
            raise ValueError("query dim mismatch")
        m = self._mask(mask)
        _check_finite(q)
        return self._search(q, q.shape[0], k, m)

    # -- lib.rs:624-661 ----------------------------------------------------
    @property
    def is_trained(self) -> bool:
        return self._h is not None

    @property
    def size(self) -> int:
        return int(self._lib.px_pq_size(self._h)) if self._h is not None else 0

    @property
    def dim(self) -> int:
        return self._dim

    @property
    def m(self) -> int:
        return self._m

    @property
    def metric(self) -> Metric:
        return self._metric

    def last_search_profile(self) -> dict:
        """Kernel launches and (with profiling on) the ADC scan's device time
        of the last search."""
        self._trained("index is not trained")
        prof = _lib.SearchProfile()
        _lib.check(self._lib.px_pq_last_profile(self._h, ctypes.byref(prof)))
        return {"path": "pq", "launches": prof.launches,
                "main_kernel_ms": prof.main_kernel_ms if prof.profiled else None}

    @property
    def codebooks(self) -> np.ndarray:
        """The trained codebooks, shape (m, 2**nbits, dim // m)."""
        self._trained("index is not trained")
        return self._books.copy()

    @property
    def memory_bytes(self) -> int:
        # pq.rs:250-252: code bytes + codebook floats.
        if self._h is None:
            return 0
        return self.size * self._m + self._books.size * 4

    @property
    def raw_bytes(self) -> int:
        return self.size * self._dim * 4

    @property
    def compression_ratio(self) -> float:
        mb = self.memory_bytes
        return self.raw_bytes / mb if mb > 0 else 0.0

    def __len__(self) -> int:
        return self.size


__all__ = ["Metric", "FlatIndex", "PqIndex", "PxError", "PX_MAX_K"]
