"""The reference's own CUDA kernel (crates/core/cuda/knn.cu), run live.

oracle/_ref/libknn_ref.so is the reference's knn_gpu_* compiled unchanged
(oracle/Makefile). Two uses, both as a checker and a floor, never as the
product:

1. an independent check of the oracle's FlatIndex::search_batch on config 2's
   integer-valued distribution, where the kernel's sequential sums and the
   CPU's 8-lane sums are exactly equal (every partial sum is an integer below
   2^24): keys bit for bit, ids except at exact ties;
2. the same-box floor on config 2's shape (1,000,000 x 128, 1,000 queries,
   k = 10): queries per second of the reference kernel and of this library,
   both called host to host through their C ABIs (printed with -s).
"""

import time

import numpy as np
import pytest

import oracle as O
from tests import _data

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_lib(px, oracle_lib):
    assert px.device_count() > 0, "GPU tests need a CUDA device"
    if not O.ref_knn_available():
        pytest.skip("oracle/_ref/libknn_ref.so was not built (no reference tree at build time)")
    return O


def _key_space(data, metric, queries, ids):
    return np.stack([O.flat_keys(data, metric, queries[q], ids[q]) for q in range(len(queries))])


def _tie_aware_equal(ref_ids, ref_keys, ids, keys):
    assert np.array_equal(ref_keys.view(np.uint32), keys.view(np.uint32))
    for q in range(len(ids)):
        for j in np.nonzero(ids[q] != ref_ids[q])[0]:
            assert np.count_nonzero(keys[q] == keys[q, j]) > 1 or keys[q, j] == keys[q, -1], (q, j)


@pytest.mark.parametrize("metric", [O.L2, O.IP])
@pytest.mark.parametrize("k", [1, 10, 46])
def test_oracle_matches_reference_kernel_on_integer_data(ref_lib, metric, k):
    base, queries = _data.sift_like(30000, 37, seed=5, centres=60)
    ref = O.RefKnn(base)
    ref_ids, ref_keys = ref.search(queries, k, metric)
    ref.close()
    ids, _ = O.flat_search_batch(base, metric, queries, k)
    _tie_aware_equal(ref_ids, ref_keys, ids, _key_space(base, metric, queries, ids))


def test_same_box_floor_config2_shape(ref_lib, px):
    base, queries = _data.sift_like(1_000_000, 1000, seed=2, centres=1000)
    k = 10
    ref = O.RefKnn(base)
    ref.search(queries[:8], k, O.L2)  # warm-up
    t = time.perf_counter()
    ref_ids, ref_keys = ref.search(queries, k, O.L2)
    t_ref = time.perf_counter() - t
    ref.close()
    idx = px.FlatIndex(128, px.Metric.L2)
    idx.add(base)
    idx.search_batch(queries, k=k)  # warm-up
    t = time.perf_counter()
    ids, d = idx.search_batch(queries, k=k)
    t_px = time.perf_counter() - t
    # Same answers (squared distances of integer data are exact on both).
    _tie_aware_equal(ref_ids, ref_keys, ids, _key_space(base, O.L2, queries, ids))
    print(f"config 2 shape, k=10, host to host: reference knn_kernel {len(queries) / t_ref:.0f} QPS "
          f"({t_ref * 1e3:.1f} ms); proxima_b200 {len(queries) / t_px:.0f} QPS ({t_px * 1e3:.2f} ms); "
          f"ratio {t_ref / t_px:.1f}x")
