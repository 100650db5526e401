"""C-ABI checks that need no GPU: the library loads, exports every symbol
include/*.h declares, and fails cleanly (status + message, no abort) when no
CUDA device is present."""

import ctypes
import glob
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        names += re.findall(r"PX_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_the_reference_abi():
    names = declared_symbols()
    # crates/core/src/gpu.rs:10-15 binds exactly these three.
    for n in ("knn_gpu_create", "knn_gpu_search", "knn_gpu_free"):
        assert n in names
    assert len(names) >= 25


def test_library_exports_every_declared_symbol(px):
    lib = px._lib.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    # And the Python binding types every one of them.
    assert set(declared_symbols()) <= set(px._lib.SIGNATURES)


def test_exports_are_c_symbols():
    so = os.path.join(ROOT, "proxima_b200", "libproxima_b200.so")
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for n in declared_symbols():
        assert n in exported, n  # unmangled, default visibility


def test_build_targets_sm100a_only():
    from proxima_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_no_gpu_errors_are_reported(px):
    lib = px._lib.load()
    if lib.px_device_count() > 0:
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = lib.px_flat_create(16, 0, None, 0, ctypes.byref(h))
    assert st == px._lib.PX_ECUDA
    assert "no CUDA device" in px._lib.last_error()
    assert lib.knn_gpu_create(None, 0, 4) is None
    with pytest.raises(px.PxError):
        px.FlatIndex(16)


def test_argument_validation_without_gpu(px):
    lib = px._lib.load()
    h = ctypes.c_void_p()
    assert lib.px_flat_create(0, 0, None, 0, ctypes.byref(h)) == px._lib.PX_EINVAL
    assert "dim must be > 0" in px._lib.last_error()
    assert lib.px_flat_create(4, 7, None, 0, ctypes.byref(h)) == px._lib.PX_EINVAL
    assert lib.px_pq_create(10, 3, 8, 0, None, None, 0, ctypes.byref(h)) == px._lib.PX_EINVAL
    assert "divisible by m" in px._lib.last_error()
    assert lib.px_pq_create(8, 2, 9, 0, None, None, 0, ctypes.byref(h)) == px._lib.PX_EINVAL
    assert "nbits" in px._lib.last_error()
    # knn_gpu_search rejects k < 1 before touching the index (knn.cu:145).
    assert lib.knn_gpu_search(None, None, 1, 0, 0, None, None) == -1
    assert lib.knn_gpu_search(None, None, 1, px.PX_MAX_K + 1, 0, None, None) == -1
    # Null handles are tolerated by destroy/free.
    assert lib.px_flat_destroy(None) == 0
    lib.knn_gpu_free(None)


def test_python_mirror_validation_without_gpu(px):
    # Checks that run before any device call, as in the PyO3 layer.
    with pytest.raises(ValueError, match="dim must be > 0"):
        px.FlatIndex(0)
    with pytest.raises(OverflowError):
        px.FlatIndex(-1)
    with pytest.raises(ValueError):
        px.PqIndex(dim=10, m=3)
    with pytest.raises(ValueError):
        px.PqIndex(dim=8, m=0)
    with pytest.raises(ValueError):
        px.PqIndex(dim=8, m=2, nbits=9)
    pq = px.PqIndex(dim=64, metric=px.Metric.L2, m=8)
    assert not pq.is_trained and pq.size == 0 and pq.memory_bytes == 0
    with pytest.raises(ValueError, match="not trained"):
        pq.add(np.zeros((4, 64), np.float32))
    with pytest.raises(ValueError, match="not trained"):
        pq.search(np.zeros(64, np.float32), k=5)
    with pytest.raises(ValueError, match="not trained"):
        pq.search_filtered(np.zeros(64, np.float32), np.zeros(0, bool), k=5)


def test_record_layout_and_new_entry_points_validate_without_gpu(px):
    """The shard-record size and the argument checks of the entry points this
    library adds beside the reference's (they fail before any device work)."""
    lib = px._lib.load()
    # ids (8 bytes) then keys (4 bytes) per entry, padded to 16 bytes.
    for nq, k in ((1, 1), (37, 10), (10000, 10), (3, 7), (0, 5)):
        rec = lib.px_shard_record_bytes(nq, k)
        assert rec % 16 == 0 and 12 * nq * k <= rec < 12 * nq * k + 16, (nq, k, rec)
    assert lib.px_shard_record_bytes(-1, 3) == 0
    vp = ctypes.c_void_p
    # Record merge: shard count, sizes and metric are checked first.
    assert lib.px_merge_shard_records_device(0, vp(16), 0, 1, 1, 0, 1, vp(16), vp(16), None) == px._lib.PX_EINVAL
    assert lib.px_merge_shard_records_device(0, vp(16), 9, 1, 1, 0, 1, vp(16), vp(16), None) == px._lib.PX_EINVAL
    assert lib.px_merge_shard_records_device(0, vp(16), 2, -1, 1, 0, 1, vp(16), vp(16), None) == px._lib.PX_EINVAL
    assert lib.px_merge_shard_records_device(0, vp(16), 2, 1, 1, 5, 1, vp(16), vp(16), None) == px._lib.PX_EINVAL
    assert lib.px_merge_shard_records_device(0, None, 2, 1, 1, 0, 1, vp(16), vp(16), None) == px._lib.PX_EINVAL
    assert lib.px_merge_shard_records_device(0, vp(8), 2, 1, 1, 0, 1, vp(16), vp(16), None) == px._lib.PX_EINVAL
    assert "16-byte aligned" in px._lib.last_error()
    # Nothing to merge is a no-op.
    assert lib.px_merge_shard_records_device(0, None, 2, 0, 1, 0, 1, None, None, None) == 0
    # Null handles.
    cands, kind = ctypes.c_int32(0), ctypes.c_int32(0)
    assert lib.px_flat_debug_candidates(None, None, 1, 10, 64, None, None, ctypes.byref(cands),
                                        ctypes.byref(kind)) == px._lib.PX_EINVAL
    assert lib.px_pq_search_device(None, None, 1, 10, 0, None, None, None) == px._lib.PX_EINVAL
    assert lib.px_flat_set_sample_pass(None, 0) == px._lib.PX_EINVAL
    totals = px._lib.ProfileTotals()
    assert lib.px_flat_profile_totals(None, 0, ctypes.byref(totals)) == px._lib.PX_EINVAL
    assert ctypes.sizeof(px._lib.ProfileTotals) == 40  # double + 4 x int64, as in px.h


def test_non_finite_inputs_are_rejected_without_gpu(px):
    """The host finiteness check (vectorized, and split over threads for long
    inputs) on every length class and position: px_pq_train runs it before it
    needs a device, so a rejected input reports EINVAL and an accepted one
    gets as far as the missing device."""
    lib = px._lib.load()
    if lib.px_device_count() > 0:
        pytest.skip("a GPU is present (the accepted case would train)")
    books = np.zeros(2 * 2 * 2, dtype=np.float32)  # m=2 subspaces x 2 centroids x dsub 2
    bad_bits = [0x7fc00000, 0xffc00000, 0x7f800000, 0xff800000, 0x7f800001]
    for count in (8, 12, 36, 4000, 2_400_000):
        base = np.full(count, 1.5, dtype=np.float32)
        base[count // 3] = np.float32(3.4028235e38)  # FLT_MAX is finite
        for pos in sorted({0, 1, 7, count // 2, count - 1}):
            for bits in bad_bits:
                x = base.copy()
                x.view(np.uint32)[pos] = bits
                st = lib.px_pq_train(x.ctypes.data_as(px._lib._f32p), count // 4, 4, 2, 1, 1, 0, 1, 0,
                                     books.ctypes.data_as(px._lib._f32p))
                assert st == px._lib.PX_EINVAL and "NaN or infinite" in px._lib.last_error(), (count, pos, hex(bits))
        st = lib.px_pq_train(base.ctypes.data_as(px._lib._f32p), count // 4, 4, 2, 1, 1, 0, 1, 0,
                             books.ctypes.data_as(px._lib._f32p))
        assert st != px._lib.PX_EINVAL, (count, px._lib.last_error())
