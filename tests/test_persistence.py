"""`.sfidx` files: the reference's bincode layouts (crates/core/src/lib.rs:19-30).

CPU: the byte layout written for a FlatIndex / PqIndex is checked field by
field against the bincode 1 encoding of the reference's structs
(flat.rs:35-40; pq.rs:40-46, 218-223), and a hand-built file in that layout
loads. GPU: the reference's tests/test_persistence.py round trips (Flat, PQ,
untrained PQ refused).
"""

import struct

import numpy as np
import pytest

from proxima_b200 import persist


class _FakeFlat:
    """Just what save_flat reads from a FlatIndex."""

    def __init__(self, data, metric):
        self.size, self.dim = data.shape
        self.metric = metric
        self._data = data

    def read_rows(self, start, count):
        return self._data[start:start + count]


def test_flat_layout_is_bincode_of_the_reference_struct(tmp_path, px):
    data = np.arange(12, dtype=np.float32).reshape(3, 4)
    path = tmp_path / "flat.sfidx"
    persist.save_flat(_FakeFlat(data, px.Metric.InnerProduct), str(path))
    raw = path.read_bytes()
    want = struct.pack("<QIQQ", 4, 1, 3, 12) + data.astype("<f4").tobytes()
    assert raw == want


class _FakePq:
    def __init__(self, books, codes, metric, dim):
        self.codebooks = books
        self._codes = codes
        self.size = codes.shape[0]
        self.metric = metric
        self.dim = dim

    def read_codes(self, start, count):
        return self._codes[start:start + count]


def test_pq_layout_is_bincode_of_the_reference_struct(tmp_path, px):
    books = np.arange(2 * 4 * 3, dtype=np.float32).reshape(2, 4, 3)  # m=2, k=4, dsub=3
    codes = np.array([[0, 1], [3, 2], [1, 1]], dtype=np.uint8)
    path = tmp_path / "pq.sfidx"
    persist.save_pq(_FakePq(books, codes, px.Metric.L2, 6), str(path))
    raw = path.read_bytes()
    want = (struct.pack("<I", 0) + struct.pack("<QQQQ", 6, 2, 3, 4) + struct.pack("<Q", 24) +
            books.astype("<f4").tobytes() + struct.pack("<Q", 6) + codes.tobytes() +
            struct.pack("<Q", 3))
    assert raw == want


def test_truncated_and_invalid_files_raise_oserror(tmp_path, px):
    p = tmp_path / "bad.sfidx"
    p.write_bytes(struct.pack("<QIQ", 4, 7, 0))
    with pytest.raises(OSError):
        px.FlatIndex.load(str(p))
    p.write_bytes(struct.pack("<QIQQ", 4, 0, 3, 11) + b"\0" * 44)  # length != n * dim
    with pytest.raises(OSError):
        px.FlatIndex.load(str(p))
    p.write_bytes(struct.pack("<QI", 4, 0))  # truncated header
    with pytest.raises(OSError):
        px.FlatIndex.load(str(p))


# ---- the reference's tests/test_persistence.py on the GPU ---------------

@pytest.fixture
def pdata():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3000, 64)).astype(np.float32)
    return x / np.linalg.norm(x, axis=1, keepdims=True)


@pytest.mark.gpu
def test_flat_roundtrip(tmp_path, pdata, px):
    idx = px.FlatIndex(dim=64, metric=px.Metric.L2)
    idx.add(pdata[:1000])
    idx.add(pdata[1000:])
    before, _ = idx.search(pdata[5].copy(), k=10)
    path = str(tmp_path / "flat.sfidx")
    idx.save(path)
    loaded = px.FlatIndex.load(path)
    after, _ = loaded.search(pdata[5].copy(), k=10)
    assert loaded.size == idx.size
    assert loaded.metric == px.Metric.L2
    assert before.tolist() == after.tolist()
    assert np.array_equal(loaded.read_rows(0, 3000), pdata)


@pytest.mark.gpu
def test_pq_roundtrip(tmp_path, pdata, px):
    idx = px.PqIndex(dim=64, metric=px.Metric.InnerProduct, m=4)
    idx.train(pdata)
    idx.add(pdata)
    before, _ = idx.search(pdata[5].copy(), k=10)
    path = str(tmp_path / "pq.sfidx")
    idx.save(path)
    loaded = px.PqIndex.load(path)
    after, _ = loaded.search(pdata[5].copy(), k=10)
    assert loaded.is_trained and loaded.size == idx.size and loaded.m == 4
    assert loaded.metric == px.Metric.InnerProduct
    assert before.tolist() == after.tolist()
    assert np.array_equal(loaded.codebooks, idx.codebooks)


@pytest.mark.gpu
def test_save_untrained_pq_raises(tmp_path, px):
    idx = px.PqIndex(dim=64, metric=px.Metric.L2, m=8)
    with pytest.raises(Exception):
        idx.save(str(tmp_path / "x.sfidx"))
