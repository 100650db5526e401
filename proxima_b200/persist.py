"""Index files in the reference's format (`.sfidx`).

The reference serialises whole index structs with bincode 1
(crates/core/src/lib.rs:19-30: `bincode::serialize_into`, whose legacy
configuration is little-endian with fixed-width integers): `usize` as u64,
a unit enum variant as its u32 index, a `Vec<T>` as a u64 length followed by
the elements, struct fields in declaration order. The layouts written and
read here are therefore

  FlatIndex (flat.rs:35-40):
      dim u64 | metric u32 | n u64 | data: len u64, f32 x len
  PqIndex (pq.rs:218-223) with ProductQuantizer (pq.rs:40-46):
      metric u32 | dim u64 | m u64 | dsub u64 | k u64 |
      codebooks: len u64, f32 x len | codes: len u64, u8 x len | n u64

so files move both ways between this package and the reference. Rows and
codes stream between the GPU and the file in chunks, so saving or loading
never holds a second full copy of a large index in host memory.
"""

from __future__ import annotations

import struct

import numpy as np

CHUNK_ROWS = 1 << 20


def _read_exact(f, n: int) -> bytes:
    b = f.read(n)
    if len(b) != n:
        raise OSError("unexpected end of file (truncated or not an index file)")
    return b


def _u64(f) -> int:
    return struct.unpack("<Q", _read_exact(f, 8))[0]


def _u32(f) -> int:
    return struct.unpack("<I", _read_exact(f, 4))[0]


def _metric(f):
    from ._core import Metric
    v = _u32(f)
    if v > 1:
        raise OSError(f"invalid value: integer `{v}`, expected variant index 0 <= i < 2")
    return Metric(v)


def save_flat(index, path) -> None:
    n, dim = index.size, index.dim
    with open(path, "wb") as f:
        f.write(struct.pack("<QIQ", dim, int(index.metric), n))
        f.write(struct.pack("<Q", n * dim))
        for start in range(0, n, CHUNK_ROWS):
            rows = index.read_rows(start, min(CHUNK_ROWS, n - start))
            f.write(rows.astype("<f4", copy=False).tobytes())


def load_flat(cls, path, **kwargs):
    with open(path, "rb") as f:
        dim = _u64(f)
        metric = _metric(f)
        n = _u64(f)
        length = _u64(f)
        if dim == 0 or length != n * dim:
            raise OSError(f"inconsistent FlatIndex file: dim {dim}, n {n}, data length {length}")
        index = cls(dim, metric, **kwargs)
        if n:
            index.reserve(n)
        left = n
        while left:
            rows = min(CHUNK_ROWS, left)
            data = np.frombuffer(_read_exact(f, rows * dim * 4), dtype="<f4").astype(np.float32)
            index.add(data.reshape(rows, dim))
            left -= rows
    return index


def save_pq(index, path) -> None:
    books = index.codebooks
    m, k, dsub = books.shape
    n = index.size
    with open(path, "wb") as f:
        f.write(struct.pack("<I", int(index.metric)))
        f.write(struct.pack("<QQQQ", index.dim, m, dsub, k))
        f.write(struct.pack("<Q", books.size))
        f.write(books.astype("<f4", copy=False).tobytes())
        f.write(struct.pack("<Q", n * m))
        for start in range(0, n, CHUNK_ROWS):
            f.write(index.read_codes(start, min(CHUNK_ROWS, n - start)).tobytes())
        f.write(struct.pack("<Q", n))


def load_pq(cls, path, **kwargs):
    with open(path, "rb") as f:
        metric = _metric(f)
        dim, m, dsub, k = (_u64(f) for _ in range(4))
        if m == 0 or dim != m * dsub or k < 2 or k & (k - 1) or k > 256:
            raise OSError(f"inconsistent PqIndex file: dim {dim}, m {m}, dsub {dsub}, k {k}")
        nb = _u64(f)
        if nb != m * k * dsub:
            raise OSError("inconsistent PqIndex file: codebook length")
        books = np.frombuffer(_read_exact(f, nb * 4), dtype="<f4").astype(np.float32).reshape(m, k, dsub)
        ncodes = _u64(f)
        if ncodes % m:
            raise OSError("inconsistent PqIndex file: code length")
        n = ncodes // m
        # lib.rs:672-678: a loaded index gets the default training parameters.
        index = cls(dim, metric, m=m, nbits=k.bit_length() - 1, **kwargs)
        index._set_codebooks(books)
        left = n
        while left:
            rows = min(CHUNK_ROWS, left)
            codes = np.frombuffer(_read_exact(f, rows * m), dtype=np.uint8).reshape(rows, m)
            index.add_codes(np.ascontiguousarray(codes))
            left -= rows
        if _u64(f) != n:
            raise OSError("inconsistent PqIndex file: row count")
    return index
