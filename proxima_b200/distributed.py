"""Row-sharded exact kNN across processes (one process per GPU).

Each rank holds a contiguous run of base rows [offset, offset + n_local) in a
single-device ``px_flat`` handle. A search runs every rank's local top-k on
its GPU (key space: squared L2 or negated inner product, sorted, ties by
global id) straight into one record buffer (ids, then keys), gathers the
records with a single NCCL all-gather over NVLink, and merges them on the
device (``px_merge_shard_records_device``). Every rank ends up with the same
final top-k, identical to a single index holding all rows.

torch.distributed provides the process group and NCCL; torch tensors hold
the device buffers. The search itself is libproxima_b200's kernels.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from ._core import FlatIndex, Metric, _check_finite, _check_k


def shard_range(n: int, world: int, rank: int):
    """Contiguous split of n rows over `world` ranks (remainder to the first)."""
    base, rem = divmod(n, world)
    begin = rank * base + min(rank, rem)
    return begin, begin + base + (1 if rank < rem else 0)


class ShardedFlatIndex:
    """A FlatIndex whose rows are spread over the ranks of a process group."""

    def __init__(self, dim: int, metric=Metric.InnerProduct, *, group=None, device=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self.metric = metric
        self.dim = dim
        self.local = FlatIndex(dim, metric, devices=[self.device.index])
        self._lib = _lib.load()
        self._bufs = {}

    # -- building ----------------------------------------------------------
    def set_offset(self, offset: int) -> None:
        """Global id of this rank's first row."""
        _lib.check(self._lib.px_flat_set_id_offset(self.local.handle, int(offset)))

    def reserve_local(self, n_local: int) -> None:
        self.local.reserve(n_local)

    def add_local_device(self, rows: torch.Tensor) -> None:
        """Appends rows (a contiguous float32 CUDA tensor on this rank's GPU)."""
        assert rows.is_cuda and rows.dtype == torch.float32 and rows.is_contiguous()
        assert rows.shape[1] == self.dim
        torch.cuda.current_stream(self.device).synchronize()
        _lib.check(self._lib.px_flat_add_device(self.local.handle, ctypes.c_void_p(rows.data_ptr()),
                                                rows.shape[0]))

    def add_local(self, rows: np.ndarray) -> None:
        self.local.add(rows)

    @property
    def local_size(self) -> int:
        return self.local.size

    # -- searching ---------------------------------------------------------
    def _buffers(self, nq: int, k: int):
        key = (nq, k)
        if key not in self._bufs:
            dev = self.device
            rec = int(self._lib.px_shard_record_bytes(nq, k))
            self._bufs = {key: dict(
                rec=rec,
                # this rank's record: ids [nq][k] int64, then keys [nq][k] float32
                record=torch.empty(rec, dtype=torch.uint8, device=dev),
                # every rank's record, back to back (rank order)
                records=torch.empty(self.world * rec, dtype=torch.uint8, device=dev),
                out_ids=torch.empty((nq, k), dtype=torch.int64, device=dev),
                out_d=torch.empty((nq, k), dtype=torch.float32, device=dev),
            )}
        return self._bufs[key]

    def search_device(self, queries: torch.Tensor, k: int):
        """queries: (nq, dim) float32 CUDA tensor, identical on every rank.
        Returns (ids int64, natural distances float32) CUDA tensors (nq, k)."""
        nq = queries.shape[0]
        _check_k(k)
        b = self._buffers(nq, k)
        stream = torch.cuda.current_stream(self.device)
        sp = ctypes.c_void_p(stream.cuda_stream)
        if self.world == 1:
            _lib.check(self._lib.px_flat_search_device(
                self.local.handle, ctypes.c_void_p(queries.data_ptr()), nq, k, 0,
                ctypes.c_void_p(b["out_ids"].data_ptr()), ctypes.c_void_p(b["out_d"].data_ptr()), sp))
            return b["out_ids"], b["out_d"]
        rec = b["record"].data_ptr()
        _lib.check(self._lib.px_flat_search_device(
            self.local.handle, ctypes.c_void_p(queries.data_ptr()), nq, k, 1,
            ctypes.c_void_p(rec), ctypes.c_void_p(rec + 8 * nq * k), sp))
        dist.all_gather_into_tensor(b["records"], b["record"], group=self.group)
        _lib.check(self._lib.px_merge_shard_records_device(
            self.device.index, ctypes.c_void_p(b["records"].data_ptr()), self.world, nq, k,
            int(self.metric), 1, ctypes.c_void_p(b["out_d"].data_ptr()),
            ctypes.c_void_p(b["out_ids"].data_ptr()), sp))
        return b["out_ids"], b["out_d"]

    def search_batch(self, queries: np.ndarray, k: int = 10):
        """Host-to-host search: numpy queries in, numpy (ids, dists) out."""
        q = np.ascontiguousarray(queries, dtype=np.float32)
        _check_finite(q)
        dq = torch.from_numpy(q).to(self.device, non_blocking=False)
        ids, d = self.search_device(dq, k)
        return ids.cpu().numpy(), d.cpu().numpy()
