"""Row-sharded search across processes.

CPU (gloo, world size 2): the sharding scheme of proxima_b200.distributed --
contiguous shard ranges, global ids by offset, each rank's key-space top-k
packed into one record (ids then keys, px_shard_record_bytes long), one
all-gather of the records, merge by (key, global id) -- reproduces a single
index's top-k (tie-aware rule). Each rank's local lists come from the CPU
oracle here, since the CPU box has no GPU; the record layout, the collective
and its dtype are the ones ShardedFlatIndex uses. (The merge kernel itself
is tested on one GPU in tests/test_merge_gpu.py.)

GPU (NCCL, 2 GPUs, skipped with fewer): ShardedFlatIndex end to end against
the oracle on the full base.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from proxima_b200 import _lib
from proxima_b200.distributed import shard_range

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_shard_range_partitions_rows():
    for n in (0, 1, 7, 100, 10_000_001):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def _key_space(data, metric, queries, ids):
    """Exact reference keys of the returned ids (what a rank sends)."""
    keys = np.full(ids.shape, np.float32(3.4028235e38), np.float32)
    for q in range(ids.shape[0]):
        ok = ids[q] >= 0
        keys[q, ok] = O.flat_keys(data, metric, queries[q], ids[q][ok])
    return keys


def _merge(all_keys, all_ids, k):
    """(key total order, global id) merge of per-rank sorted lists."""
    nq = all_keys.shape[1]
    out_ids = np.full((nq, k), -1, np.int64)
    out_keys = np.zeros((nq, k), np.float32)
    for q in range(nq):
        cand = [(all_keys[r, q, j], all_ids[r, q, j]) for r in range(all_keys.shape[0])
                for j in range(k) if all_ids[r, q, j] >= 0]
        cand.sort(key=lambda t: (np.float32(t[0]).view(np.int32) ^ ((np.float32(t[0]).view(np.int32) >> 31) & 0x7FFFFFFF), t[1]))
        for j, (key, i) in enumerate(cand[:k]):
            out_ids[q, j], out_keys[q, j] = i, key
    return out_ids, out_keys


def _gloo_worker(rank, world, port, metric, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        n, dim, nq, k = 3001, 24, 17, 10
        data = O.gen_uniform(n, dim, 5)
        # integer-valued copies force exact ties across shard boundaries
        data[1500:1600] = data[:100]
        queries = O.gen_uniform(nq, dim, 6)
        lo, hi = shard_range(n, world, rank)
        ids, d = O.flat_search_batch(data[lo:hi], metric, queries, k)
        ids = np.where(ids >= 0, ids + lo, -1)
        keys = _key_space(data, metric, queries, ids)
        # Same layout as ShardedFlatIndex: one record per rank, ids then keys.
        rec = int(_lib.load().px_shard_record_bytes(nq, k))
        record = np.zeros(rec, np.uint8)
        record[: 8 * nq * k] = ids.astype(np.int64).reshape(-1).view(np.uint8)
        record[8 * nq * k: 12 * nq * k] = keys.astype(np.float32).reshape(-1).view(np.uint8)
        records = torch.empty(world * rec, dtype=torch.uint8)
        dist.all_gather_into_tensor(records, torch.from_numpy(record))
        if rank == 0:
            r = records.numpy().reshape(world, rec)
            all_ids = r[:, : 8 * nq * k].copy().view(np.int64).reshape(world, nq, k)
            all_keys = r[:, 8 * nq * k: 12 * nq * k].copy().view(np.float32).reshape(world, nq, k)
            mids, mkeys = _merge(all_keys, all_ids, k)
            nat = np.where(mids >= 0, np.sqrt(mkeys) if metric == O.L2 else -mkeys, 0).astype(np.float32)
            ref_ids, ref_d = O.flat_search_batch(data, metric, queries, k)
            from tests import _parity
            ties = _parity.check(mids, nat, ref_ids, ref_d, _parity.flat_natural(data, metric, queries))
            result_q.put(("ok", ties))
    except Exception as e:  # report to the parent instead of hanging it
        result_q.put(("error", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_gloo_two_ranks_shard_and_merge(oracle_lib, metric):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, metric, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    status, detail = q.get(timeout=5)
    assert status == "ok", detail


def _nccl_worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        import proxima_b200 as px
        from proxima_b200.distributed import ShardedFlatIndex
        from tests import _data, _parity
        n, dim, nq, k = 40000, 128, 200, 10
        data = _data.unit_gaussian(n, dim, 1)
        queries = _data.unit_gaussian(nq, dim, 2)
        idx = ShardedFlatIndex(dim, px.Metric.InnerProduct, device=rank)
        lo, hi = shard_range(n, world, rank)
        idx.set_offset(lo)
        idx.add_local(data[lo:hi])
        ids, d = idx.search_batch(queries, k=k)
        ids1, d1 = idx.search_batch(queries[:3], k=k)  # small batch: exact scan path
        if rank == 0:
            _parity.check_flat(data, O.IP, queries, ids, d, k)
            _parity.check_flat(data, O.IP, queries[:3], ids1, d1, k)
        result_q.put(("ok", rank))
    except Exception as e:
        result_q.put(("error", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_two_gpus_sharded_index(px, oracle_lib):
    if px.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [q.get(timeout=5) for _ in range(2)]
    assert all(s == "ok" for s, _ in res), res
