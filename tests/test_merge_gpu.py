"""The cross-shard merge kernel (K6) on one GPU.

Every multi-GPU search ends in this merge: each rank's sorted key-space top-k
(global ids, ties by smaller id) is gathered and the G lists per query are
merged on the device. Here the per-shard lists are built by the CPU oracle
(FlatIndex::search_batch, crates/core/src/flat.rs:150-191) on contiguous row
ranges of one base, laid out both as [G][nq][k] arrays
(px_merge_shards_device) and as the records one all-gather moves
(px_merge_shard_records_device), and the merged result must equal the
oracle's search of the whole base under the tie-aware, bit-exact rule, and
the (key, id) order exactly. Duplicated rows in different shards force ties
across shards; shards shorter than k force padding.
"""

import ctypes

import numpy as np
import pytest

import oracle as O
from proxima_b200.distributed import shard_range
from tests import _parity

pytestmark = pytest.mark.gpu


def _ord(keys):
    b = np.asarray(keys, np.float32).view(np.uint32).astype(np.uint64)
    return np.where(b & 0x80000000, ~b & 0xFFFFFFFF, b | 0x80000000)


def _shard_lists(data, metric, queries, k, G):
    nq = queries.shape[0]
    ids = np.full((G, nq, k), -1, np.int64)
    keys = np.full((G, nq, k), np.float32(3.4028235e38), np.float32)
    for g in range(G):
        lo, hi = shard_range(data.shape[0], G, g)
        if hi == lo:
            continue
        li, _ = O.flat_search_batch(data[lo:hi], metric, queries, k)
        gi = np.where(li >= 0, li + lo, -1)
        for q in range(nq):
            ok = gi[q] >= 0
            kk = O.flat_keys(data, metric, queries[q], gi[q][ok])
            # a rank's list is sorted by (key, global id)
            order = np.lexsort((gi[q][ok], _ord(kk)))
            ids[g, q, : ok.sum()] = gi[q][ok][order]
            keys[g, q, : ok.sum()] = kk[order]
    return ids, keys


@pytest.mark.parametrize("G", [2, 3, 5, 8])
@pytest.mark.parametrize("metric", [O.L2, O.IP])
@pytest.mark.parametrize("n,k", [(3001, 10), (40, 10), (2000, 100)])
def test_merge_shards_matches_single_index(px, oracle_lib, G, metric, n, k):
    import torch

    assert px.device_count() > 0, "GPU tests need a CUDA device"
    lib = px._lib.load()
    dim, nq = 16, 23
    data = O.gen_uniform(n, dim, 31 + n)
    data = np.rint(data * 4).astype(np.float32)  # small integers: many exact ties
    data[n // 2: n // 2 + min(50, n // 4)] = data[: min(50, n // 4)]  # duplicates across shards
    queries = np.rint(O.gen_uniform(nq, dim, 77) * 4).astype(np.float32)
    ids, keys = _shard_lists(data, metric, queries, k, G)

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    out_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
    out_i = torch.empty((nq, k), dtype=torch.int64, device=dev)
    ref_ids, ref_d = O.flat_search_batch(data, metric, queries, k)
    nat = _parity.flat_natural(data, metric, queries)

    # (1) [G][nq][k] arrays
    d_keys = torch.from_numpy(keys).to(dev)
    d_ids = torch.from_numpy(ids).to(dev)
    st = lib.px_merge_shards_device(0, ctypes.c_void_p(d_keys.data_ptr()), ctypes.c_void_p(d_ids.data_ptr()),
                                    G, nq, k, metric, 1, ctypes.c_void_p(out_d.data_ptr()),
                                    ctypes.c_void_p(out_i.data_ptr()), sp)
    assert st == 0, px._lib.last_error()
    torch.cuda.synchronize()
    got_i, got_d = out_i.cpu().numpy(), out_d.cpu().numpy()
    _parity.check(got_i, got_d, ref_ids, ref_d, nat)

    # The exact (key, smaller id) order of the union of the lists.
    for q in range(nq):
        flat_ids = ids[:, q, :].reshape(-1)
        flat_keys = keys[:, q, :].reshape(-1)
        ok = flat_ids >= 0
        order = np.lexsort((flat_ids[ok], _ord(flat_keys[ok])))[:k]
        want = flat_ids[ok][order]
        assert np.array_equal(got_i[q, : len(want)], want), (q, got_i[q], want)
        assert np.all(got_i[q, len(want):] == -1)

    # (2) the records one all-gather moves: ids then keys, record after record
    rec = int(lib.px_shard_record_bytes(nq, k))
    assert rec % 16 == 0 and rec >= 12 * nq * k
    records = np.zeros((G, rec), np.uint8)
    for g in range(G):
        records[g, : 8 * nq * k] = ids[g].reshape(-1).view(np.uint8)
        records[g, 8 * nq * k: 12 * nq * k] = keys[g].reshape(-1).view(np.uint8)
    d_rec = torch.from_numpy(records.reshape(-1)).to(dev)
    out_d.fill_(0)
    out_i.fill_(0)
    st = lib.px_merge_shard_records_device(0, ctypes.c_void_p(d_rec.data_ptr()), G, nq, k, metric, 1,
                                           ctypes.c_void_p(out_d.data_ptr()), ctypes.c_void_p(out_i.data_ptr()),
                                           sp)
    assert st == 0, px._lib.last_error()
    torch.cuda.synchronize()
    assert np.array_equal(out_i.cpu().numpy(), got_i)
    assert np.array_equal(out_d.cpu().numpy().view(np.uint32), got_d.view(np.uint32))


@pytest.mark.parametrize("metric", [O.L2, O.IP])
def test_sharded_index_record_path_on_one_gpu(px, oracle_lib, monkeypatch, metric):
    """ShardedFlatIndex.search_device for two ranks, both on one GPU, with the
    all-gather replaced by a local copy of the two ranks' records (NCCL needs
    one GPU per rank). Exercises what every rank does around the collective:
    the key-space search written into its record, the record layout, and the
    record merge; the answer must equal the oracle's on the whole base."""
    import torch

    import proxima_b200.distributed as D
    from proxima_b200.distributed import ShardedFlatIndex

    assert px.device_count() > 0, "GPU tests need a CUDA device"
    rng = np.random.default_rng(4)
    n, dim, nq, k = 9001, 64, 37, 10
    data = np.rint(rng.standard_normal((n, dim)).astype(np.float32) * 3)
    data[4600:4700] = data[:100]  # exact ties across the two shards
    queries = np.rint(rng.standard_normal((nq, dim)).astype(np.float32) * 3)
    ranks = []
    for r in range(2):
        idx = ShardedFlatIndex(dim, px.Metric.L2 if metric == O.L2 else px.Metric.InnerProduct, device=0)
        idx.world, idx.rank, idx._bufs = 2, r, {}
        lo, hi = shard_range(n, 2, r)
        idx.set_offset(lo)
        idx.add_local(data[lo:hi])
        ranks.append(idx)
    dq = torch.from_numpy(queries).cuda()
    records = {}

    def fake_all_gather(out, inp, group=None):
        records[len(records)] = inp.clone()
        if len(records) == 2:
            out.copy_(torch.cat([records[0], records[1]]))
        else:
            out.fill_(255)  # rank 0 merges before rank 1 has searched: all ids -1, i.e. padding

    monkeypatch.setattr(D.dist, "all_gather_into_tensor", fake_all_gather)
    for path in ("tensor", "exact"):
        records.clear()
        for idx in ranks:
            idx.local.set_search_path(path)
        ranks[0].search_device(dq, k)  # rank 0's record; its merge waits for rank 1's
        ids, d = ranks[1].search_device(dq, k)
        torch.cuda.synchronize()
        _parity.check_flat(data, metric, queries, ids.cpu().numpy(), d.cpu().numpy(), k)
