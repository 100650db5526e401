"""px_flat_search_noalloc: the search entry point that allocates nothing.

It exists for callers that may not allocate GPU memory themselves (a plugin
working inside a fixed arena its host program hands it, a service whose
allocator must own every byte): they pass the base, queries and outputs in
device memory, and the library uses only a fixed device array it carries.
This test calls it through the C ABI twice in a row and checks each result
against px_flat_search on the same data -- bit for bit, the tolerance of
every other parity test here -- and that the calls leave the device's free
memory unchanged (from the second call on: the very first call on a device
may load the library's device image, which brings the fixed array with it).
The file name makes pytest collect it last.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_matches_flat_search_twice(px):
    import torch

    assert px.device_count() > 0, "GPU tests need a CUDA device"
    lib = px._lib.load()
    rng = np.random.default_rng(12)
    n, dim, k = 50000, 96, 10
    base = rng.standard_normal((n, dim)).astype(np.float32)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    d_base = torch.from_numpy(base).to(dev)
    first = True
    for metric in (px.Metric.L2, px.Metric.InnerProduct):
        ref = px.FlatIndex(dim, metric)
        ref.add(base)
        ref.set_search_path("exact")
        for call, nq in enumerate((37, 5)):
            q = rng.standard_normal((nq, dim)).astype(np.float32)
            want_ids, want_d = ref.search_batch(q, k=k)
            d_q = torch.from_numpy(q).to(dev)
            out_ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
            out_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
            stream = torch.cuda.current_stream(dev)
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info(dev)[0]
            st = lib.px_flat_search_noalloc(
                ctypes.c_void_p(d_base.data_ptr()), n, dim, int(metric),
                ctypes.c_void_p(d_q.data_ptr()), nq, k, ctypes.c_void_p(out_ids.data_ptr()),
                ctypes.c_void_p(out_d.data_ptr()), ctypes.c_void_p(stream.cuda_stream))
            assert st == 0, px._lib.last_error()
            torch.cuda.synchronize()
            if not first:
                assert torch.cuda.mem_get_info(dev)[0] == free_before, f"call {call} allocated memory"
            first = False
            got_ids, got_d = out_ids.cpu().numpy(), out_d.cpu().numpy()
            assert np.array_equal(got_d.view(np.uint32), want_d.view(np.uint32)), f"call {call}"
            assert np.array_equal(got_ids, want_ids), f"call {call}"


def test_noalloc_rejects_what_does_not_fit(px):
    lib = px._lib.load()
    vp = ctypes.c_void_p
    # dim must be a multiple of 4; nq * k beyond the fixed scratch is refused.
    assert lib.px_flat_search_noalloc(vp(16), 10, 6, 0, vp(16), 1, 1, vp(16), vp(16), None) == px._lib.PX_EUNSUPPORTED
    assert "multiple of 4" in px._lib.last_error()
    assert lib.px_flat_search_noalloc(vp(16), 10, 8, 0, vp(16), 200000, 700, vp(16), vp(16), None) == px._lib.PX_EUNSUPPORTED
    assert "scratch" in px._lib.last_error()


def _noalloc(px, d_base, n, dim, metric, q, k):
    import torch

    lib = px._lib.load()
    dev = d_base.device
    nq = q.shape[0]
    d_q = torch.from_numpy(q).to(dev)
    out_ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
    out_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
    st = lib.px_flat_search_noalloc(
        ctypes.c_void_p(d_base.data_ptr()), n, dim, int(metric), ctypes.c_void_p(d_q.data_ptr()), nq, k,
        ctypes.c_void_p(out_ids.data_ptr()), ctypes.c_void_p(out_d.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert st == 0, px._lib.last_error()
    torch.cuda.synchronize()
    return out_ids.cpu().numpy(), out_d.cpu().numpy()


@pytest.mark.parametrize("n,dim,nq,k", [
    (50000, 96, 4096, 200),   # nq * k near the scratch budget: the row splits shrink to one
    (50000, 96, 5, 700),      # the largest candidate buffer
    (1000003, 16, 64, 10),    # n not a multiple of the 128-row split granule
    (0, 32, 3, 10),           # empty base: every slot is padding
])
def test_noalloc_edges_match_flat_search(px, n, dim, nq, k):
    import torch

    rng = np.random.default_rng(n + k)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    base = rng.standard_normal((max(n, 1), dim)).astype(np.float32)[:n]
    d_base = torch.from_numpy(np.ascontiguousarray(base) if n else np.zeros((1, dim), np.float32)).to(dev)
    q = rng.standard_normal((nq, dim)).astype(np.float32)
    for metric in (px.Metric.L2, px.Metric.InnerProduct):
        got_ids, got_d = _noalloc(px, d_base, n, dim, metric, q, k)
        if n == 0:
            assert np.all(got_ids == -1)
            pad = np.float32(3.4028235e38) * (1 if metric == px.Metric.L2 else -1)
            assert np.all(got_d == pad)
            continue
        ref = px.FlatIndex(dim, metric)
        ref.add(base)
        ref.set_search_path("exact")
        want_ids, want_d = ref.search_batch(q, k=k)
        assert np.array_equal(got_d.view(np.uint32), want_d.view(np.uint32))
        assert np.array_equal(got_ids, want_ids)


def test_noalloc_matches_the_oracle(px, oracle_lib):
    import torch

    import oracle as O
    from tests import _parity

    rng = np.random.default_rng(44)
    n, dim, nq, k = 20000, 64, 24, 10
    base = rng.standard_normal((n, dim)).astype(np.float32)
    q = rng.standard_normal((nq, dim)).astype(np.float32)
    dev = torch.device("cuda", 0)
    d_base = torch.from_numpy(base).to(dev)
    for metric, om in ((px.Metric.L2, O.L2), (px.Metric.InnerProduct, O.IP)):
        ids, d = _noalloc(px, d_base, n, dim, metric, q, k)
        _parity.check_flat(base, om, q, ids, d, k)
