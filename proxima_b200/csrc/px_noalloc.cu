// px_flat_search_noalloc: exact kNN over a base the caller already holds in
// device memory, without allocating anything.
//
// Who needs it: callers that run inside a host program which owns all GPU
// memory and hands out fixed buffers -- a database or serving plugin given an
// arena, a framework whose allocator must account for every byte -- and that
// therefore may not call cudaMalloc (or have this library call it) on the
// search path. They pass the base, the queries and the output buffers; the
// only other memory the search needs, its candidate lists, comes from the
// fixed array below, which the library image brings with it.
//
// The array: kScratchBytes (16 MiB) of file-scope device memory. Every GPU on
// which the library is loaded holds it until the process exits. Host code may
// not use `g_noalloc_scratch` as a device address (on the host the name is a
// stand-in); the first call on each device resolves the real address with
// cudaGetSymbolAddress while that device is current, checks the result and
// caches it, so the first call on a device should be made before any stream
// capture begins. Every call shares the array and it keeps the previous
// call's contents: the call clears the part that must start at zero (its id
// segment table), and the scan overwrites the rest. Two calls whose work
// overlaps on the GPU (concurrent streams, or threads on the same device)
// race on the array; callers must order them.
//
// Limits: nq * (ncta + 1) * k * 8 bytes of candidate lists must fit in the
// array (the number of row splits ncta shrinks to make it fit; a request that
// does not fit even with one split is rejected), dim must be a multiple of 4
// and the base 16-byte aligned (the scan reads rows with 128-bit loads), and
// n < 2^32.
#include <algorithm>
#include <mutex>
#include <string>

#include "../../include/px.h"
#include "px_common.cuh"
#include "px_kernels.h"
#include "px_runtime.h"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr size_t kSegBytes = 256;  // zeroed (local_begin, global_begin) table

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

px_status scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return px::cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return px::set_error(PX_EUNSUPPORTED, "device ordinal too large");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return px::cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                             "cudaGetSymbolAddress(no-allocation scratch)");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return PX_OK;
}

}  // namespace

extern "C" PX_API px_status px_flat_search_noalloc(const float* d_base, int64_t n, int32_t dim,
                                                   int32_t metric, const float* d_queries, int64_t nq,
                                                   int32_t k, int64_t* d_out_ids, float* d_out_dists,
                                                   void* stream) {
  using px::set_error;
  if (dim <= 0) return set_error(PX_EINVAL, "dim must be > 0");
  if (metric != PX_METRIC_L2 && metric != PX_METRIC_IP)
    return set_error(PX_EINVAL, "metric must be 0 (L2) or 1 (inner product)");
  if (n < 0 || nq < 0 || k < 0) return set_error(PX_EINVAL, "n, nq and k must be >= 0");
  if (k > PX_MAX_K)
    return set_error(PX_EUNSUPPORTED, "k=" + std::to_string(k) + " exceeds PX_MAX_K=" + std::to_string(PX_MAX_K));
  if (n > 0xFFFFFFFFll) return set_error(PX_EUNSUPPORTED, "n must be < 2^32");
  if (dim % 4 != 0)
    return set_error(PX_EUNSUPPORTED, "the no-allocation search needs dim to be a multiple of 4");
  if (k == 0 || nq == 0) return PX_OK;
  if (d_queries == nullptr || d_out_ids == nullptr || d_out_dists == nullptr || (n > 0 && d_base == nullptr))
    return set_error(PX_EINVAL, "null buffer");
  if (reinterpret_cast<uintptr_t>(d_base) % 16 != 0)
    return set_error(PX_EINVAL, "the base must be 16-byte aligned");

  // Row splits: as many as fill the GPU, fewer if the lists would not fit.
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) sms = px::device_sm_count(dev);
  const int group = px::exact_group_for(nq);
  const int64_t groups = (nq + group - 1) / group;
  if (groups > 65535) return set_error(PX_EUNSUPPORTED, "too many queries in one call");
  const int64_t rows_total = n > 0 ? n : 1;
  int64_t ncta = (static_cast<int64_t>(sms) * 4 + groups - 1) / groups;
  ncta = std::min<int64_t>(std::min<int64_t>(std::max<int64_t>(ncta, 1), (rows_total + 127) / 128), 1024);
  const int64_t per_list = nq * static_cast<int64_t>(k) * 8;
  const int64_t budget = static_cast<int64_t>(kScratchBytes - kSegBytes) - 256;
  if (per_list * 2 > budget)
    return set_error(PX_EUNSUPPORTED, "nq * k = " + std::to_string(nq * k) + " exceeds the no-allocation "
                                      "scratch (at most " + std::to_string(budget / 16) + ")");
  while (ncta > 1 && per_list * (ncta + 1) > budget) --ncta;
  int64_t rows = ((rows_total + ncta - 1) / ncta + 127) / 128 * 128;
  ncta = (rows_total + rows - 1) / rows;

  void* base = nullptr;
  px_status s = scratch_for_current_device(&base);
  if (s != PX_OK) return s;
  unsigned char* scratch = static_cast<unsigned char*>(base);
  int64_t* seg = reinterpret_cast<int64_t*>(scratch);
  uint64_t* partial = reinterpret_cast<uint64_t*>(scratch + kSegBytes);
  uint64_t* final_c = partial + nq * ncta * k;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  cudaError_t e = cudaMemsetAsync(seg, 0, kSegBytes, st);
  if (e != cudaSuccess) return px::cuda_status(e, "scratch clear");
  px::ExactScanArgs a;
  a.base = d_base;
  a.n = n;
  a.ld = dim;
  a.d = dim;
  a.queries = d_queries;
  a.nq = static_cast<int>(nq);
  a.k = k;
  a.group = group;
  a.ncta = static_cast<int>(ncta);
  a.rows_per_cta = rows;
  a.mask = nullptr;
  a.l2 = metric == PX_METRIC_L2;
  a.partial = partial;
  e = px::launch_exact_scan(a, st);
  if (e != cudaSuccess) return px::cuda_status(e, "exact scan launch");
  e = px::launch_merge_lists(partial, nq, static_cast<int>(ncta), k, k, final_c, st);
  if (e != cudaSuccess) return px::cuda_status(e, "merge launch");
  px::IdSegments segs;
  segs.local_begin = seg;
  segs.global_begin = seg + 1;
  segs.nseg = 1;
  segs.id_offset = 0;
  e = px::launch_emit(final_c, nq, k, metric == PX_METRIC_L2, true, segs, d_out_ids, d_out_dists, st);
  if (e != cudaSuccess) return px::cuda_status(e, "emit launch");
  px::g_launches += 3;
  return PX_OK;
}
