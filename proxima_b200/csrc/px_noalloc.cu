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
// stand-in). Its device address belongs to one CUDA context: a host program
// may bind its own driver-API contexts, hold several on one device, or reset
// a device, and an address resolved in another context would point at
// invalid memory. So the first call in each context (told apart by the
// driver's unique context id, which is never reused) resolves the address
// with cudaGetSymbolAddress while that context is current, checks the result
// and caches it under that id; that first call should come before any stream
// capture in the context. Every call shares the array and it keeps the previous
// call's contents: the call clears the part that must start at zero (its id
// segment table), and the scan overwrites the rest. Two calls whose work
// overlaps on the GPU (concurrent streams, or threads on the same device)
// race on the array; callers must order them.
//
// Limits: nq * (ncta + 1) * k * 8 bytes of candidate lists must fit in the
// array (the number of row splits ncta shrinks to make it fit; a request that
// does not fit even with one split is rejected), dim must be a multiple of 4
// and the base 16-byte aligned (the scan reads rows with 128-bit loads),
// n < 2^32, and one query's row plus its candidate buffer must fit in a
// block's shared memory (about dim <= 50,000 at k <= 768 on B200).
#include <algorithm>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include <cuda.h>

#include "../../include/px.h"
#include "px_common.cuh"
#include "px_kernels.h"
#include "px_runtime.h"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr size_t kSegBytes = 256;  // zeroed (local_begin, global_begin) table

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// The driver's current context and its process-unique id, through the
// runtime's driver entry points (the library links no libcuda).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

struct CtxFns {
  CtxGetCurrentFn get_current = nullptr;
  CtxGetIdFn get_id = nullptr;
};

const CtxFns& ctx_fns() {
  static const CtxFns fns = [] {
    CtxFns f;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.get_id = reinterpret_cast<CtxGetIdFn>(p);
    cudaGetLastError();
    return f;
  }();
  return fns;
}

// Id of the current context, or 0 when there is none yet or it cannot be read.
unsigned long long current_ctx_id() {
  const CtxFns& f = ctx_fns();
  if (!f.get_current || !f.get_id) return 0;
  CUcontext ctx = nullptr;
  if (f.get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (f.get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

constexpr size_t kMaxContexts = 64;
std::mutex g_scratch_mu;
std::vector<std::pair<unsigned long long, void*>> g_scratch_addr;  // (context id, address), newest last

px_status lookup_scratch(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr)
    return px::cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                           "cudaGetSymbolAddress(no-allocation scratch)");
  *out = p;
  return PX_OK;
}

// The scratch array's device address in the current context.
px_status scratch_for_current_context(void** out) {
  unsigned long long id = current_ctx_id();
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (id != 0) {
    for (const auto& kv : g_scratch_addr)
      if (kv.first == id) {
        *out = kv.second;
        return PX_OK;
      }
  }
  // Not seen before, or no context bound yet: the runtime binds the device's
  // primary context during this lookup.
  px_status s = lookup_scratch(out);
  if (s != PX_OK) return s;
  if (id == 0) id = current_ctx_id();
  if (id != 0) {
    if (g_scratch_addr.size() >= kMaxContexts) g_scratch_addr.erase(g_scratch_addr.begin());
    g_scratch_addr.emplace_back(id, *out);
  }
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
  const int group = px::exact_group_for(nq, k, dim, px::device_smem_optin(dev));
  if (group == 0)
    return set_error(PX_EUNSUPPORTED, "dim=" + std::to_string(dim) + " with k=" + std::to_string(k) +
                                          " exceeds the exact scan's shared memory");
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
  px_status s = scratch_for_current_context(&base);
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
