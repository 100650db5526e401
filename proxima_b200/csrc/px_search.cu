// Flat-search planning: chooses the kernel path for a shard and lays out its
// workspace. The exact streaming scan (K2) serves small batches and any
// request the tensor-core path cannot take.
#include <algorithm>

#include "px_common.cuh"
#include "px_runtime.h"

px_status GatherBuf::ensure(int dev, size_t entries) {
  if (device == dev && entries <= cap) return PX_OK;
  release_all();
  px::DeviceGuard dg(dev);
  cudaError_t e = cudaMalloc(&keys, entries * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&ids, entries * sizeof(int64_t));
  if (e == cudaSuccess) e = cudaMalloc(&out_dists, entries * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&out_ids, entries * sizeof(int64_t));
  for (auto& ev : events)
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    release_all();
    return px::cuda_status(e, "gather buffer allocation");
  }
  device = dev;
  cap = entries;
  return PX_OK;
}

void GatherBuf::release_all() {
  if (device >= 0) {
    px::DeviceGuard dg(device);
    if (keys) cudaFree(keys);
    if (ids) cudaFree(ids);
    if (out_dists) cudaFree(out_dists);
    if (out_ids) cudaFree(out_ids);
  }
  for (auto& ev : events) {
    if (ev) cudaEventDestroy(ev);
    ev = nullptr;
  }
  keys = out_dists = nullptr;
  ids = out_ids = nullptr;
  cap = 0;
  device = -1;
}

namespace px {

px_status plan_flat_search(const px_flat* h, const FlatShard& sh, int64_t nq, int k, SearchPlan& plan) {
  plan = SearchPlan{};
  plan.path = FlatPath::Exact;
  const int group = exact_group_for(nq);
  const int64_t groups = (nq + group - 1) / group;
  if (groups > 65535) return set_error(PX_EUNSUPPORTED, "too many queries in one call");
  // Aim for about four resident CTAs per SM across the whole grid.
  const int64_t target = static_cast<int64_t>(sh.sms) * 4;
  int64_t ncta = std::max<int64_t>(1, (target + groups - 1) / groups);
  const int64_t n = std::max<int64_t>(sh.n, 1);
  ncta = std::min<int64_t>(ncta, (n + 127) / 128);
  ncta = std::min<int64_t>(ncta, 1024);
  int64_t rows = (n + ncta - 1) / ncta;
  rows = (rows + 127) / 128 * 128;
  ncta = (n + rows - 1) / rows;
  plan.group = group;
  plan.ncta = static_cast<int>(ncta);
  plan.rows_per_cta = rows;
  Carver c;
  c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * ncta * k);
  c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * k);
  plan.ws_bytes = c.used;
  (void)h;
  return PX_OK;
}

px_status run_flat_search(const px_flat* h, FlatShard& sh, SearchPlan& plan, int metric,
                          const float* d_q, int64_t nq, int k, const uint8_t* d_mask,
                          cudaStream_t stream) {
  Carver c(sh.ws.ptr);
  plan.partial = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * plan.ncta * k));
  plan.final_cands = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * k));
  ExactScanArgs a;
  a.base = sh.x;
  a.n = sh.n;
  a.ld = h->ld;
  a.d = h->dim;
  a.queries = d_q;
  a.nq = static_cast<int>(nq);
  a.k = k;
  a.group = plan.group;
  a.ncta = plan.ncta;
  a.rows_per_cta = plan.rows_per_cta;
  a.mask = d_mask;
  a.l2 = metric == PX_METRIC_L2;
  a.partial = plan.partial;
  cudaError_t e = launch_exact_scan(a, stream);
  if (e != cudaSuccess) return cuda_status(e, "exact scan launch");
  e = launch_merge_lists(plan.partial, nq, plan.ncta, k, k, plan.final_cands, stream);
  if (e != cudaSuccess) return cuda_status(e, "merge launch");
  return PX_OK;
}

px_status check_device_flags(FlatShard& sh) {
  (void)sh;
  return PX_OK;
}

}  // namespace px
