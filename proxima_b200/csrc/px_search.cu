// Flat-search planning and execution on one shard.
//
// Paths:
//   Exact (K2)  : the exact streaming scan; bit-exact keys, no rescoring.
//                 Serves small batches (nq < kGemmMinQueries) and k beyond
//                 the tensor-core path's candidate capacity.
//   Gemm (K1+K5): 3xTF32 tcgen05 contraction with a fused per-query
//                 top-CAP, split merge, exact rescoring and a certificate;
//                 queries whose certificate fails are re-run through K2.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <numeric>
#include <vector>

#include "px_common.cuh"
#include "px_runtime.h"

namespace px {

std::atomic<int64_t> g_launches{0};
std::atomic<int> g_profiling{0};

namespace {

constexpr int kGemmMinQueries = 16;
constexpr int kGemmMinRows = 4096;

int64_t gcd64(int64_t a, int64_t b) {
  while (b) {
    int64_t t = a % b;
    a = b;
    b = t;
  }
  return a;
}

}  // namespace

px_status plan_flat_search(const px_flat* h, const FlatShard& sh, int64_t nq, int k, bool masked,
                           SearchPlan& plan) {
  plan = SearchPlan{};
  const int cap = gemm_cap_for(k);
  bool gemm = cap > 0 && h->ld % 32 == 0 && sh.hl != nullptr;
  if (h->path_mode == PX_PATH_EXACT) gemm = false;
  if (h->path_mode == PX_PATH_AUTO) gemm = gemm && nq >= kGemmMinQueries && sh.n >= kGemmMinRows;
  if (h->path_mode == PX_PATH_TENSOR && !gemm)
    return set_error(PX_EUNSUPPORTED, "the tensor-core path cannot serve this request (k, mask or layout)");
  if (nq > (int64_t(1) << 30)) return set_error(PX_EUNSUPPORTED, "too many queries in one call");
  Carver c;
  if (gemm) {
    plan.path = FlatPath::Gemm;
    plan.cap = cap;
    plan.cands = gemm_cands_for(k);
    // Work items: (group of QT query tiles, run of base tiles of BN rows).
    const int qt = gemm_qt_for(k);
    const int bn = gemm_bn_for(k);
    const int64_t T = ((nq + 127) / 128 + qt - 1) / qt;
    const int64_t nb = std::max<int64_t>(1, (sh.n + bn - 1) / bn);
    // Splits so that T * S is a whole number of waves of one CTA per SM.
    int64_t S = sh.sms / gcd64(T, sh.sms);
    while (S * 2 <= 1024 && S * T < 2 * sh.sms && S * 2 <= nb) S *= 2;
    S = std::min<int64_t>(S, nb);
    S = std::max<int64_t>(S, 1);
    const int64_t tps = (nb + S - 1) / S;
    S = (nb + tps - 1) / tps;
    plan.T = static_cast<int>(T);
    plan.S = static_cast<int>(S);
    plan.nb = static_cast<int>(nb);
    plan.tiles_per_split = static_cast<int>(tps);
    plan.n_items = static_cast<int>(T * S);
    plan.grid = static_cast<int>(std::min<int64_t>(sh.sms, T * S));
    plan.q_rows = T * qt * 128;
    c.take(sizeof(float) * static_cast<size_t>(plan.q_rows) * 2 * h->ld);  // query split plane
    c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * S * cap);      // split lists
    c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * plan.cands);   // merged
    c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * k);            // final
    c.take(sizeof(int) * static_cast<size_t>(nq));                     // status
    c.take(sizeof(int) * static_cast<size_t>(nq));                     // fail list
    c.take(sizeof(int) * 4);                                           // counters
    if (masked) c.take(sizeof(uint32_t) * static_cast<size_t>((sh.n + 31) / 32 + 8));  // mask bits
  } else {
    plan.path = FlatPath::Exact;
    const int group = exact_group_for(nq);
    const int64_t groups = (nq + group - 1) / group;
    if (groups > 65535) return set_error(PX_EUNSUPPORTED, "too many queries in one call");
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
    c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * ncta * k);
    c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * k);
  }
  plan.ws_bytes = c.used;
  return PX_OK;
}

static px_status run_exact(const px_flat* h, FlatShard& sh, int metric, const float* d_q, int64_t nq,
                           int k, const uint8_t* d_mask, uint64_t* partial, int ncta, int group,
                           int64_t rows_per_cta, uint64_t* out, cudaStream_t stream, bool profile_main) {
  ExactScanArgs a;
  a.base = sh.x;
  a.n = sh.n;
  a.ld = h->ld;
  a.d = h->dim;
  a.queries = d_q;
  a.nq = static_cast<int>(nq);
  a.k = k;
  a.group = group;
  a.ncta = ncta;
  a.rows_per_cta = rows_per_cta;
  a.mask = d_mask;
  a.l2 = metric == PX_METRIC_L2;
  a.partial = partial;
  if (profile_main) cudaEventRecord(sh.ev_start, stream);
  cudaError_t e = launch_exact_scan(a, stream);
  if (profile_main) cudaEventRecord(sh.ev_stop, stream);
  if (e != cudaSuccess) return cuda_status(e, "exact scan launch");
  e = launch_merge_lists(partial, nq, ncta, k, k, out, stream);
  if (e != cudaSuccess) return cuda_status(e, "merge launch");
  g_launches += 2;
  return PX_OK;
}

px_status run_flat_search(const px_flat* h, FlatShard& sh, SearchPlan& plan, int metric,
                          const float* d_q, int64_t nq, int k, const uint8_t* d_mask,
                          cudaStream_t stream) {
  const bool prof = g_profiling.load() != 0;
  sh.last_path = static_cast<int>(plan.path);
  sh.last_fallback = 0;
  sh.last_profiled = prof;
  const int64_t launches0 = g_launches.load();
  Carver c(sh.ws.ptr);
  if (plan.path == FlatPath::Exact) {
    plan.partial = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * plan.ncta * k));
    plan.final_cands = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * k));
    px_status s = run_exact(h, sh, metric, d_q, nq, k, d_mask, plan.partial, plan.ncta, plan.group,
                            plan.rows_per_cta, plan.final_cands, stream, prof);
    sh.last_launches = static_cast<int>(g_launches.load() - launches0);
    return s;
  }

  // ---- tensor-core path ----
  const int cap = plan.cap;
  float* q_hl = static_cast<float*>(c.take(sizeof(float) * static_cast<size_t>(plan.q_rows) * 2 * h->ld));
  uint64_t* partial = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * plan.S * cap));
  const int cands = plan.cands;
  uint64_t* merged = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * cands));
  plan.final_cands = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * k));
  int* status = static_cast<int*>(c.take(sizeof(int) * static_cast<size_t>(nq)));
  int* fail_list = static_cast<int*>(c.take(sizeof(int) * static_cast<size_t>(nq)));
  int* counters = static_cast<int*>(c.take(sizeof(int) * 4));  // [0] n_fail, [1] q lo flag
  uint32_t* mask_bits =
      d_mask ? static_cast<uint32_t*>(c.take(sizeof(uint32_t) * static_cast<size_t>((sh.n + 31) / 32 + 8))) : nullptr;
  const bool l2 = metric == PX_METRIC_L2;

  cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(int) * 4, stream);
  if (e == cudaSuccess) e = launch_split_queries(d_q, nq, h->dim, h->ld, plan.q_rows, q_hl, counters + 1, stream);
  if (e == cudaSuccess && mask_bits) e = launch_pack_mask(d_mask, sh.n, mask_bits, stream);
  if (e != cudaSuccess) return cuda_status(e, "query split");
  // One pass over the hi halves suffices when neither side has a lo part
  // (e.g. integer-valued data); the query side is known only after the split.
  bool hi_only = false;
  if (!sh.lo_nonzero) {
    int q_lo_host = 1;
    e = cudaMemcpyAsync(&q_lo_host, counters + 1, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_status(e, "query split readback");
    hi_only = q_lo_host == 0;
  }
  GemmTopkArgs g;
  g.nq = static_cast<int>(nq);
  g.n = sh.n;
  g.ld = h->ld;
  g.k = k;
  g.T = plan.T;
  g.S = plan.S;
  g.tiles_per_split = plan.tiles_per_split;
  g.nb = plan.nb;
  g.n_items = plan.n_items;
  g.l2 = l2;
  g.norms = sh.norms;
  g.x_lo_nonzero = sh.lo_nonzero ? 1 : 0;
  g.q_lo_flag = counters + 1;
  g.partial = partial;
  g.err = sh.flag + 1;
  g.mask_bits = mask_bits;
  if (prof) cudaEventRecord(sh.ev_start, stream);
  e = launch_gemm_topk(g, q_hl, plan.q_rows, sh.hl, hi_only, plan.grid, stream);
  if (prof) cudaEventRecord(sh.ev_stop, stream);
  if (e != cudaSuccess) return cuda_status(e, "tensor-core kernel launch");
  e = launch_merge_lists(partial, nq, plan.S, cap, cands, merged, stream);
  if (e != cudaSuccess) return cuda_status(e, "split merge launch");
  RescoreArgs r;
  r.merged = merged;
  r.nq = nq;
  r.cap = cands;
  r.k = k;
  r.lists = partial;
  r.nlists = plan.S;
  r.list_cap = cap;
  r.queries = d_q;
  r.base = sh.x;
  r.ld = h->ld;
  r.d = h->dim;
  r.l2 = l2;
  r.max_norm = std::sqrt(sh.max_norm_sq);
  r.x_lo_nonzero = sh.lo_nonzero ? 1 : 0;
  r.q_lo_flag = counters + 1;
  r.out = plan.final_cands;
  r.status = status;
  r.n_fail = counters;
  r.fail_list = fail_list;
  e = launch_rescore(r, stream);
  if (e != cudaSuccess) return cuda_status(e, "rescore launch");
  g_launches += 5;  // split, gemm, merge, rescore (+ memset counted as one)

  // Certificate failures: re-run those queries through the exact scan.
  int n_fail = 0;
  e = cudaMemcpyAsync(&n_fail, counters, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_status(e, "certificate readback");
  px_status s = check_device_flags(sh);
  if (s != PX_OK) return s;
  sh.last_fallback = n_fail;
  if (n_fail > 0) {
    const int group = exact_group_for(n_fail);
    const int64_t groups = (n_fail + group - 1) / group;
    const int64_t n = std::max<int64_t>(sh.n, 1);
    int64_t ncta = std::max<int64_t>(1, (static_cast<int64_t>(sh.sms) * 4 + groups - 1) / groups);
    ncta = std::min<int64_t>(std::min<int64_t>(ncta, (n + 127) / 128), 1024);
    int64_t rows = ((n + ncta - 1) / ncta + 127) / 128 * 128;
    ncta = (n + rows - 1) / rows;
    Carver fc;
    fc.take(sizeof(float) * static_cast<size_t>(n_fail) * h->dim);
    fc.take(sizeof(uint64_t) * static_cast<size_t>(n_fail) * ncta * k);
    fc.take(sizeof(uint64_t) * static_cast<size_t>(n_fail) * k);
    e = sh.fb.reserve(fc.used);
    if (e != cudaSuccess) return cuda_status(e, "fallback workspace allocation");
    fc = Carver(sh.fb.ptr);
    float* fq = static_cast<float*>(fc.take(sizeof(float) * static_cast<size_t>(n_fail) * h->dim));
    uint64_t* fpart = static_cast<uint64_t*>(fc.take(sizeof(uint64_t) * static_cast<size_t>(n_fail) * ncta * k));
    uint64_t* fout = static_cast<uint64_t*>(fc.take(sizeof(uint64_t) * static_cast<size_t>(n_fail) * k));
    e = launch_gather_rows(d_q, h->dim, fail_list, n_fail, fq, stream);
    if (e != cudaSuccess) return cuda_status(e, "fallback gather");
    s = run_exact(h, sh, metric, fq, n_fail, k, d_mask, fpart, static_cast<int>(ncta), group, rows, fout,
                  stream, false);
    if (s != PX_OK) return s;
    e = launch_scatter_cands(fout, k, fail_list, n_fail, plan.final_cands, stream);
    if (e != cudaSuccess) return cuda_status(e, "fallback scatter");
    g_launches += 2;
  }
  sh.last_launches = static_cast<int>(g_launches.load() - launches0);
  return PX_OK;
}

px_status check_device_flags(FlatShard& sh) {
  int err = 0;
  cudaError_t e = cudaMemcpy(&err, sh.flag + 1, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "device status readback");
  if (err != 0) {
    cudaMemset(sh.flag + 1, 0, sizeof(int));
    return set_error(PX_ETIMEOUT, "a tensor-core pipeline wait timed out on device " +
                                      std::to_string(sh.device) + "; the search was abandoned");
  }
  return PX_OK;
}

}  // namespace px

px_status GatherBuf::ensure(int dev, size_t entries) {
  if (device == dev && entries <= cap) return PX_OK;
  release_all();
  device = dev;
  px::DeviceGuard dg(dev);
  cudaError_t e = cudaMalloc(&keys, entries * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&ids, entries * sizeof(int64_t));
  if (e == cudaSuccess) e = cudaMalloc(&out_dists, entries * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&out_ids, entries * sizeof(int64_t));
  if (e != cudaSuccess) {
    cudaGetLastError();
    release_all();
    return px::cuda_status(e, "gather buffer allocation");
  }
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
  keys = out_dists = nullptr;
  ids = out_ids = nullptr;
  cap = 0;
  device = -1;
}
