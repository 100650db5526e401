// Host runtime and C ABI of libproxima_b200 (declared in include/px.h).
//
// A handle owns one shard per device: the rows it holds (fp32, plus the tf32
// split planes and squared norms the tensor-core path reads), a stream, and
// grow-only workspaces, so a warmed-up search performs no device allocation.
// Searches run every shard on its own device and stream, gather the per-shard
// sorted top-k lists on the first device and merge them there (ties on the
// key go to the smaller global id).
//
// Validation and messages restate the reference's checks
// (crates/core/src/flat.rs:72-85, 106-123, 150-172; pq.rs:54-72, 266-309,
// 361-377; crates/py/src/lib.rs) as status codes instead of panics.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/px.h"
#include "px_common.cuh"
#include "px_kernels.h"
#include "px_runtime.h"

using namespace px;

namespace px {

thread_local std::string g_last_error;

px_status set_error(px_status s, const std::string& msg) {
  g_last_error = msg;
  return s;
}

px_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PX_OK;
  return set_error(e == cudaErrorMemoryAllocation ? PX_ENOMEM : PX_ECUDA,
                   std::string(what) + ": " + cudaGetErrorString(e));
}

DeviceGuard::DeviceGuard(int dev) {
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  cudaSetDevice(dev);
}
DeviceGuard::~DeviceGuard() {
  if (prev >= 0) cudaSetDevice(prev);
}

cudaError_t DevBuf::reserve(size_t need) {
  if (need <= bytes) return cudaSuccess;
  release();
  cudaError_t e = cudaMalloc(&ptr, need);
  if (e != cudaSuccess) {
    ptr = nullptr;
    cudaGetLastError();
    return e;
  }
  bytes = need;
  return cudaSuccess;
}

void DevBuf::release() {
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  bytes = 0;
}

// Carves 256-byte aligned sub-buffers out of one reserved block.
void* Carver::take(size_t bytes) {
  size_t off = (used + 255) & ~size_t(255);
  used = off + bytes;
  return base ? static_cast<char*>(base) + off : nullptr;
}

bool is_pinned(const void* p) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return attr.type == cudaMemoryTypeHost;
}

px_status HostBuf::reserve(size_t need) {
  if (need <= bytes) return PX_OK;
  release();
  cudaError_t e = cudaMallocHost(&ptr, need);
  if (e != cudaSuccess) {
    ptr = nullptr;
    cudaGetLastError();
    return set_error(PX_ENOMEM, std::string("pinned staging allocation failed: ") + cudaGetErrorString(e));
  }
  bytes = need;
  return PX_OK;
}

void HostBuf::release() {
  if (ptr) cudaFreeHost(ptr);
  ptr = nullptr;
  bytes = 0;
}

// A float is NaN or infinite exactly when its exponent bits are all ones.
// The loop has no early exit, so the compiler vectorizes it; inputs of more
// than 2M values are split over host threads, at least 1M values each
// (config 4's 10k queries are 7.7M values, 1.9 ms on one core and 0.45 ms on
// seven; a host add can be billions).
// The same loop built for AVX2 (eight values per compare) runs at about twice
// the rate of the baseline-x86-64 build (config 1's 384k query values: 62
// against 121 us); it is used only where the CPU reports AVX2.
static bool finite_range_portable(const float* p, size_t count) {
  const uint32_t* u = reinterpret_cast<const uint32_t*>(p);
  uint32_t bad = 0;
  for (size_t i = 0; i < count; ++i) bad |= (u[i] & 0x7f800000u) == 0x7f800000u ? 1u : 0u;
  return bad == 0;
}

#if defined(__x86_64__)
__attribute__((target("avx2"))) static bool finite_range_avx2(const float* p, size_t count) {
  const uint32_t* u = reinterpret_cast<const uint32_t*>(p);
  uint32_t bad = 0;
  for (size_t i = 0; i < count; ++i) bad |= (u[i] & 0x7f800000u) == 0x7f800000u ? 1u : 0u;
  return bad == 0;
}
#endif

static bool finite_range(const float* p, size_t count) {
#if defined(__x86_64__)
  static const bool avx2 = __builtin_cpu_supports("avx2");
  if (avx2) return finite_range_avx2(p, count);
#endif
  return finite_range_portable(p, count);
}

bool all_finite(const float* p, int64_t count) {
  if (count <= 0) return true;
  const size_t n = static_cast<size_t>(count);
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const size_t threads = std::min<size_t>(std::min<size_t>(hw, 32), n / (size_t(1) << 20));
  if (threads <= 1) return finite_range(p, n);
  std::vector<char> ok(threads, 1);
  std::vector<std::thread> pool;
  const size_t per = (n + threads - 1) / threads;
  for (size_t t = 0; t < threads; ++t) {
    const size_t b = t * per, e = std::min(n, b + per);
    pool.emplace_back([&, t, b, e] { ok[t] = finite_range(p + b, e - b) ? 1 : 0; });
  }
  for (auto& th : pool) th.join();
  for (char o : ok)
    if (!o) return false;
  return true;
}

int device_sm_count(int dev) {
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 148;
  return sms;
}

size_t device_smem_optin(int dev) {
  static std::atomic<int> cached[64] = {};
  if (dev >= 0 && dev < 64 && cached[dev].load() > 0) return static_cast<size_t>(cached[dev].load());
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0) {
    cudaGetLastError();
    v = 48 * 1024;  // the limit every device offers
  }
  if (dev >= 0 && dev < 64) cached[dev] = v;
  return static_cast<size_t>(v);
}

px_status resolve_devices(const int32_t* devices, int32_t ndev, std::vector<int>& out) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();
    return set_error(PX_ECUDA, std::string("no CUDA device available: ") +
                                   (e == cudaSuccess ? "device count is 0" : cudaGetErrorString(e)));
  }
  out.clear();
  if (devices == nullptr || ndev <= 0) {
    int cur = 0;
    cudaGetDevice(&cur);
    out.push_back(cur);
    return PX_OK;
  }
  if (ndev > 8) return set_error(PX_EINVAL, "at most 8 devices per handle");
  for (int i = 0; i < ndev; ++i) {
    if (devices[i] < 0 || devices[i] >= count)
      return set_error(PX_EINVAL, "device ordinal " + std::to_string(devices[i]) +
                                      " out of range (visible devices: " + std::to_string(count) + ")");
    for (int j = 0; j < i; ++j)
      if (devices[j] == devices[i]) return set_error(PX_EINVAL, "duplicate device ordinal");
    out.push_back(devices[i]);
  }
  return PX_OK;
}

// Splits n rows into `parts` contiguous runs (remainder spread over the first).
void split_rows(int64_t n, int parts, std::vector<int64_t>& begin, std::vector<int64_t>& count) {
  begin.resize(parts);
  count.resize(parts);
  int64_t base = n / parts, rem = n % parts, at = 0;
  for (int p = 0; p < parts; ++p) {
    count[p] = base + (p < rem ? 1 : 0);
    begin[p] = at;
    at += count[p];
  }
}

px_status Segments::sync_device() {
  if (!dirty) return PX_OK;
  const size_t need = sizeof(int64_t) * 2 * std::max<size_t>(1, local.size());
  cudaError_t e = dev.reserve(need);
  if (e != cudaSuccess) return cuda_status(e, "segment table allocation");
  std::vector<int64_t> host(2 * std::max<size_t>(1, local.size()), 0);
  for (size_t i = 0; i < local.size(); ++i) {
    host[i] = local[i];
    host[local.size() + i] = global[i];
  }
  e = cudaMemcpy(dev.ptr, host.data(), sizeof(int64_t) * host.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_status(e, "segment table upload");
  dirty = false;
  return PX_OK;
}

IdSegments Segments::view(int64_t id_offset) const {
  IdSegments s;
  const size_t ns = std::max<size_t>(1, local.size());
  s.local_begin = static_cast<const int64_t*>(dev.ptr);
  s.global_begin = static_cast<const int64_t*>(dev.ptr) + ns;
  s.nseg = static_cast<int>(local.empty() ? 1 : local.size());
  s.id_offset = id_offset;
  return s;
}

// Builds the shard-local mask from a global one through the segment table.
void Segments::local_mask(const uint8_t* global_mask, int64_t n_local, std::vector<uint8_t>& out) const {
  out.assign(static_cast<size_t>(n_local), 0);
  for (size_t i = 0; i < local.size(); ++i) {
    int64_t end = (i + 1 < local.size()) ? local[i + 1] : n_local;
    std::memcpy(out.data() + local[i], global_mask + global[i], static_cast<size_t>(end - local[i]));
  }
}

}  // namespace px

// ===========================================================================
// FlatIndex
// ===========================================================================

px_status FlatShard::ensure_capacity(int64_t need, int ld, int ldb) {
  if (need <= cap) return PX_OK;
  int64_t new_cap = std::max<int64_t>(need, cap + cap / 2);
  const size_t row_bytes = sizeof(float) * ld;
  const size_t brow_bytes = 2 * static_cast<size_t>(ldb);
  size_t free_b = 0, total_b = 0;
  if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess) {
    const size_t need_b = static_cast<size_t>(new_cap) * (3 * row_bytes + brow_bytes + sizeof(float));
    if (need_b > free_b && new_cap > need) {
      new_cap = need;  // drop the growth slack before giving up
    }
  }
  float *nx = nullptr, *nhl = nullptr, *nn = nullptr;
  void* nxb = nullptr;
  const size_t pb = static_cast<size_t>(new_cap) * row_bytes;
  cudaError_t e = cudaMalloc(&nx, pb);
  if (e == cudaSuccess) e = cudaMalloc(&nhl, 2 * pb);
  if (e == cudaSuccess) e = cudaMalloc(&nxb, static_cast<size_t>(new_cap) * brow_bytes);
  // Norms are padded to a whole number of 256-row tiles: the tensor-core
  // epilogue reads them 32 rows at a time, past the last row of a shard.
  const int64_t norm_cap = (new_cap + 255) / 256 * 256;
  if (e == cudaSuccess) e = cudaMalloc(&nn, sizeof(float) * norm_cap);
  if (e == cudaSuccess) e = cudaMemset(nn, 0, sizeof(float) * norm_cap);
  if (e != cudaSuccess) {
    cudaGetLastError();
    if (nx) cudaFree(nx);
    if (nhl) cudaFree(nhl);
    if (nxb) cudaFree(nxb);
    if (nn) cudaFree(nn);
    return set_error(PX_ENOMEM, "device allocation of " + std::to_string(new_cap) +
                                    " rows failed on device " + std::to_string(device) + ": " +
                                    cudaGetErrorString(e));
  }
  if (n > 0) {
    const size_t used = static_cast<size_t>(n) * row_bytes;
    cudaMemcpyAsync(nx, x, used, cudaMemcpyDeviceToDevice, stream);
    cudaMemcpyAsync(nhl, hl, 2 * used, cudaMemcpyDeviceToDevice, stream);
    cudaMemcpyAsync(nxb, xb, static_cast<size_t>(n) * brow_bytes, cudaMemcpyDeviceToDevice, stream);
    cudaMemcpyAsync(nn, norms, sizeof(float) * n, cudaMemcpyDeviceToDevice, stream);
    cudaStreamSynchronize(stream);
  }
  if (x) cudaFree(x);
  if (hl) cudaFree(hl);
  if (xb) cudaFree(xb);
  if (norms) cudaFree(norms);
  x = nx;
  hl = nhl;
  xb = nxb;
  norms = nn;
  cap = new_cap;
  return PX_OK;
}

void FlatShard::release() {
  DeviceGuard g(device);
  if (stream) cudaStreamSynchronize(stream);
  if (x) cudaFree(x);
  if (hl) cudaFree(hl);
  if (xb) cudaFree(xb);
  if (norms) cudaFree(norms);
  x = hl = norms = nullptr;
  xb = nullptr;
  if (flag) cudaFree(flag);
  flag = nullptr;
  if (ev_start) cudaEventDestroy(ev_start);
  if (ev_stop) cudaEventDestroy(ev_stop);
  if (ev_done) cudaEventDestroy(ev_done);
  ev_start = ev_stop = ev_done = nullptr;
  fb.release();
  ws2.release();
  ws.release();
  stage.release();
  segs.dev.release();
  if (counters_h) cudaFreeHost(counters_h);
  counters_h = nullptr;
  if (stream) cudaStreamDestroy(stream);
  stream = nullptr;
}

// Appends rows that are already on this shard's device.
px_status FlatShard::append_device(const float* d_src, int64_t count, int d, int ld, int ldb,
                                   int64_t global_begin) {
  px_status s = ensure_capacity(n + count, ld, ldb);
  if (s != PX_OK) return s;
  cudaError_t e = launch_prepare_rows(d_src, count, d, ld, ldb, x + n * ld, hl + n * 2 * ld,
                                      static_cast<uint16_t*>(xb) + n * ldb, norms + n, flag, flag + 1,
                                      flag + 2, stream, false, flag + 3);
  if (e != cudaSuccess) return cuda_status(e, "prepare_rows launch");
  segs.local.push_back(n);
  segs.global.push_back(global_begin);
  segs.dirty = true;
  n += count;
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_status(e, "add");
  int h_flag[kShardFlags] = {};
  e = cudaMemcpy(h_flag, flag, sizeof(h_flag), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "add flag readback");
  lo_nonzero = h_flag[0] != 0;
  bf_inexact = h_flag[1] != 0;
  std::memcpy(&max_norm_sq, &h_flag[2], sizeof(float));
  std::memcpy(&bf_resid, &h_flag[3], sizeof(float));
  std::memcpy(&tf_resid, &h_flag[4], sizeof(float));
  g_launches += 1;
  return PX_OK;
}

static void clear_flat_graphs(px_flat* h);

static px_status flat_check(const px_flat* h) {
  if (h == nullptr) return set_error(PX_EINVAL, "null handle");
  return PX_OK;
}

extern "C" {

PX_API const char* px_last_error(void) { return g_last_error.c_str(); }
PX_API const char* px_version(void) { return "proxima_b200 0.1.0 (sm_100a)"; }

PX_API int32_t px_device_count(void) {
  int c = 0;
  if (cudaGetDeviceCount(&c) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return c;
}

PX_API px_status px_flat_create(int32_t dim, int32_t metric, const int32_t* devices, int32_t ndev,
                                px_flat** out) {
  if (out == nullptr) return set_error(PX_EINVAL, "out is null");
  *out = nullptr;
  if (dim <= 0) return set_error(PX_EINVAL, "dim must be > 0");
  if (metric != PX_METRIC_L2 && metric != PX_METRIC_IP)
    return set_error(PX_EINVAL, "metric must be 0 (L2) or 1 (inner product)");
  std::vector<int> devs;
  px_status s = resolve_devices(devices, ndev, devs);
  if (s != PX_OK) return s;
  px_flat* h = new px_flat();
  h->dim = dim;
  h->ld = (dim + 31) & ~31;
  // bf16 rows: dim rounded up to 64, so one 128-byte TMA row is one K slice.
  // An L2 index of dim <= 256 also keeps room after the dim columns for each
  // row's folded norm (three bf16 values): at small dim the bf16 pass is
  // bound by its epilogue, and folding removes the epilogue's per-element
  // norm term for at most one more K slice.
  h->ldb = (dim + 63) & ~63;
  if (metric == PX_METRIC_L2 && dim <= 256 && dim + 3 > h->ldb) h->ldb += 64;
  h->metric = metric;
  h->shards.resize(devs.size());
  for (size_t i = 0; i < devs.size(); ++i) {
    FlatShard& sh = h->shards[i];
    sh.device = devs[i];
    DeviceGuard g(sh.device);
    cudaError_t e = cudaStreamCreateWithFlags(&sh.stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&sh.flag, kShardFlags * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(sh.flag, 0, kShardFlags * sizeof(int));
    if (e == cudaSuccess) e = cudaEventCreate(&sh.ev_start);
    if (e == cudaSuccess) e = cudaEventCreate(&sh.ev_stop);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sh.ev_done, cudaEventDisableTiming);
    if (e != cudaSuccess) {
      px_status st = cuda_status(e, "create");
      for (auto& x : h->shards) x.release();
      delete h;
      return st;
    }
    sh.sms = device_sm_count(sh.device);
  }
  *out = h;
  return PX_OK;
}

PX_API px_status px_flat_destroy(px_flat* h) {
  if (h == nullptr) return PX_OK;
  {
    std::lock_guard<std::mutex> lk(h->mu);
    clear_flat_graphs(h);
    for (auto& sh : h->shards) sh.release();
    h->gather.release_all();
    h->pinned.release();
  }
  delete h;
  return PX_OK;
}

PX_API int64_t px_flat_size(const px_flat* h) { return h ? h->total : 0; }
PX_API int32_t px_flat_dim(const px_flat* h) { return h ? h->dim : 0; }
PX_API int32_t px_flat_metric(const px_flat* h) { return h ? h->metric : -1; }

PX_API px_status px_flat_set_path(px_flat* h, int32_t mode) {
  px_status s = flat_check(h);
  if (s != PX_OK) return s;
  if (mode != PX_PATH_AUTO && mode != PX_PATH_EXACT && mode != PX_PATH_TENSOR && mode != PX_PATH_TENSOR_3XTF32)
    return set_error(PX_EINVAL,
                     "path mode must be PX_PATH_AUTO, PX_PATH_EXACT, PX_PATH_TENSOR or PX_PATH_TENSOR_3XTF32");
  h->path_mode = mode;
  return PX_OK;
}

PX_API px_status px_flat_set_sample_pass(px_flat* h, int32_t mode) {
  px_status s = flat_check(h);
  if (s != PX_OK) return s;
  if (mode != PX_SAMPLE_AUTO && mode != PX_SAMPLE_OFF && mode != PX_SAMPLE_ON)
    return set_error(PX_EINVAL, "sample pass mode must be PX_SAMPLE_AUTO, PX_SAMPLE_OFF or PX_SAMPLE_ON");
  h->sample_mode = mode;
  return PX_OK;
}

PX_API void px_set_profiling(int32_t enable) { g_profiling = enable ? 1 : 0; }

PX_API int64_t px_launch_count(void) { return g_launches.load(); }

PX_API px_status px_flat_profile_totals(px_flat* h, int32_t reset, px_profile_totals* out) {
  px_status s = flat_check(h);
  if (s != PX_OK) return s;
  if (out == nullptr) return set_error(PX_EINVAL, "out is null");
  std::lock_guard<std::mutex> lk(h->mu);
  FlatShard& sh = h->shards[0];
  s = flush_search_profile(sh);
  if (s != PX_OK) return s;
  out->main_kernel_ms = sh.tot_ms;
  out->profiled_searches = sh.tot_profiled;
  out->searches = sh.tot_searches;
  out->fallback_queries = sh.tot_fallback;
  out->refined_queries = sh.tot_refined;
  if (reset) {
    sh.tot_ms = 0.0;
    sh.tot_profiled = sh.tot_searches = sh.tot_fallback = sh.tot_refined = 0;
  }
  return PX_OK;
}

PX_API px_status px_flat_last_profile(const px_flat* h, px_search_profile* out) {
  px_status s = flat_check(h);
  if (s != PX_OK) return s;
  if (out == nullptr) return set_error(PX_EINVAL, "out is null");
  const FlatShard& sh = h->shards[0];
  out->path = sh.last_path;
  out->launches = sh.last_launches;
  out->fallback_queries = sh.last_fallback;
  out->refined_queries = sh.last_refined;
  out->first_pass = sh.last_pass;
  out->sample_tiles = sh.last_sample_tiles;
  out->profiled = 0;
  out->main_kernel_ms = 0.f;
  if (sh.last_profiled) {
    DeviceGuard dg(sh.device);
    float ms = 0.f;
    cudaError_t e = cudaEventSynchronize(sh.ev_stop);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, sh.ev_start, sh.ev_stop);
    if (e != cudaSuccess) return cuda_status(e, "profile events");
    out->profiled = 1;
    out->main_kernel_ms = ms;
  }
  return PX_OK;
}

PX_API px_status px_flat_set_id_offset(px_flat* h, int64_t offset) {
  px_status s = flat_check(h);
  if (s != PX_OK) return s;
  if (offset < 0) return set_error(PX_EINVAL, "id offset must be >= 0");
  h->id_offset = offset;
  return PX_OK;
}

PX_API px_status px_flat_add(px_flat* h, const float* rows, int64_t n) {
  px_status s = flat_check(h);
  if (s != PX_OK) return s;
  if (n < 0) return set_error(PX_EINVAL, "row count must be >= 0");
  if (n == 0) return PX_OK;
  if (rows == nullptr) return set_error(PX_EINVAL, "rows is null");
  if (!all_finite(rows, n * h->dim))
    return set_error(PX_EINVAL, "vectors must not contain NaN or infinite values");
  std::lock_guard<std::mutex> lk(h->mu);
  clear_flat_graphs(h);  // the rows they read may move
  const int G = static_cast<int>(h->shards.size());
  std::vector<int64_t> begin, count;
  split_rows(n, G, begin, count);
  for (int g = 0; g < G; ++g) {
    if (count[g] == 0) continue;
    FlatShard& sh = h->shards[g];
    if (sh.n + count[g] > 0xFFFFFFFFll)
      return set_error(PX_EUNSUPPORTED, "a shard holds at most 2^32-1 rows");
    DeviceGuard dg(sh.device);
    // Stage the run in device memory (contiguous n x dim), then lay it out.
    const size_t bytes = sizeof(float) * static_cast<size_t>(count[g]) * h->dim;
    cudaError_t e = sh.stage.reserve(bytes);
    if (e != cudaSuccess) return cuda_status(e, "staging allocation");
    e = cudaMemcpyAsync(sh.stage.ptr, rows + begin[g] * h->dim, bytes, cudaMemcpyHostToDevice,
                        sh.stream);
    if (e != cudaSuccess) return cuda_status(e, "row upload");
    s = sh.append_device(static_cast<const float*>(sh.stage.ptr), count[g], h->dim, h->ld, h->ldb,
                         h->total + begin[g]);
    if (s != PX_OK) return s;
  }
  h->total += n;
  return PX_OK;
}

PX_API px_status px_flat_read_rows(const px_flat* hc, int64_t start, int64_t count, float* out) {
  px_status s = flat_check(hc);
  if (s != PX_OK) return s;
  if (start < 0 || count < 0 || start + count > hc->total)
    return set_error(PX_EINVAL, "row range out of bounds");
  if (count == 0) return PX_OK;
  if (out == nullptr) return set_error(PX_EINVAL, "out is null");
  px_flat* h = const_cast<px_flat*>(hc);
  std::lock_guard<std::mutex> lk(h->mu);
  for (auto& sh : h->shards) {
    DeviceGuard dg(sh.device);
    s = sh.segs.for_range(sh.n, start, start + count, [&](int64_t local, int64_t global, int64_t rows) {
      cudaError_t e = cudaMemcpy2D(out + (global - start) * h->dim, sizeof(float) * h->dim,
                                   sh.x + local * h->ld, sizeof(float) * h->ld, sizeof(float) * h->dim,
                                   static_cast<size_t>(rows), cudaMemcpyDeviceToHost);
      return cuda_status(e, "row readback");
    });
    if (s != PX_OK) return s;
  }
  return PX_OK;
}

PX_API px_status px_flat_reserve(px_flat* h, int64_t n_total) {
  px_status s = flat_check(h);
  if (s != PX_OK) return s;
  if (n_total < 0) return set_error(PX_EINVAL, "row count must be >= 0");
  std::lock_guard<std::mutex> lk(h->mu);
  clear_flat_graphs(h);  // the rows they read may move
  const int64_t G = static_cast<int64_t>(h->shards.size());
  const int64_t per = (n_total + G - 1) / G;
  for (auto& sh : h->shards) {
    if (per > 0xFFFFFFFFll) return set_error(PX_EUNSUPPORTED, "a shard holds at most 2^32-1 rows");
    DeviceGuard dg(sh.device);
    s = sh.ensure_capacity(std::max(per, sh.n), h->ld, h->ldb);
    if (s != PX_OK) return s;
  }
  return PX_OK;
}

PX_API px_status px_flat_add_device(px_flat* h, const float* d_rows, int64_t n) {
  px_status s = flat_check(h);
  if (s != PX_OK) return s;
  if (h->shards.size() != 1) return set_error(PX_EUNSUPPORTED, "px_flat_add_device needs a single-device handle");
  if (n < 0) return set_error(PX_EINVAL, "row count must be >= 0");
  if (n == 0) return PX_OK;
  std::lock_guard<std::mutex> lk(h->mu);
  clear_flat_graphs(h);  // the rows they read may move
  FlatShard& sh = h->shards[0];
  if (sh.n + n > 0xFFFFFFFFll) return set_error(PX_EUNSUPPORTED, "a shard holds at most 2^32-1 rows");
  DeviceGuard dg(sh.device);
  s = sh.append_device(d_rows, n, h->dim, h->ld, h->ldb, h->total);
  if (s != PX_OK) return s;
  h->total += n;
  return PX_OK;
}

}  // extern "C"

// A search of this shard has been enqueued in full: its counts go to the
// totals now, its kernel time (if profiled) when flush_search_profile runs.
static void note_search_done(FlatShard& sh) {
  sh.tot_searches += 1;
  sh.tot_fallback += sh.last_fallback;
  sh.tot_refined += sh.last_refined;
  if (sh.last_profiled) sh.prof_pending = true;  // an unprofiled search records no events
}

// Runs one shard's search on its device. d_q: nq x dim on the shard's device.
// Writes nq x k ids (global) and distances (natural or key space).
static px_status shard_search(const px_flat* h, FlatShard& sh, int metric, const float* d_q,
                              int64_t nq, int k, const uint8_t* d_mask, bool natural,
                              int64_t* d_ids, float* d_dists, cudaStream_t stream) {
  const bool l2 = metric == PX_METRIC_L2;
  px_status s = sh.segs.sync_device();
  if (s != PX_OK) return s;
  SearchPlan plan;
  s = plan_flat_search(h, sh, nq, k, d_mask != nullptr, plan);
  if (s != PX_OK) return s;
  cudaError_t e = sh.ws.reserve(plan.ws_bytes);
  if (e != cudaSuccess) return cuda_status(e, "search workspace allocation");
  // The emit is enqueued before the certificate is read back, so the stream
  // runs on without waiting for the host; the rare search with uncertified
  // queries emits again after their fallback.
  TensorPending pend;
  s = run_flat_search(h, sh, plan, metric, d_q, nq, k, d_mask, stream, nullptr, &pend);
  if (s != PX_OK) return s;
  e = launch_emit(plan.final_cands, nq, k, l2, natural, sh.segs.view(h->id_offset), d_ids, d_dists,
                  stream);
  if (e != cudaSuccess) return cuda_status(e, "emit launch");
  g_launches += 1;
  sh.last_launches += 1;
  if (pend.active) {
    bool changed = false;
    s = finish_flat_search(h, sh, pend, &changed);  // recounts the launches, the emit included
    if (s != PX_OK) return s;
    if (changed) {
      e = launch_emit(plan.final_cands, nq, k, l2, natural, sh.segs.view(h->id_offset), d_ids, d_dists,
                      stream);
      if (e != cudaSuccess) return cuda_status(e, "emit launch");
      g_launches += 1;
      sh.last_launches += 1;
    }
  }
  note_search_done(sh);
  return PX_OK;
}

// Small batches on a single-shard handle, when the plan is the exact scan (no
// host wait inside the search): the upload, scan, merge, emit and download
// are captured once as a CUDA graph and replayed, which replaces five
// launches and copies by one graph launch. Each graph owns its page-locked
// staging and its device buffers; besides those it reads only the shard's
// rows and segment table, and every call that can reallocate those first
// destroys the handle's graphs (clear_flat_graphs).
static constexpr size_t kMaxFlatGraphs = 8;

static void destroy_flat_graph(FlatSearchGraph& g) {
  if (g.exec) cudaGraphExecDestroy(g.exec);
  if (g.dev) cudaFree(g.dev);
  if (g.pinned) cudaFreeHost(g.pinned);
  g.exec = nullptr;
  g.dev = nullptr;
  g.pinned = nullptr;
}

static void clear_flat_graphs(px_flat* h) {
  if (h->graphs.empty()) return;
  DeviceGuard dg(h->shards[0].device);
  cudaStreamSynchronize(h->shards[0].stream);
  for (auto& g : h->graphs) destroy_flat_graph(g);
  h->graphs.clear();
}

// Sets *captured = false (and returns PX_OK) when the graph cannot be built,
// so the caller runs the search without one.
static px_status flat_search_replay(px_flat* h, FlatShard& sh, const SearchPlan& plan_in, int metric,
                                    const float* queries, int64_t nq, int32_t k, bool natural, int64_t* out_ids,
                                    float* out_dists, bool* captured) {
  *captured = true;
  // A graph captured with profiling on records the profiling events when it
  // is replayed: take the last profiled search's time first (and never wait
  // on an event inside the capture below).
  px_status fs = flush_search_profile(sh);
  if (fs != PX_OK) return fs;
  SearchPlan plan = plan_in;
  const size_t qbytes = sizeof(float) * static_cast<size_t>(nq) * h->dim;
  const size_t obytes = static_cast<size_t>(nq) * k;
  const size_t q_al = (qbytes + 15) & ~size_t(15);
  FlatSearchGraph key;
  key.nq = nq;
  key.n = sh.n;
  key.id_offset = h->id_offset;
  key.rows_per_cta = plan.rows_per_cta;
  key.k = k;
  key.metric = metric;
  key.natural = natural ? 1 : 0;
  key.group = plan.group;
  key.ncta = plan.ncta;
  auto same = [&](const FlatSearchGraph& g) {
    return g.nq == key.nq && g.n == key.n && g.id_offset == key.id_offset && g.rows_per_cta == key.rows_per_cta &&
           g.k == key.k && g.metric == key.metric && g.natural == key.natural && g.group == key.group &&
           g.ncta == key.ncta;
  };
  FlatSearchGraph* hit = nullptr;
  for (auto& g : h->graphs)
    if (same(g)) hit = &g;

  if (hit == nullptr) {
    // Buffers for this graph alone: [queries | ids | dists] page-locked, and
    // [queries | ids | dists | workspace] on the device.
    Carver c;
    c.take(qbytes);
    c.take(obytes * sizeof(int64_t));
    c.take(obytes * sizeof(float));
    void* ws_at = c.take(plan.ws_bytes);
    (void)ws_at;
    if (cudaMallocHost(&key.pinned, q_al + obytes * 12 + 16) != cudaSuccess ||
        cudaMalloc(&key.dev, c.used) != cudaSuccess) {
      cudaGetLastError();
      destroy_flat_graph(key);
      *captured = false;
      return PX_OK;
    }
    c = Carver{key.dev};
    float* d_q = static_cast<float*>(c.take(qbytes));
    int64_t* d_ids = static_cast<int64_t*>(c.take(obytes * sizeof(int64_t)));
    float* d_d = static_cast<float*>(c.take(obytes * sizeof(float)));
    void* d_ws = c.take(plan.ws_bytes);
    char* pin = static_cast<char*>(key.pinned);
    const int64_t launches0 = g_launches.load();
    cudaGraph_t graph = nullptr;
    cudaError_t ce = cudaStreamBeginCapture(sh.stream, cudaStreamCaptureModeThreadLocal);
    px_status ps = PX_OK;
    if (ce == cudaSuccess) {
      ce = cudaMemcpyAsync(d_q, pin, qbytes, cudaMemcpyHostToDevice, sh.stream);
      if (ce == cudaSuccess) ps = run_flat_search(h, sh, plan, metric, d_q, nq, k, nullptr, sh.stream, d_ws);
      if (ps == PX_OK && ce == cudaSuccess)
        ce = launch_emit(plan.final_cands, nq, k, metric == PX_METRIC_L2, natural, sh.segs.view(h->id_offset),
                         d_ids, d_d, sh.stream);
      if (ps == PX_OK && ce == cudaSuccess)
        ce = cudaMemcpyAsync(pin + q_al, d_ids, obytes * sizeof(int64_t), cudaMemcpyDeviceToHost, sh.stream);
      if (ps == PX_OK && ce == cudaSuccess)
        ce = cudaMemcpyAsync(pin + q_al + obytes * sizeof(int64_t), d_d, obytes * sizeof(float),
                             cudaMemcpyDeviceToHost, sh.stream);
      const cudaError_t ee = cudaStreamEndCapture(sh.stream, &graph);
      if (ce == cudaSuccess) ce = ee;
    }
    g_launches.fetch_sub(g_launches.load() - launches0);  // counted when replayed
    if (ps == PX_OK && ce == cudaSuccess) ce = cudaGraphInstantiate(&key.exec, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    if (ps != PX_OK || ce != cudaSuccess) {
      cudaGetLastError();
      destroy_flat_graph(key);
      *captured = false;
      return PX_OK;
    }
    if (h->graphs.size() >= kMaxFlatGraphs) {
      auto oldest = h->graphs.begin();
      for (auto it = h->graphs.begin(); it != h->graphs.end(); ++it)
        if (it->last_use < oldest->last_use) oldest = it;
      destroy_flat_graph(*oldest);
      h->graphs.erase(oldest);
    }
    h->graphs.push_back(key);
    hit = &h->graphs.back();
  }
  hit->last_use = ++h->graph_clock;
  char* pin = static_cast<char*>(hit->pinned);
  std::memcpy(pin, queries, qbytes);
  cudaError_t e = cudaGraphLaunch(hit->exec, sh.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(sh.stream);
  if (e != cudaSuccess) return cuda_status(e, "search");
  // The replayed kernels: the exact scan, its merge, and the emit.
  g_launches += 3;
  sh.last_path = static_cast<int>(FlatPath::Exact);
  sh.last_fallback = 0;
  sh.last_refined = 0;
  sh.last_pass = -1;
  sh.last_sample_tiles = 0;
  sh.last_launches = 3;
  sh.last_profiled = false;
  note_search_done(sh);
  std::memcpy(out_ids, pin + q_al, obytes * sizeof(int64_t));
  std::memcpy(out_dists, pin + q_al + obytes * sizeof(int64_t), obytes * sizeof(float));
  return PX_OK;
}

// Full host-to-host search over every shard.
static px_status flat_search_host(const px_flat* hc, int metric, const float* queries, int64_t nq,
                                  int32_t k, const uint8_t* mask, bool natural, int64_t* out_ids,
                                  float* out_dists) {
  px_flat* h = const_cast<px_flat*>(hc);
  std::lock_guard<std::mutex> lk(h->mu);
  const int G = static_cast<int>(h->shards.size());
  const size_t qbytes = sizeof(float) * static_cast<size_t>(nq) * h->dim;
  const size_t obytes = static_cast<size_t>(nq) * k;
  std::vector<uint8_t> local_mask;

  if (G == 1 && mask == nullptr && g_profiling.load() == 0) {
    FlatShard& sh = h->shards[0];
    DeviceGuard dg(sh.device);
    px_status s = sh.segs.sync_device();
    if (s != PX_OK) return s;
    SearchPlan plan;
    s = plan_flat_search(h, sh, nq, k, false, plan);
    if (s != PX_OK) return s;
    if (plan.path == FlatPath::Exact) {
      bool captured = false;
      s = flat_search_replay(h, sh, plan, metric, queries, nq, k, natural, out_ids, out_dists, &captured);
      if (s != PX_OK || captured) return s;
    }
  }

  // Host buffers that are not page-locked go through a pinned staging buffer
  // of the handle, so the copies are asynchronous DMA transfers.
  const bool stage_in = !is_pinned(queries);
  const bool stage_out = !is_pinned(out_ids) || !is_pinned(out_dists);
  const size_t pin_bytes = (stage_in ? qbytes : 0) + (stage_out ? obytes * 12 + 16 : 0);
  if (pin_bytes > 0) {
    px_status ps = h->pinned.reserve(pin_bytes);
    if (ps != PX_OK) return ps;
  }
  char* pin = static_cast<char*>(h->pinned.ptr);
  const float* q_src = queries;
  if (stage_in) {
    std::memcpy(pin, queries, qbytes);
    q_src = reinterpret_cast<const float*>(pin);
    pin += (qbytes + 15) & ~size_t(15);
  }
  int64_t* pin_ids = stage_out ? reinterpret_cast<int64_t*>(pin) : out_ids;
  float* pin_d = stage_out ? reinterpret_cast<float*>(pin + obytes * sizeof(int64_t)) : out_dists;

  // Per-shard: upload queries (+ mask), search, leave results on device.
  for (int g = 0; g < G; ++g) {
    FlatShard& sh = h->shards[g];
    DeviceGuard dg(sh.device);
    Carver c;
    c.take(qbytes);
    c.take(obytes * sizeof(int64_t));
    c.take(obytes * sizeof(float));
    if (mask) c.take(static_cast<size_t>(std::max<int64_t>(sh.n, 1)));
    cudaError_t e = sh.stage.reserve(c.used);
    if (e != cudaSuccess) return cuda_status(e, "query staging allocation");
    c = Carver{sh.stage.ptr};
    float* d_q = static_cast<float*>(c.take(qbytes));
    int64_t* d_ids = static_cast<int64_t*>(c.take(obytes * sizeof(int64_t)));
    float* d_d = static_cast<float*>(c.take(obytes * sizeof(float)));
    uint8_t* d_mask = nullptr;
    if (mask) {
      d_mask = static_cast<uint8_t*>(c.take(static_cast<size_t>(std::max<int64_t>(sh.n, 1))));
      sh.segs.local_mask(mask, sh.n, local_mask);
      if (sh.n > 0) {
        e = cudaMemcpyAsync(d_mask, local_mask.data(), static_cast<size_t>(sh.n), cudaMemcpyHostToDevice,
                            sh.stream);
        if (e != cudaSuccess) return cuda_status(e, "mask upload");
      }
    }
    e = cudaMemcpyAsync(d_q, q_src, qbytes, cudaMemcpyHostToDevice, sh.stream);
    if (e != cudaSuccess) return cuda_status(e, "query upload");
    px_status s = shard_search(h, sh, metric, d_q, nq, k, d_mask, natural && G == 1, d_ids, d_d,
                               sh.stream);
    if (s != PX_OK) return s;
    sh.out_ids = d_ids;
    sh.out_dists = d_d;
  }

  FlatShard& s0 = h->shards[0];
  DeviceGuard dg(s0.device);
  const int64_t* res_ids = s0.out_ids;
  const float* res_d = s0.out_dists;
  if (G > 1) {
    // Gather every shard's key-space lists on device 0 and merge them.
    px_status s = h->gather.ensure(s0.device, static_cast<size_t>(G) * obytes);
    if (s != PX_OK) return s;
    for (int g = 0; g < G; ++g) {
      FlatShard& sh = h->shards[g];
      DeviceGuard dgs(sh.device);  // copies and the event go on this shard's own stream
      cudaError_t e = cudaMemcpyPeerAsync(h->gather.ids + g * obytes, s0.device, sh.out_ids, sh.device,
                                          obytes * sizeof(int64_t), sh.stream);
      if (e == cudaSuccess)
        e = cudaMemcpyPeerAsync(h->gather.keys + g * obytes, s0.device, sh.out_dists, sh.device,
                                obytes * sizeof(float), sh.stream);
      if (e == cudaSuccess && g > 0) e = cudaEventRecord(sh.ev_done, sh.stream);
      if (e != cudaSuccess) return cuda_status(e, "shard gather");
    }
    for (int g = 1; g < G; ++g) {
      cudaError_t ew = cudaStreamWaitEvent(s0.stream, h->shards[g].ev_done, 0);
      if (ew != cudaSuccess) return cuda_status(ew, "shard gather wait");
    }
    cudaError_t e = launch_merge_shards(h->gather.keys, h->gather.ids, G, nq, k,
                                        metric == PX_METRIC_L2, natural, h->gather.out_dists,
                                        h->gather.out_ids, s0.stream);
    if (e != cudaSuccess) return cuda_status(e, "shard merge launch");
    res_ids = h->gather.out_ids;
    res_d = h->gather.out_dists;
  }
  cudaError_t e = cudaMemcpyAsync(pin_ids, res_ids, obytes * sizeof(int64_t), cudaMemcpyDeviceToHost,
                                  s0.stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(pin_d, res_d, obytes * sizeof(float), cudaMemcpyDeviceToHost, s0.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s0.stream);
  if (e != cudaSuccess) return cuda_status(e, "search");
  // (The tensor-core path reads its device status word itself.)
  if (stage_out) {
    std::memcpy(out_ids, pin_ids, obytes * sizeof(int64_t));
    std::memcpy(out_dists, pin_d, obytes * sizeof(float));
  }
  return PX_OK;
}

static px_status validate_search(const px_flat* h, const float* queries, int64_t nq, int32_t k,
                                 const int64_t* out_ids, const float* out_dists) {
  px_status s = flat_check(h);
  if (s != PX_OK) return s;
  if (k < 0) return set_error(PX_EINVAL, "k must be >= 0");
  if (nq < 0) return set_error(PX_EINVAL, "query count must be >= 0");
  if (k > PX_MAX_K)
    return set_error(PX_EUNSUPPORTED, "k=" + std::to_string(k) + " exceeds PX_MAX_K=" +
                                          std::to_string(PX_MAX_K));
  if (nq > 0 && k > 0 && (queries == nullptr || out_ids == nullptr || out_dists == nullptr))
    return set_error(PX_EINVAL, "null buffer");
  return PX_OK;
}

extern "C" {

PX_API px_status px_flat_search(const px_flat* h, const float* queries, int64_t nq, int32_t k,
                                int64_t* out_ids, float* out_dists) {
  px_status s = validate_search(h, queries, nq, k, out_ids, out_dists);
  if (s != PX_OK) return s;
  if (k == 0 || nq == 0) return PX_OK;
  if (!all_finite(queries, nq * h->dim))
    return set_error(PX_EINVAL, "query must not contain NaN or infinite values");
  return flat_search_host(h, h->metric, queries, nq, k, nullptr, true, out_ids, out_dists);
}

PX_API px_status px_flat_search_filtered(const px_flat* h, const float* queries, int64_t nq,
                                         int32_t k, const uint8_t* mask, int64_t* out_ids,
                                         float* out_dists) {
  px_status s = validate_search(h, queries, nq, k, out_ids, out_dists);
  if (s != PX_OK) return s;
  if (mask == nullptr && h->total > 0) return set_error(PX_EINVAL, "mask is null");
  if (k == 0 || nq == 0) return PX_OK;
  if (!all_finite(queries, nq * h->dim))
    return set_error(PX_EINVAL, "query must not contain NaN or infinite values");
  return flat_search_host(h, h->metric, queries, nq, k, mask, true, out_ids, out_dists);
}

PX_API px_status px_flat_search_device(const px_flat* hc, const float* d_queries, int64_t nq,
                                       int32_t k, int32_t key_space, int64_t* d_out_ids,
                                       float* d_out_dists, void* stream) {
  px_status s = validate_search(hc, d_queries, nq, k, d_out_ids, d_out_dists);
  if (s != PX_OK) return s;
  if (hc->shards.size() != 1)
    return set_error(PX_EUNSUPPORTED, "px_flat_search_device needs a single-device handle");
  if (k == 0 || nq == 0) return PX_OK;
  px_flat* h = const_cast<px_flat*>(hc);
  std::lock_guard<std::mutex> lk(h->mu);
  FlatShard& sh = h->shards[0];
  DeviceGuard dg(sh.device);
  // NULL is CUDA's default stream, as for every device entry point: torch's
  // default stream has a null handle, and a search put on any other stream
  // would not be ordered with the caller's collectives and merges.
  return shard_search(h, sh, h->metric, d_queries, nq, k, nullptr, key_space == 0, d_out_ids,
                      d_out_dists, static_cast<cudaStream_t>(stream));
}

PX_API px_status px_flat_debug_candidates(const px_flat* hc, const float* queries, int64_t nq, int32_t k,
                                          int32_t max_cands, int64_t* out_ids, float* out_keys,
                                          int32_t* out_cands, int32_t* out_pass) {
  px_status s = validate_search(hc, queries, nq, k, out_ids, out_keys);
  if (s != PX_OK) return s;
  if (hc->shards.size() != 1)
    return set_error(PX_EUNSUPPORTED, "px_flat_debug_candidates needs a single-device handle");
  if (max_cands < 1 || out_cands == nullptr || out_pass == nullptr)
    return set_error(PX_EINVAL, "max_cands must be >= 1 and out_cands / out_pass non-null");
  if (k < 1 || nq < 1) return set_error(PX_EINVAL, "k and the query count must be >= 1");
  if (!all_finite(queries, nq * hc->dim))
    return set_error(PX_EINVAL, "query must not contain NaN or infinite values");
  px_flat* h = const_cast<px_flat*>(hc);
  std::lock_guard<std::mutex> lk(h->mu);
  FlatShard& sh = h->shards[0];
  DeviceGuard dg(sh.device);
  const size_t qbytes = sizeof(float) * static_cast<size_t>(nq) * h->dim;
  cudaError_t e = sh.stage.reserve(qbytes);
  if (e != cudaSuccess) return cuda_status(e, "query staging allocation");
  e = cudaMemcpyAsync(sh.stage.ptr, queries, qbytes, cudaMemcpyHostToDevice, sh.stream);
  if (e != cudaSuccess) return cuda_status(e, "query upload");
  const uint64_t* d_merged = nullptr;
  int cands = 0, pass = 0;
  s = first_pass_candidates(h, sh, h->metric, static_cast<const float*>(sh.stage.ptr), nq, k, sh.stream,
                            &d_merged, &cands, &pass);
  if (s != PX_OK) return s;
  std::vector<uint64_t> merged(static_cast<size_t>(nq) * cands);
  e = cudaMemcpyAsync(merged.data(), d_merged, merged.size() * sizeof(uint64_t), cudaMemcpyDeviceToHost,
                      sh.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(sh.stream);
  if (e != cudaSuccess) return cuda_status(e, "candidate readback");
  const int m = std::min(cands, max_cands);
  for (int64_t q = 0; q < nq; ++q) {
    for (int j = 0; j < max_cands; ++j) {
      const size_t o = static_cast<size_t>(q) * max_cands + j;
      const uint64_t c = j < m ? merged[static_cast<size_t>(q) * cands + j] : PX_EMPTY;
      if (c == PX_EMPTY) {
        out_ids[o] = -1;
        out_keys[o] = 3.40282347e+38f;
        continue;
      }
      // Shard row -> global id through the segment table.
      const int64_t row = cand_row(c);
      size_t seg = 0;
      while (seg + 1 < sh.segs.local.size() && sh.segs.local[seg + 1] <= row) ++seg;
      out_ids[o] = sh.segs.global[seg] + (row - sh.segs.local[seg]) + h->id_offset;
      out_keys[o] = cand_key(c);
    }
  }
  *out_cands = m;
  *out_pass = pass;
  return PX_OK;
}

PX_API px_status px_merge_shards_device(int32_t device, const float* d_keys, const int64_t* d_ids,
                                        int32_t nshard, int64_t nq, int32_t k, int32_t metric,
                                        int32_t natural, float* d_out_dists, int64_t* d_out_ids,
                                        void* stream) {
  if (nshard < 1 || nshard > 8) return set_error(PX_EINVAL, "nshard must be in 1..=8");
  if (k < 0 || nq < 0) return set_error(PX_EINVAL, "negative size");
  if (metric != PX_METRIC_L2 && metric != PX_METRIC_IP) return set_error(PX_EINVAL, "bad metric");
  DeviceGuard dg(device);
  cudaError_t e = launch_merge_shards(d_keys, d_ids, nshard, nq, k, metric == PX_METRIC_L2,
                                      natural != 0, d_out_dists, d_out_ids,
                                      static_cast<cudaStream_t>(stream));
  return cuda_status(e, "merge_shards launch");
}

PX_API int64_t px_shard_record_bytes(int64_t nq, int32_t k) {
  if (nq < 0 || k < 0) return 0;
  return (nq * k * 12 + 15) / 16 * 16;
}

PX_API px_status px_merge_shard_records_device(int32_t device, const void* d_records, int32_t nshard, int64_t nq,
                                               int32_t k, int32_t metric, int32_t natural, float* d_out_dists,
                                               int64_t* d_out_ids, void* stream) {
  if (nshard < 1 || nshard > 8) return set_error(PX_EINVAL, "nshard must be in 1..=8");
  if (k < 0 || nq < 0) return set_error(PX_EINVAL, "negative size");
  if (metric != PX_METRIC_L2 && metric != PX_METRIC_IP) return set_error(PX_EINVAL, "bad metric");
  if (nq == 0 || k == 0) return PX_OK;
  if (d_records == nullptr || d_out_dists == nullptr || d_out_ids == nullptr)
    return set_error(PX_EINVAL, "null buffer");
  if (reinterpret_cast<uintptr_t>(d_records) % 16 != 0)
    return set_error(PX_EINVAL, "records must be 16-byte aligned");
  const int64_t rec = px_shard_record_bytes(nq, k);
  const char* base = static_cast<const char*>(d_records);
  DeviceGuard dg(device);
  cudaError_t e = launch_merge_shards_strided(reinterpret_cast<const float*>(base + 8 * nq * k), rec,
                                              reinterpret_cast<const int64_t*>(base), rec, nshard, nq, k,
                                              metric == PX_METRIC_L2, natural != 0, d_out_dists, d_out_ids,
                                              static_cast<cudaStream_t>(stream));
  return cuda_status(e, "merge_shards launch");
}

// ---- reference-compatible ABI (knn.cu:123-180) ----------------------------

struct PxGpuIndex {
  px_flat* flat;
};

PX_API PxGpuIndex* knn_gpu_create(const float* base, int n, int dim) {
  if (n < 0 || dim <= 0 || (n > 0 && base == nullptr)) return nullptr;
  px_flat* f = nullptr;
  if (px_flat_create(dim, PX_METRIC_L2, nullptr, 0, &f) != PX_OK) return nullptr;
  if (n > 0) {
    // The reference copies the base without checking values (knn.cu:130-141).
    std::lock_guard<std::mutex> lk(f->mu);
    FlatShard& sh = f->shards[0];
    DeviceGuard dg(sh.device);
    const size_t bytes = sizeof(float) * static_cast<size_t>(n) * dim;
    if (sh.stage.reserve(bytes) != cudaSuccess ||
        cudaMemcpyAsync(sh.stage.ptr, base, bytes, cudaMemcpyHostToDevice, sh.stream) != cudaSuccess ||
        sh.append_device(static_cast<const float*>(sh.stage.ptr), n, dim, f->ld, f->ldb, 0) != PX_OK) {
      px_flat_destroy(f);
      return nullptr;
    }
    f->total = n;
  }
  return new PxGpuIndex{f};
}

PX_API int knn_gpu_search(const PxGpuIndex* idx, const float* queries, int nq, int k, int metric,
                          long long* out_ids, float* out_keys) {
  if (k < 1 || k > PX_MAX_K) return -1;
  if (idx == nullptr || nq < 0) return static_cast<int>(cudaErrorInvalidValue);
  if (nq == 0) return 0;
  if (metric != PX_METRIC_L2 && metric != PX_METRIC_IP) return static_cast<int>(cudaErrorInvalidValue);
  px_status s = flat_search_host(idx->flat, metric, queries, nq, k, nullptr, false,
                                 reinterpret_cast<int64_t*>(out_ids), out_keys);
  if (s == PX_OK) return 0;
  cudaError_t last = cudaGetLastError();
  return static_cast<int>(last != cudaSuccess ? last : cudaErrorUnknown);
}

PX_API void knn_gpu_free(PxGpuIndex* idx) {
  if (!idx) return;
  px_flat_destroy(idx->flat);
  delete idx;
}

}  // extern "C"
