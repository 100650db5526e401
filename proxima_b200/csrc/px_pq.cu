// PqIndex on the GPU: training, encoding and the ADC scan (C ABI in px.h).
//
// Training restates ProductQuantizer::train and kmeans
// (crates/core/src/pq.rs:54-105, 139-193). The m per-subspace k-means runs
// advance in lockstep: one nearest-centroid launch per iteration assigns all
// subspaces at once on the device (bit-exact: same l2_sqr order, strict '<'),
// and the host then applies the reference's sequential mean update and
// empty-cluster reseeding with each subspace's own SplitMix stream
// (pq.rs:169-190). The result is bit-identical to the reference's codebooks.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/px.h"
#include "px_common.cuh"
#include "px_kernels.h"
#include "px_runtime.h"

using namespace px;

namespace {

struct SplitMix {  // pq.rs:25-37
  uint64_t s;
  uint64_t next_u64() {
    s += 0x9E3779B97F4A7C15ull;
    uint64_t z = s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  uint64_t below(uint64_t n) { return next_u64() % n; }
};

}  // namespace

struct PqShard {
  int device = 0;
  int sms = 148;
  cudaStream_t stream = nullptr;
  uint8_t* codes = nullptr;
  int64_t n = 0, cap = 0;
  float* books = nullptr;
  px::Segments segs;
  px::DevBuf ws;
  px::DevBuf stage;
  int64_t* out_ids = nullptr;
  float* out_dists = nullptr;
  cudaEvent_t ev_start = nullptr, ev_stop = nullptr;  // bracket the scan kernel when profiling
  cudaEvent_t ev_done = nullptr;  // results copied to the gather buffer (own device)
  bool last_profiled = false;
  int last_launches = 0;

  void release() {
    px::DeviceGuard g(device);
    if (stream) cudaStreamSynchronize(stream);
    if (ev_start) cudaEventDestroy(ev_start);
    if (ev_stop) cudaEventDestroy(ev_stop);
    if (ev_done) cudaEventDestroy(ev_done);
    ev_start = ev_stop = ev_done = nullptr;
    if (codes) cudaFree(codes);
    if (books) cudaFree(books);
    codes = nullptr;
    books = nullptr;
    ws.release();
    stage.release();
    segs.dev.release();
    if (stream) cudaStreamDestroy(stream);
    stream = nullptr;
  }

  px_status ensure_capacity(int64_t need, int m) {
    if (need <= cap) return PX_OK;
    const int64_t new_cap = std::max<int64_t>(need, cap + cap / 2);
    uint8_t* nc = nullptr;
    // 16 bytes of slack so the scan's 128-bit code loads stay in bounds.
    cudaError_t e = cudaMalloc(&nc, static_cast<size_t>(new_cap) * m + 16);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_error(PX_ENOMEM, std::string("code allocation failed: ") + cudaGetErrorString(e));
    }
    if (n > 0) {
      cudaMemcpyAsync(nc, codes, static_cast<size_t>(n) * m, cudaMemcpyDeviceToDevice, stream);
      cudaStreamSynchronize(stream);
    }
    if (codes) cudaFree(codes);
    codes = nc;
    cap = new_cap;
    return PX_OK;
  }
};

struct px_pq {
  int dim = 0, m = 0, nbits = 0, ksub = 0, dsub = 0, metric = 0;
  int64_t total = 0;
  std::vector<float> books;  // host copy, m * ksub * dsub
  std::vector<PqShard> shards;
  GatherBuf gather;
  std::mutex mu;
};

static px_status pq_check(const px_pq* h) {
  if (h == nullptr) return set_error(PX_EINVAL, "null handle");
  return PX_OK;
}

static px_status validate_pq_shape(int32_t dim, int32_t m, int32_t nbits) {
  if (m <= 0) return set_error(PX_EINVAL, "m must be >= 1");
  if (dim <= 0 || dim % m != 0) return set_error(PX_EINVAL, "dim must be > 0 and divisible by m");
  if (nbits < 1 || nbits > 8) return set_error(PX_EINVAL, "nbits must be in 1..=8");
  return PX_OK;
}

// Encodes n host vectors on shard `sh` into codes appended at sh.n (append)
// or into a host buffer (out != nullptr).
static px_status pq_encode_on(const px_pq* h, PqShard& sh, const float* vectors, int64_t n,
                              uint8_t* host_out, bool append, int64_t global_begin) {
  px::DeviceGuard dg(sh.device);
  const size_t vbytes = sizeof(float) * static_cast<size_t>(n) * h->dim;
  const size_t cbytes = static_cast<size_t>(n) * h->m;
  px::Carver c;
  c.take(vbytes);
  c.take(cbytes);
  cudaError_t e = sh.stage.reserve(c.used);
  if (e != cudaSuccess) return cuda_status(e, "encode staging allocation");
  c = px::Carver(sh.stage.ptr);
  float* d_v = static_cast<float*>(c.take(vbytes));
  uint8_t* d_c = static_cast<uint8_t*>(c.take(cbytes));
  if (append) {
    px_status s = sh.ensure_capacity(sh.n + n, h->m);
    if (s != PX_OK) return s;
    d_c = sh.codes + sh.n * h->m;
  }
  e = cudaMemcpyAsync(d_v, vectors, vbytes, cudaMemcpyHostToDevice, sh.stream);
  if (e == cudaSuccess)
    e = launch_nearest_centroid(d_v, n, h->m, h->dsub, h->ksub, sh.books, nullptr, d_c, sh.stream);
  if (e == cudaSuccess && host_out)
    e = cudaMemcpyAsync(host_out, d_c, cbytes, cudaMemcpyDeviceToHost, sh.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(sh.stream);
  if (e != cudaSuccess) return cuda_status(e, "encode");
  if (append) {
    sh.segs.local.push_back(sh.n);
    sh.segs.global.push_back(global_begin);
    sh.segs.dirty = true;
    sh.n += n;
  }
  return PX_OK;
}

static px_status pq_shard_search(const px_pq* h, PqShard& sh, const float* d_q, int64_t nq, int k,
                                 const uint8_t* d_mask, bool natural, int64_t* d_ids, float* d_dists,
                                 cudaStream_t stream) {
  const bool l2 = h->metric == PX_METRIC_L2;
  px_status s = sh.segs.sync_device();
  if (s != PX_OK) return s;
  const int group = pq_group_for(h->m, h->ksub, nq, k);
  const int64_t groups = (nq + group - 1) / group;
  if (groups > 65535) return set_error(PX_EUNSUPPORTED, "too many queries in one call");
  const size_t smem = pq_smem_for(group, h->m, h->ksub, k);
  if (smem > 227 * 1024) return set_error(PX_EUNSUPPORTED, "PQ table too large for shared memory");
  const int per_sm = std::max<int>(1, static_cast<int>((227 * 1024) / smem));
  const int64_t slots = static_cast<int64_t>(sh.sms) * std::min(per_sm, 4);  // co-resident CTAs
  const int64_t n = std::max<int64_t>(sh.n, 1);
  // Row slices per query group: at least two waves of CTAs, and a total that
  // fills its last wave (a 2.5-wave grid leaves half the GPU idle at the end).
  const int64_t max_cta = std::max<int64_t>(1, std::min<int64_t>((n + 511) / 512, 1024));
  const int64_t lo = std::min<int64_t>(max_cta, std::max<int64_t>(1, (2 * slots + groups - 1) / groups));
  int64_t ncta = lo;
  double best = 0.0;
  for (int64_t cand = lo; cand <= std::min<int64_t>(max_cta, 4 * lo); ++cand) {
    const int64_t total = groups * cand;
    const double fill = static_cast<double>(total) / (static_cast<double>((total + slots - 1) / slots) * slots);
    if (fill > best + 1e-9) {
      best = fill;
      ncta = cand;
    }
    if (fill >= 0.97) break;
  }
  const int64_t rpi = pq_rows_per_iter(group, h->m, h->ksub, k);
  int64_t rows = (n + ncta - 1) / ncta;
  rows = (rows + rpi - 1) / rpi * rpi;
  ncta = (n + rows - 1) / rows;

  px::Carver c;
  c.take(sizeof(float) * static_cast<size_t>(nq) * h->m * h->ksub);
  c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * ncta * k);
  c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * k);
  cudaError_t e = sh.ws.reserve(c.used);
  if (e != cudaSuccess) return cuda_status(e, "PQ workspace allocation");
  c = px::Carver(sh.ws.ptr);
  float* lut = static_cast<float*>(c.take(sizeof(float) * static_cast<size_t>(nq) * h->m * h->ksub));
  uint64_t* partial = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * ncta * k));
  uint64_t* cands = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * k));

  e = launch_pq_lut(sh.books, h->m, h->ksub, h->dsub, l2, d_q, static_cast<int>(nq), lut, stream);
  if (e != cudaSuccess) return cuda_status(e, "PQ table launch");
  PqScanArgs a;
  a.codes = sh.codes;
  a.n = sh.n;
  a.m = h->m;
  a.ksub = h->ksub;
  a.lut = lut;
  a.nq = static_cast<int>(nq);
  a.k = k;
  a.group = group;
  a.ncta = static_cast<int>(ncta);
  a.rows_per_cta = rows;
  a.mask = d_mask;
  a.partial = partial;
  const bool prof = px::g_profiling.load() != 0;
  sh.last_profiled = prof;
  if (prof) cudaEventRecord(sh.ev_start, stream);
  e = launch_pq_scan(a, stream);
  if (prof) cudaEventRecord(sh.ev_stop, stream);
  if (e != cudaSuccess) return cuda_status(e, "PQ scan launch");
  px::g_launches += 4;  // table, scan, merge, emit
  sh.last_launches = 4;
  e = launch_merge_lists(partial, nq, static_cast<int>(ncta), k, k, cands, stream);
  if (e != cudaSuccess) return cuda_status(e, "merge launch");
  e = launch_emit(cands, nq, k, l2, natural, sh.segs.view(0), d_ids, d_dists, stream);
  if (e != cudaSuccess) return cuda_status(e, "emit launch");
  return PX_OK;
}

static px_status pq_search_host(const px_pq* hc, const float* queries, int64_t nq, int32_t k,
                                const uint8_t* mask, int64_t* out_ids, float* out_dists) {
  px_pq* h = const_cast<px_pq*>(hc);
  std::lock_guard<std::mutex> lk(h->mu);
  const int G = static_cast<int>(h->shards.size());
  const size_t qbytes = sizeof(float) * static_cast<size_t>(nq) * h->dim;
  const size_t obytes = static_cast<size_t>(nq) * k;
  std::vector<uint8_t> local_mask;
  for (int g = 0; g < G; ++g) {
    PqShard& sh = h->shards[g];
    px::DeviceGuard dg(sh.device);
    px::Carver c;
    c.take(qbytes);
    c.take(obytes * sizeof(int64_t));
    c.take(obytes * sizeof(float));
    if (mask) c.take(static_cast<size_t>(std::max<int64_t>(sh.n, 1)));
    cudaError_t e = sh.stage.reserve(c.used);
    if (e != cudaSuccess) return cuda_status(e, "query staging allocation");
    c = px::Carver(sh.stage.ptr);
    float* d_q = static_cast<float*>(c.take(qbytes));
    int64_t* d_ids = static_cast<int64_t*>(c.take(obytes * sizeof(int64_t)));
    float* d_d = static_cast<float*>(c.take(obytes * sizeof(float)));
    uint8_t* d_mask = nullptr;
    if (mask) {
      d_mask = static_cast<uint8_t*>(c.take(static_cast<size_t>(std::max<int64_t>(sh.n, 1))));
      sh.segs.local_mask(mask, sh.n, local_mask);
      if (sh.n > 0) {
        e = cudaMemcpyAsync(d_mask, local_mask.data(), static_cast<size_t>(sh.n),
                            cudaMemcpyHostToDevice, sh.stream);
        if (e != cudaSuccess) return cuda_status(e, "mask upload");
      }
    }
    e = cudaMemcpyAsync(d_q, queries, qbytes, cudaMemcpyHostToDevice, sh.stream);
    if (e != cudaSuccess) return cuda_status(e, "query upload");
    px_status s = pq_shard_search(h, sh, d_q, nq, k, d_mask, G == 1, d_ids, d_d, sh.stream);
    if (s != PX_OK) return s;
    sh.out_ids = d_ids;
    sh.out_dists = d_d;
  }
  PqShard& s0 = h->shards[0];
  px::DeviceGuard dg(s0.device);
  const int64_t* res_ids = s0.out_ids;
  const float* res_d = s0.out_dists;
  if (G > 1) {
    px_status s = h->gather.ensure(s0.device, static_cast<size_t>(G) * obytes);
    if (s != PX_OK) return s;
    for (int g = 0; g < G; ++g) {
      PqShard& sh = h->shards[g];
      px::DeviceGuard dgs(sh.device);  // copies and the event go on this shard's own stream
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
                                        h->metric == PX_METRIC_L2, true, h->gather.out_dists,
                                        h->gather.out_ids, s0.stream);
    if (e != cudaSuccess) return cuda_status(e, "shard merge launch");
    res_ids = h->gather.out_ids;
    res_d = h->gather.out_dists;
  }
  cudaError_t e = cudaMemcpyAsync(out_ids, res_ids, obytes * sizeof(int64_t), cudaMemcpyDeviceToHost,
                                  s0.stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(out_dists, res_d, obytes * sizeof(float), cudaMemcpyDeviceToHost, s0.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s0.stream);
  if (e != cudaSuccess) return cuda_status(e, "PQ search");
  return PX_OK;
}

extern "C" {

PX_API px_status px_pq_train(const float* training, int64_t n_all, int32_t dim, int32_t m,
                             int32_t nbits, int32_t train_iters, int64_t train_sample,
                             uint64_t seed, int32_t device, float* out_codebooks) {
  px_status s = validate_pq_shape(dim, m, nbits);
  if (s != PX_OK) return s;
  if (training == nullptr || out_codebooks == nullptr) return set_error(PX_EINVAL, "null buffer");
  if (train_iters < 0 || train_sample < 0) return set_error(PX_EINVAL, "negative training parameter");
  const int64_t ksub = int64_t(1) << nbits;
  const int dsub = dim / m;
  if (n_all < ksub)
    return set_error(PX_EINVAL, "need at least k=" + std::to_string(ksub) + " training vectors, got " +
                                    std::to_string(n_all));
  if (!all_finite(training, n_all * dim))
    return set_error(PX_EINVAL, "training data must not contain NaN or infinite values");
  std::vector<int> devs;
  const int32_t dev_arr[1] = {device};
  s = resolve_devices(device >= 0 ? dev_arr : nullptr, device >= 0 ? 1 : 0, devs);
  if (s != PX_OK) return s;

  // Sample selection (pq.rs:73-83).
  SplitMix rng{seed};
  int64_t n = n_all;
  if (train_sample > 0) n = std::min<int64_t>(std::max<int64_t>(train_sample, ksub), n_all);
  std::vector<int64_t> sample(static_cast<size_t>(n));
  if (n == n_all) {
    for (int64_t i = 0; i < n; ++i) sample[i] = i;
  } else {
    for (int64_t i = 0; i < n; ++i) sample[i] = static_cast<int64_t>(rng.below(static_cast<uint64_t>(n_all)));
  }
  std::vector<float> data(static_cast<size_t>(n) * dim);
  for (int64_t i = 0; i < n; ++i)
    std::memcpy(&data[i * dim], &training[sample[i] * dim], sizeof(float) * dim);

  // kmeans seeding per subspace (pq.rs:140-148).
  std::vector<SplitMix> rngs(m);
  std::vector<float> books(static_cast<size_t>(m) * ksub * dsub, 0.f);
  std::vector<int64_t> order(static_cast<size_t>(n));
  for (int sub = 0; sub < m; ++sub) {
    rngs[sub].s = seed ^ (static_cast<uint64_t>(sub) * 0x9E3779B97F4A7C15ull);
    for (int64_t i = 0; i < n; ++i) order[i] = i;
    for (int64_t c = 0; c < ksub; ++c) {
      int64_t j = c + static_cast<int64_t>(rngs[sub].below(static_cast<uint64_t>(n - c)));
      std::swap(order[c], order[j]);
      std::memcpy(&books[(sub * ksub + c) * dsub], &data[order[c] * dim + sub * dsub],
                  sizeof(float) * dsub);
    }
  }

  px::DeviceGuard dg(devs[0]);
  cudaStream_t st = nullptr;
  float* d_data = nullptr;
  float* d_books = nullptr;
  uint32_t* d_assign = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&d_data, sizeof(float) * data.size());
  if (e == cudaSuccess) e = cudaMalloc(&d_books, sizeof(float) * books.size());
  if (e == cudaSuccess) e = cudaMalloc(&d_assign, sizeof(uint32_t) * static_cast<size_t>(n) * m);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(d_data, data.data(), sizeof(float) * data.size(), cudaMemcpyHostToDevice, st);
  std::vector<uint32_t> assign(static_cast<size_t>(n) * m);
  std::vector<float> sums(static_cast<size_t>(ksub) * dsub);
  std::vector<uint32_t> counts(static_cast<size_t>(ksub));
  for (int it = 0; it < train_iters && e == cudaSuccess; ++it) {
    e = cudaMemcpyAsync(d_books, books.data(), sizeof(float) * books.size(), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = launch_nearest_centroid(d_data, n, m, dsub, static_cast<int>(ksub), d_books,
                                                      d_assign, nullptr, st);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(assign.data(), d_assign, sizeof(uint32_t) * assign.size(),
                          cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) break;
    // Sequential update (pq.rs:169-190), one subspace at a time.
    for (int sub = 0; sub < m; ++sub) {
      std::fill(sums.begin(), sums.end(), 0.f);
      std::fill(counts.begin(), counts.end(), 0u);
      for (int64_t i = 0; i < n; ++i) {
        const uint32_t c = assign[i * m + sub];
        counts[c] += 1;
        const float* v = &data[i * dim + sub * dsub];
        float* sm = &sums[static_cast<size_t>(c) * dsub];
        for (int j = 0; j < dsub; ++j) sm[j] = sm[j] + v[j];
      }
      float* book = &books[static_cast<size_t>(sub) * ksub * dsub];
      for (int64_t c = 0; c < ksub; ++c) {
        if (counts[c] == 0) {
          const int64_t idx = static_cast<int64_t>(rngs[sub].below(static_cast<uint64_t>(n)));
          std::memcpy(&book[c * dsub], &data[idx * dim + sub * dsub], sizeof(float) * dsub);
        } else {
          const float inv = 1.0f / static_cast<float>(counts[c]);
          for (int j = 0; j < dsub; ++j) book[c * dsub + j] = sums[c * dsub + j] * inv;
        }
      }
    }
  }
  if (d_data) cudaFree(d_data);
  if (d_books) cudaFree(d_books);
  if (d_assign) cudaFree(d_assign);
  if (st) cudaStreamDestroy(st);
  if (e != cudaSuccess) return cuda_status(e, "PQ training");
  std::memcpy(out_codebooks, books.data(), sizeof(float) * books.size());
  return PX_OK;
}

PX_API px_status px_pq_create(int32_t dim, int32_t m, int32_t nbits, int32_t metric,
                              const float* codebooks, const int32_t* devices, int32_t ndev,
                              px_pq** out) {
  if (out == nullptr) return set_error(PX_EINVAL, "out is null");
  *out = nullptr;
  px_status s = validate_pq_shape(dim, m, nbits);
  if (s != PX_OK) return s;
  if (metric != PX_METRIC_L2 && metric != PX_METRIC_IP)
    return set_error(PX_EINVAL, "metric must be 0 (L2) or 1 (inner product)");
  if (codebooks == nullptr) return set_error(PX_EINVAL, "codebooks is null");
  std::vector<int> devs;
  s = resolve_devices(devices, ndev, devs);
  if (s != PX_OK) return s;
  px_pq* h = new px_pq();
  h->dim = dim;
  h->m = m;
  h->nbits = nbits;
  h->ksub = 1 << nbits;
  h->dsub = dim / m;
  h->metric = metric;
  h->books.assign(codebooks, codebooks + static_cast<size_t>(m) * h->ksub * h->dsub);
  h->shards.resize(devs.size());
  for (size_t i = 0; i < devs.size(); ++i) {
    PqShard& sh = h->shards[i];
    sh.device = devs[i];
    sh.sms = device_sm_count(sh.device);
    px::DeviceGuard g(sh.device);
    const size_t bb = sizeof(float) * h->books.size();
    cudaError_t e = cudaStreamCreateWithFlags(&sh.stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&sh.books, bb);
    if (e == cudaSuccess) e = cudaEventCreate(&sh.ev_start);
    if (e == cudaSuccess) e = cudaEventCreate(&sh.ev_stop);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sh.ev_done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMemcpy(sh.books, h->books.data(), bb, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      px_status st = cuda_status(e, "PQ create");
      for (auto& x : h->shards) x.release();
      delete h;
      return st;
    }
  }
  *out = h;
  return PX_OK;
}

PX_API px_status px_pq_destroy(px_pq* h) {
  if (h == nullptr) return PX_OK;
  {
    std::lock_guard<std::mutex> lk(h->mu);
    for (auto& sh : h->shards) sh.release();
    h->gather.release_all();
  }
  delete h;
  return PX_OK;
}

PX_API int64_t px_pq_size(const px_pq* h) { return h ? h->total : 0; }

PX_API px_status px_pq_read_codes(const px_pq* hc, int64_t start, int64_t count, uint8_t* out) {
  px_status s = pq_check(hc);
  if (s != PX_OK) return s;
  if (start < 0 || count < 0 || start + count > hc->total)
    return set_error(PX_EINVAL, "row range out of bounds");
  if (count == 0) return PX_OK;
  if (out == nullptr) return set_error(PX_EINVAL, "out is null");
  px_pq* h = const_cast<px_pq*>(hc);
  std::lock_guard<std::mutex> lk(h->mu);
  for (auto& sh : h->shards) {
    px::DeviceGuard dg(sh.device);
    s = sh.segs.for_range(sh.n, start, start + count, [&](int64_t local, int64_t global, int64_t rows) {
      cudaError_t e = cudaMemcpy(out + (global - start) * h->m, sh.codes + local * h->m,
                                 static_cast<size_t>(rows) * h->m, cudaMemcpyDeviceToHost);
      return cuda_status(e, "code readback");
    });
    if (s != PX_OK) return s;
  }
  return PX_OK;
}

PX_API px_status px_pq_last_profile(const px_pq* h, px_search_profile* out) {
  px_status s = pq_check(h);
  if (s != PX_OK) return s;
  if (out == nullptr) return set_error(PX_EINVAL, "out is null");
  const PqShard& sh = h->shards[0];
  out->path = 2;
  out->launches = sh.last_launches;
  out->fallback_queries = 0;
  out->refined_queries = 0;
  out->first_pass = -1;
  out->sample_tiles = 0;
  out->profiled = 0;
  out->main_kernel_ms = 0.f;
  if (sh.last_profiled) {
    px::DeviceGuard dg(sh.device);
    float ms = 0.f;
    cudaError_t e = cudaEventSynchronize(sh.ev_stop);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, sh.ev_start, sh.ev_stop);
    if (e != cudaSuccess) return cuda_status(e, "profile events");
    out->profiled = 1;
    out->main_kernel_ms = ms;
  }
  return PX_OK;
}

PX_API px_status px_pq_add(px_pq* h, const float* vectors, int64_t n) {
  px_status s = pq_check(h);
  if (s != PX_OK) return s;
  if (n < 0) return set_error(PX_EINVAL, "row count must be >= 0");
  if (n == 0) return PX_OK;
  if (vectors == nullptr) return set_error(PX_EINVAL, "vectors is null");
  if (!all_finite(vectors, n * h->dim))
    return set_error(PX_EINVAL, "vectors must not contain NaN or infinite values");
  std::lock_guard<std::mutex> lk(h->mu);
  const int G = static_cast<int>(h->shards.size());
  std::vector<int64_t> begin, count;
  split_rows(n, G, begin, count);
  for (int g = 0; g < G; ++g) {
    if (count[g] == 0) continue;
    if (h->shards[g].n + count[g] > 0xFFFFFFFFll)
      return set_error(PX_EUNSUPPORTED, "a shard holds at most 2^32-1 rows");
    s = pq_encode_on(h, h->shards[g], vectors + begin[g] * h->dim, count[g], nullptr, true,
                     h->total + begin[g]);
    if (s != PX_OK) return s;
  }
  h->total += n;
  return PX_OK;
}

PX_API px_status px_pq_add_codes(px_pq* h, const uint8_t* codes, int64_t n) {
  px_status s = pq_check(h);
  if (s != PX_OK) return s;
  if (n < 0) return set_error(PX_EINVAL, "row count must be >= 0");
  if (n == 0) return PX_OK;
  if (codes == nullptr) return set_error(PX_EINVAL, "codes is null");
  for (int64_t i = 0; i < n * h->m; ++i)
    if (codes[i] >= h->ksub) return set_error(PX_EINVAL, "code value out of range for nbits");
  std::lock_guard<std::mutex> lk(h->mu);
  const int G = static_cast<int>(h->shards.size());
  std::vector<int64_t> begin, count;
  split_rows(n, G, begin, count);
  for (int g = 0; g < G; ++g) {
    if (count[g] == 0) continue;
    PqShard& sh = h->shards[g];
    if (sh.n + count[g] > 0xFFFFFFFFll)
      return set_error(PX_EUNSUPPORTED, "a shard holds at most 2^32-1 rows");
    px::DeviceGuard dg(sh.device);
    s = sh.ensure_capacity(sh.n + count[g], h->m);
    if (s != PX_OK) return s;
    cudaError_t e = cudaMemcpy(sh.codes + sh.n * h->m, codes + begin[g] * h->m,
                               static_cast<size_t>(count[g]) * h->m, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_status(e, "code upload");
    sh.segs.local.push_back(sh.n);
    sh.segs.global.push_back(h->total + begin[g]);
    sh.segs.dirty = true;
    sh.n += count[g];
  }
  h->total += n;
  return PX_OK;
}

PX_API px_status px_pq_encode(const px_pq* hc, const float* vectors, int64_t n, uint8_t* out_codes) {
  px_status s = pq_check(hc);
  if (s != PX_OK) return s;
  if (n < 0) return set_error(PX_EINVAL, "row count must be >= 0");
  if (n == 0) return PX_OK;
  if (vectors == nullptr || out_codes == nullptr) return set_error(PX_EINVAL, "null buffer");
  if (!all_finite(vectors, n * hc->dim))
    return set_error(PX_EINVAL, "vectors must not contain NaN or infinite values");
  px_pq* h = const_cast<px_pq*>(hc);
  std::lock_guard<std::mutex> lk(h->mu);
  return pq_encode_on(h, h->shards[0], vectors, n, out_codes, false, 0);
}

PX_API px_status px_pq_search(const px_pq* h, const float* queries, int64_t nq, int32_t k,
                              int64_t* out_ids, float* out_dists) {
  px_status s = pq_check(h);
  if (s != PX_OK) return s;
  if (k < 0 || nq < 0) return set_error(PX_EINVAL, "k and nq must be >= 0");
  if (k > PX_MAX_K)
    return set_error(PX_EUNSUPPORTED, "k=" + std::to_string(k) + " exceeds PX_MAX_K=" + std::to_string(PX_MAX_K));
  if (k == 0 || nq == 0) return PX_OK;
  if (queries == nullptr || out_ids == nullptr || out_dists == nullptr)
    return set_error(PX_EINVAL, "null buffer");
  if (!all_finite(queries, nq * h->dim))
    return set_error(PX_EINVAL, "query must not contain NaN or infinite values");
  return pq_search_host(h, queries, nq, k, nullptr, out_ids, out_dists);
}

PX_API px_status px_pq_search_device(const px_pq* hc, const float* d_queries, int64_t nq, int32_t k,
                                     int32_t key_space, int64_t* d_out_ids, float* d_out_dists, void* stream) {
  px_status s = pq_check(hc);
  if (s != PX_OK) return s;
  if (k < 0 || nq < 0) return set_error(PX_EINVAL, "k and nq must be >= 0");
  if (k > PX_MAX_K)
    return set_error(PX_EUNSUPPORTED, "k=" + std::to_string(k) + " exceeds PX_MAX_K=" + std::to_string(PX_MAX_K));
  if (hc->shards.size() != 1)
    return set_error(PX_EUNSUPPORTED, "px_pq_search_device needs a single-device handle");
  if (k == 0 || nq == 0) return PX_OK;
  if (d_queries == nullptr || d_out_ids == nullptr || d_out_dists == nullptr)
    return set_error(PX_EINVAL, "null buffer");
  px_pq* h = const_cast<px_pq*>(hc);
  std::lock_guard<std::mutex> lk(h->mu);
  PqShard& sh = h->shards[0];
  DeviceGuard dg(sh.device);
  return pq_shard_search(h, sh, d_queries, nq, k, nullptr, key_space == 0, d_out_ids, d_out_dists,
                         static_cast<cudaStream_t>(stream));
}

PX_API px_status px_pq_search_filtered(const px_pq* h, const float* queries, int64_t nq, int32_t k,
                                       const uint8_t* mask, int64_t* out_ids, float* out_dists) {
  px_status s = pq_check(h);
  if (s != PX_OK) return s;
  if (k < 0 || nq < 0) return set_error(PX_EINVAL, "k and nq must be >= 0");
  if (k > PX_MAX_K)
    return set_error(PX_EUNSUPPORTED, "k=" + std::to_string(k) + " exceeds PX_MAX_K=" + std::to_string(PX_MAX_K));
  if (k == 0 || nq == 0) return PX_OK;
  if (queries == nullptr || out_ids == nullptr || out_dists == nullptr)
    return set_error(PX_EINVAL, "null buffer");
  if (mask == nullptr && h->total > 0) return set_error(PX_EINVAL, "mask is null");
  if (!all_finite(queries, nq * h->dim))
    return set_error(PX_EINVAL, "query must not contain NaN or infinite values");
  return pq_search_host(h, queries, nq, k, mask, out_ids, out_dists);
}

}  // extern "C"
