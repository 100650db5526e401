// Flat-search planning and execution on one shard.
//
// Paths:
//   Exact (K2)  : the exact streaming scan; bit-exact keys, no rescoring.
//                 Serves small batches (nq < kGemmMinQueries) and k beyond
//                 the tensor-core path's candidate capacity.
//   Gemm (K1+K5): tcgen05 contraction with a fused per-query top-CAP, split
//                 merge, exact rescoring and a certificate. The first pass
//                 reads only the tf32 hi planes; uncertified queries get a
//                 3xTF32 pass when enough of them fail, and the exact scan
//                 (K2) serves whatever is still uncertified.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <numeric>
#include <string>
#include <vector>

#include "px_common.cuh"
#include "px_runtime.h"

namespace px {

std::atomic<int64_t> g_launches{0};
std::atomic<int> g_profiling{0};

namespace {

constexpr int kGemmMinQueries = 16;
constexpr int kGemmMinRows = 4096;
// The bf16 pass's sample pass: this many single base tiles spread evenly over
// the shard (8,192 rows), taken when the shard holds at least four times as
// many tiles and (PX_SAMPLE_AUTO) its splits are at least kSeedMinSplitTiles
// long.
constexpr int kSeedSplits = 32;
constexpr int kSeedMinSplitTiles = 512;

int64_t gcd64(int64_t a, int64_t b) {
  while (b) {
    int64_t t = a % b;
    a = b;
    b = t;
  }
  return a;
}

}  // namespace

// Work split of one tensor-core candidate pass over nq queries. Workers are
// the persistent CTAs (one per SM), or CTA pairs for the bf16 pass.
static void plan_gemm(const FlatShard& sh, int64_t nq, int k, PassKind kind, int sample_mode, SearchPlan& plan) {
  plan.path = FlatPath::Gemm;
  const bool pair = kind == kPassBf16;
  plan.cap = pair ? gemm_pair_cap(k) : gemm_cap_for(k);
  plan.cands = pair ? gemm_pair_cands(k) : gemm_cands_for(k);
  // Work items: (group of query tiles, run of base tiles).
  const int64_t group_rows = pair ? 256 : static_cast<int64_t>(gemm_qt_for(k)) * 128;
  const int64_t bn = pair ? 256 : gemm_bn_for(k);
  const int64_t workers = pair ? gemm_pair_clusters(sh.device) : sh.sms;
  const int64_t T = (nq + group_rows - 1) / group_rows;
  const int64_t nb = std::max<int64_t>(1, (sh.n + bn - 1) / bn);
  // Splits so that T * S is a whole number of waves of the workers.
  int64_t S = workers / gcd64(T, workers);
  while (S * 2 <= 1024 && S * T < 2 * workers && S * 2 <= nb) S *= 2;
  S = std::min<int64_t>(S, nb);
  S = std::max<int64_t>(S, 1);
  // Fewer, longer splits: each (query, split) list starts with a loose
  // threshold and refills about CAP * (1 + ln(rows / CAP)) times, so a list
  // twice as long costs far less than two lists. When one wave of longer
  // splits keeps nine tenths of the workers busy it does the same MMA work
  // with fewer lists: config 1 goes from 36 splits of 11 tiles to 18 of 22,
  // config 2 (4 query groups) from 37 splits to 18.
  const int64_t one_wave = workers / T;
  if (one_wave >= 1 && one_wave < S && T * one_wave * 10 >= workers * 9) S = std::min<int64_t>(one_wave, nb);
  const int64_t tps = (nb + S - 1) / S;
  S = (nb + tps - 1) / tps;
  plan.T = static_cast<int>(T);
  plan.S = static_cast<int>(S);
  plan.lists = static_cast<int>(pair ? 4 * S : S);
  plan.nb = static_cast<int>(nb);
  plan.tiles_per_split = static_cast<int>(tps);
  plan.n_items = static_cast<int>(T * S);
  plan.grid = static_cast<int>(pair ? 2 * std::min<int64_t>(workers, T * S) : std::min<int64_t>(workers, T * S));
  plan.q_rows = T * group_rows;
  // Sample pass: each list of a fresh split accepts every row until it holds
  // CAP of them and then refills about CAP * (1 + ln(rows / CAP)) times. A
  // first pass over a strided sample of kSeedSplits tiles gives every query
  // the cands-th best key among 8,192 rows, and the main pass's lists admit
  // only keys at or below it. The cands-th, not the k-th: that key also
  // bounds the certificate, and the merged candidates' own bound is their
  // cands-th key, so the start costs the certificate nothing (on clustered
  // data the sample's k-th key lies within the bf16 error of the true k-th).
  // It pays on long splits (config 5: 269 -> 259 ms; config 4 unchanged).
  // On short ones (configs 1, 2) it costs more than it saves: their lists
  // still refill often enough that nearly every 32-column block has some
  // lane of the warp on the insertion path, while the sample pass and its
  // merge add a fixed 20-50 us.
  const bool seed_ok = pair && nb >= 4 * kSeedSplits;
  plan.seed_S = 0;
  if (seed_ok && (sample_mode == PX_SAMPLE_ON || (sample_mode == PX_SAMPLE_AUTO && tps >= kSeedMinSplitTiles)))
    plan.seed_S = kSeedSplits;
}

namespace {

// Device workspace of one tensor-core candidate pass.
struct TensorWs {
  float* q_hl = nullptr;            // query split plane, q_rows x 2*ld (tf32 passes)
  void* qb = nullptr;               // query bf16 plane, q_rows x ldb (bf16 pass)
  uint64_t* partial = nullptr;      // [nq][S][cap] per-split lists
  uint64_t* seed_partial = nullptr; // [nq][4 * seed_S][cap] the sample pass's lists
  uint64_t* seed = nullptr;         // [nq][cands] their merged best: the main pass's thresholds
  uint64_t* merged = nullptr;       // [nq][cands]
  uint64_t* final_cands = nullptr;  // [nq][k] exact candidates
  int* status = nullptr;            // [nq]
  int* fail_list = nullptr;         // [nq] uncertified queries
  int* counters = nullptr;          // [0] uncertified count, [1] query lo plane in use, [2] timeout,
                                    // [3] some query value inexact in bf16
};

// The first candidate pass: bf16 where enough candidates can be rescored for
// its wider bound to certify typical data (k <= 100), tf32 hi values
// otherwise.
PassKind first_pass_for(const px_flat* h, int k) {
  if (h->path_mode == PX_PATH_TENSOR_3XTF32) return kPass3xTf32;
  return gemm_pair_cands(k) > 0 ? kPassBf16 : kPassTf32;
}

void carve_tensor_ws(Carver& c, const SearchPlan& plan, int64_t nq, int ld, int ldb, int k, PassKind kind,
                     TensorWs& w) {
  if (kind == kPassBf16)
    w.qb = c.take(2 * static_cast<size_t>(plan.q_rows) * ldb);
  else
    w.q_hl = static_cast<float*>(c.take(sizeof(float) * static_cast<size_t>(plan.q_rows) * 2 * ld));
  w.partial = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * plan.lists * plan.cap));
  if (kind == kPassBf16 && plan.seed_S > 0) {
    w.seed_partial =
        static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * 4 * plan.seed_S * plan.cap));
    w.seed = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * plan.cands));
  }
  w.merged = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * plan.cands));
  w.final_cands = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * k));
  w.status = static_cast<int*>(c.take(sizeof(int) * static_cast<size_t>(nq)));
  w.fail_list = static_cast<int*>(c.take(sizeof(int) * static_cast<size_t>(nq)));
  w.counters = static_cast<int*>(c.take(sizeof(int) * 4));
}

size_t mask_words(int64_t n) { return static_cast<size_t>((n + 31) / 32 + 8); }

// A three-pass candidate pass over the uncertified queries pays when it is
// cheaper than exact scans of them. Per query, the exact scan issues 2*d
// FP32 instructions per row (no FMA, reference order) at ~36 T/s, while the
// three-pass contraction runs at ~186 TFLOP/s of 2*d FLOP per row but over
// whole groups of 128 * QT queries: the pass pays once the uncertified
// queries fill about a fifth of one group.
bool refine_pays(int64_t n_fail, int k) { return n_fail * 5 >= static_cast<int64_t>(gemm_qt_for(k)) * 128; }

}  // namespace

px_status plan_flat_search(const px_flat* h, const FlatShard& sh, int64_t nq, int k, bool masked,
                           SearchPlan& plan) {
  plan = SearchPlan{};
  const int cap = gemm_cap_for(k);
  bool gemm = cap > 0 && h->ld % 32 == 0 && sh.hl != nullptr;
  if (h->path_mode == PX_PATH_EXACT) gemm = false;
  if (h->path_mode == PX_PATH_AUTO) gemm = gemm && nq >= kGemmMinQueries && sh.n >= kGemmMinRows;
  if ((h->path_mode == PX_PATH_TENSOR || h->path_mode == PX_PATH_TENSOR_3XTF32) && !gemm)
    return set_error(PX_EUNSUPPORTED, "the tensor-core path cannot serve this request (k, mask or layout)");
  if (nq > (int64_t(1) << 30)) return set_error(PX_EUNSUPPORTED, "too many queries in one call");
  Carver c;
  if (gemm) {
    const PassKind first = first_pass_for(h, k);
    plan_gemm(sh, nq, k, first, h->sample_mode, plan);
    TensorWs w;
    carve_tensor_ws(c, plan, nq, h->ld, h->ldb, k, first, w);
    if (masked) c.take(sizeof(uint32_t) * mask_words(sh.n));
  } else {
    plan.path = FlatPath::Exact;
    const int group = exact_group_for(nq, k, h->dim, device_smem_optin(sh.device));
    if (group == 0)
      return set_error(PX_EUNSUPPORTED, "dim=" + std::to_string(h->dim) + " with k=" + std::to_string(k) +
                                            " exceeds the exact scan's shared memory");
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

// The exact scan for `count` queries of `src_q` picked by the device list
// `idx`; their k exact candidates are scattered to dst[idx[j]].
static px_status exact_for_list(const px_flat* h, FlatShard& sh, int metric, const float* src_q,
                                const int* idx, int count, int k, const uint8_t* d_mask,
                                uint64_t* dst, cudaStream_t stream) {
  const int group = exact_group_for(count, k, h->dim, device_smem_optin(sh.device));
  if (group == 0)
    return set_error(PX_EUNSUPPORTED, "dim=" + std::to_string(h->dim) + " with k=" + std::to_string(k) +
                                          " exceeds the exact scan's shared memory");
  const int64_t groups = (count + group - 1) / group;
  const int64_t n = std::max<int64_t>(sh.n, 1);
  int64_t ncta = std::max<int64_t>(1, (static_cast<int64_t>(sh.sms) * 4 + groups - 1) / groups);
  ncta = std::min<int64_t>(std::min<int64_t>(ncta, (n + 127) / 128), 1024);
  int64_t rows = ((n + ncta - 1) / ncta + 127) / 128 * 128;
  ncta = (n + rows - 1) / rows;
  Carver fc;
  fc.take(sizeof(float) * static_cast<size_t>(count) * h->dim);
  fc.take(sizeof(uint64_t) * static_cast<size_t>(count) * ncta * k);
  fc.take(sizeof(uint64_t) * static_cast<size_t>(count) * k);
  cudaError_t e = sh.fb.reserve(fc.used);
  if (e != cudaSuccess) return cuda_status(e, "fallback workspace allocation");
  fc = Carver(sh.fb.ptr);
  float* fq = static_cast<float*>(fc.take(sizeof(float) * static_cast<size_t>(count) * h->dim));
  uint64_t* fpart = static_cast<uint64_t*>(fc.take(sizeof(uint64_t) * static_cast<size_t>(count) * ncta * k));
  uint64_t* fout = static_cast<uint64_t*>(fc.take(sizeof(uint64_t) * static_cast<size_t>(count) * k));
  e = launch_gather_rows(src_q, h->dim, idx, count, fq, stream);
  if (e != cudaSuccess) return cuda_status(e, "fallback gather");
  px_status s = run_exact(h, sh, metric, fq, count, k, d_mask, fpart, static_cast<int>(ncta), group, rows, fout,
                          stream, false);
  if (s != PX_OK) return s;
  e = launch_scatter_cands(fout, k, idx, count, dst, stream);
  if (e != cudaSuccess) return cuda_status(e, "fallback scatter");
  g_launches += 2;
  return PX_OK;
}

// One tensor-core candidate pass: convert the queries, K1 over the shard
// (bf16 copies, tf32 hi values, or the three-pass tf32 sum), split merge,
// exact rescoring and certificate. Leaves exact candidates in w.final_cands
// and the uncertified queries in w.fail_list, and enqueues the copy of the
// pass's counters to the shard's page-locked sh.counters_h (read by
// tensor_pass_read once the stream has reached it).
static px_status tensor_pass_launch(const px_flat* h, FlatShard& sh, const SearchPlan& plan, int metric,
                                    const float* d_q, int64_t nq, int k, const uint32_t* mask_bits,
                                    PassKind kind, const TensorWs& w, bool profile_main, cudaStream_t stream) {
  const bool l2 = metric == PX_METRIC_L2;
  // An L2 bf16 pass over rows that carry their norms in the padding runs as
  // an inner product of 2q with them: no per-element norm term in the
  // epilogue.
  const bool folded = l2 && kind == kPassBf16 && h->dim + 3 <= h->ldb;
  cudaError_t e = cudaMemsetAsync(w.counters, 0, sizeof(int) * 4, stream);
  if (e == cudaSuccess)
    e = launch_split_queries(d_q, nq, h->dim, h->ld, h->ldb, plan.q_rows, w.q_hl, w.qb, w.counters + 1,
                             w.counters + 3, stream, folded);
  if (e != cudaSuccess) return cuda_status(e, "query split");
  GemmTopkArgs g;
  g.nq = static_cast<int>(nq);
  g.n = sh.n;
  g.ld = h->ld;
  g.ldb = h->ldb;
  g.k = k;
  g.T = plan.T;
  g.S = plan.S;
  g.tiles_per_split = plan.tiles_per_split;
  g.split_stride = plan.tiles_per_split;
  g.nb = plan.nb;
  g.n_items = plan.n_items;
  g.l2 = l2 && !folded;
  g.norms = sh.norms;
  g.x_lo_nonzero = sh.lo_nonzero ? 1 : 0;
  g.q_lo_flag = w.counters + 1;
  g.partial = w.partial;
  g.err = w.counters + 2;
  g.mask_bits = mask_bits;
  g.seed = nullptr;
  g.seed_k = plan.cands;
  const bool seeded = w.seed != nullptr;
  if (profile_main) cudaEventRecord(sh.ev_start, stream);
  if (seeded) {
    // The sample pass: one tile per split, the splits kSeedSplits evenly
    // spaced tiles apart, same kernel and filter; then the cands best words
    // of its lists per query.
    GemmTopkArgs gs = g;
    gs.S = plan.seed_S;
    gs.tiles_per_split = 1;
    gs.split_stride = plan.nb / plan.seed_S;
    gs.n_items = plan.T * plan.seed_S;
    gs.partial = w.seed_partial;
    const int seed_grid =
        2 * static_cast<int>(std::min<int64_t>(gemm_pair_clusters(sh.device), static_cast<int64_t>(gs.n_items)));
    e = launch_gemm_topk(gs, w.qb, plan.q_rows, sh.xb, kind, seed_grid, stream);
    if (e != cudaSuccess) return cuda_status(e, "tensor-core sample pass launch");
    e = launch_merge_lists(w.seed_partial, nq, 4 * plan.seed_S, plan.cap, plan.cands, w.seed, stream);
    if (e != cudaSuccess) return cuda_status(e, "sample merge launch");
    g.seed = w.seed;
    g_launches += 2;
  }
  if (kind == kPassBf16)
    e = launch_gemm_topk(g, w.qb, plan.q_rows, sh.xb, kind, plan.grid, stream);
  else
    e = launch_gemm_topk(g, w.q_hl, plan.q_rows, sh.hl, kind, plan.grid, stream);
  if (profile_main) cudaEventRecord(sh.ev_stop, stream);
  if (e != cudaSuccess) return cuda_status(e, "tensor-core kernel launch");
  e = launch_merge_lists(w.partial, nq, plan.lists, plan.cap, plan.cands, w.merged, stream);
  if (e != cudaSuccess) return cuda_status(e, "split merge launch");
  RescoreArgs r;
  r.merged = w.merged;
  r.nq = nq;
  r.cap = plan.cands;
  r.k = k;
  r.lists = w.partial;
  r.nlists = plan.lists;
  r.list_cap = plan.cap;
  r.queries = d_q;
  r.base = sh.x;
  r.ld = h->ld;
  r.d = h->dim;
  r.l2 = l2;
  r.max_norm_sq = sh.max_norm_sq;
  r.x_resid = kind == kPassBf16 ? sh.bf_resid : (kind == kPassTf32 ? sh.tf_resid : 0.f);
  r.x_lo_nonzero = sh.lo_nonzero ? 1 : 0;
  r.q_lo_flag = w.counters + 1;
  r.pass_kind = kind;
  r.norm_folded = folded ? 1 : 0;
  r.seed = g.seed;
  r.seed_k = plan.cands;
  r.out = w.final_cands;
  r.status = w.status;
  r.n_fail = w.counters;
  r.fail_list = w.fail_list;
  e = launch_rescore(r, stream);
  if (e != cudaSuccess) return cuda_status(e, "rescore launch");
  g_launches += 5;  // split, gemm, merge, rescore (+ memset counted as one)
  if (sh.counters_h == nullptr) {
    e = cudaMallocHost(&sh.counters_h, sizeof(int) * 4);
    if (e != cudaSuccess) {
      sh.counters_h = nullptr;
      return cuda_status(e, "certificate readback buffer");
    }
  }
  e = cudaMemcpyAsync(sh.counters_h, w.counters, sizeof(int) * 4, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return cuda_status(e, "certificate readback");
  return PX_OK;
}

// After the stream has passed a tensor pass's counter copy: the count of
// uncertified queries, and whether the pass's operands were inexact, i.e.
// whether a more precise pass could certify them.
static px_status tensor_pass_read(const FlatShard& sh, PassKind kind, int* n_fail, bool* inexact) {
  const int* hc = sh.counters_h;
  if (hc[2] != 0)
    return set_error(PX_ETIMEOUT, "a tensor-core pipeline wait timed out on device " +
                                      std::to_string(sh.device) + "; the search was abandoned");
  *n_fail = hc[0];
  *inexact = kind == kPassBf16 ? (sh.bf_inexact || hc[3] != 0) : (sh.lo_nonzero || hc[1] != 0);
  return PX_OK;
}

// The whole pass with its one host wait.
static px_status tensor_pass(const px_flat* h, FlatShard& sh, const SearchPlan& plan, int metric,
                             const float* d_q, int64_t nq, int k, const uint32_t* mask_bits, PassKind kind,
                             const TensorWs& w, bool profile_main, cudaStream_t stream, int* n_fail,
                             bool* inexact) {
  px_status s = tensor_pass_launch(h, sh, plan, metric, d_q, nq, k, mask_bits, kind, w, profile_main, stream);
  if (s != PX_OK) return s;
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_status(e, "certificate readback");
  return tensor_pass_read(sh, kind, n_fail, inexact);
}

// Refinement or exact scan for the queries a first tensor pass left
// uncertified (n_fail of them, listed in fail_list); their exact candidates
// are scattered into final_cands.
static px_status certify_rest(const px_flat* h, FlatShard& sh, int metric, const float* d_q, int k,
                              const uint8_t* d_mask, const uint32_t* mask_bits, PassKind first, int n_fail,
                              bool inexact, int* fail_list, uint64_t* final_cands, cudaStream_t stream) {
  if (first != kPass3xTf32 && inexact && refine_pays(n_fail, k)) {
    SearchPlan p2;
    plan_gemm(sh, n_fail, k, kPass3xTf32, h->sample_mode, p2);
    Carver c2;
    c2.take(sizeof(float) * static_cast<size_t>(n_fail) * h->dim);
    TensorWs w2;
    carve_tensor_ws(c2, p2, n_fail, h->ld, h->ldb, k, kPass3xTf32, w2);
    cudaError_t e = sh.ws2.reserve(c2.used);
    if (e != cudaSuccess) return cuda_status(e, "refinement workspace allocation");
    c2 = Carver(sh.ws2.ptr);
    float* fq = static_cast<float*>(c2.take(sizeof(float) * static_cast<size_t>(n_fail) * h->dim));
    carve_tensor_ws(c2, p2, n_fail, h->ld, h->ldb, k, kPass3xTf32, w2);
    e = launch_gather_rows(d_q, h->dim, fail_list, n_fail, fq, stream);
    if (e != cudaSuccess) return cuda_status(e, "refinement gather");
    int n_fail2 = 0;
    bool inexact2 = false;
    px_status s = tensor_pass(h, sh, p2, metric, fq, n_fail, k, mask_bits, kPass3xTf32, w2, false, stream,
                              &n_fail2, &inexact2);
    if (s != PX_OK) return s;
    if (n_fail2 > 0) {
      s = exact_for_list(h, sh, metric, fq, w2.fail_list, n_fail2, k, d_mask, w2.final_cands, stream);
      if (s != PX_OK) return s;
    }
    e = launch_scatter_cands(w2.final_cands, k, fail_list, n_fail, final_cands, stream);
    if (e != cudaSuccess) return cuda_status(e, "refinement scatter");
    g_launches += 2;
    sh.last_refined = n_fail;
    sh.last_fallback = n_fail2;
    return PX_OK;
  }
  px_status s = exact_for_list(h, sh, metric, d_q, fail_list, n_fail, k, d_mask, final_cands, stream);
  if (s != PX_OK) return s;
  sh.last_fallback = n_fail;
  return PX_OK;
}

px_status flush_search_profile(FlatShard& sh) {
  if (!sh.prof_pending) return PX_OK;
  sh.prof_pending = false;
  DeviceGuard dg(sh.device);
  float ms = 0.f;
  cudaError_t e = cudaEventSynchronize(sh.ev_stop);
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, sh.ev_start, sh.ev_stop);
  if (e != cudaSuccess) return cuda_status(e, "profile events");
  sh.tot_ms += ms;
  sh.tot_profiled += 1;
  return PX_OK;
}

px_status finish_flat_search(const px_flat* h, FlatShard& sh, TensorPending& pend, bool* changed) {
  *changed = false;
  pend.active = false;
  cudaError_t e = cudaStreamSynchronize(pend.stream);
  if (e != cudaSuccess) return cuda_status(e, "certificate readback");
  int n_fail = 0;
  bool inexact = false;
  const PassKind first = static_cast<PassKind>(pend.first);
  px_status s = tensor_pass_read(sh, first, &n_fail, &inexact);
  if (s != PX_OK) return s;
  if (n_fail > 0) {
    s = certify_rest(h, sh, pend.metric, pend.d_q, pend.k, pend.d_mask, pend.mask_bits, first, n_fail, inexact,
                     pend.fail_list, pend.final_cands, pend.stream);
    if (s != PX_OK) return s;
    *changed = true;
  }
  sh.last_launches = static_cast<int>(g_launches.load() - pend.launches0);
  return PX_OK;
}

px_status run_flat_search(const px_flat* h, FlatShard& sh, SearchPlan& plan, int metric,
                          const float* d_q, int64_t nq, int k, const uint8_t* d_mask,
                          cudaStream_t stream, void* ws, TensorPending* pend) {
  px_status fs = flush_search_profile(sh);
  if (fs != PX_OK) return fs;
  const bool prof = g_profiling.load() != 0;
  sh.last_path = static_cast<int>(plan.path);
  sh.last_fallback = 0;
  sh.last_refined = 0;
  sh.last_pass = -1;
  sh.last_sample_tiles = 0;
  sh.last_profiled = prof;
  const int64_t launches0 = g_launches.load();
  Carver c(ws ? ws : sh.ws.ptr);
  if (plan.path == FlatPath::Exact) {
    plan.partial = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * plan.ncta * k));
    plan.final_cands = static_cast<uint64_t*>(c.take(sizeof(uint64_t) * static_cast<size_t>(nq) * k));
    px_status s = run_exact(h, sh, metric, d_q, nq, k, d_mask, plan.partial, plan.ncta, plan.group,
                            plan.rows_per_cta, plan.final_cands, stream, prof);
    sh.last_launches = static_cast<int>(g_launches.load() - launches0);
    return s;
  }

  // ---- tensor-core path ----
  // 1. One pass over bf16 copies (k <= 16) or tf32 hi values for every
  //    query. Its keys carry a rounding error, which the certificate's bound
  //    covers; on typical data nearly every query is certified.
  // 2. The uncertified queries, if that pass's operands were inexact and
  //    there are enough of them, get a three-pass (~fp32) candidate pass.
  // 3. Whatever is still uncertified goes through the exact scan.
  const PassKind first = first_pass_for(h, k);
  sh.last_pass = first;
  sh.last_sample_tiles = first == kPassBf16 ? plan.seed_S : 0;
  TensorWs w;
  carve_tensor_ws(c, plan, nq, h->ld, h->ldb, k, first, w);
  plan.final_cands = w.final_cands;
  uint32_t* mask_bits = d_mask ? static_cast<uint32_t*>(c.take(sizeof(uint32_t) * mask_words(sh.n))) : nullptr;
  if (mask_bits) {
    cudaError_t e = launch_pack_mask(d_mask, sh.n, mask_bits, stream);
    if (e != cudaSuccess) return cuda_status(e, "mask pack");
  }
  px_status s = tensor_pass_launch(h, sh, plan, metric, d_q, nq, k, mask_bits, first, w, prof, stream);
  if (s != PX_OK) return s;
  TensorPending local;
  TensorPending& p = pend ? *pend : local;
  p.active = true;
  p.metric = metric;
  p.k = k;
  p.first = first;
  p.nq = nq;
  p.launches0 = launches0;
  p.d_q = d_q;
  p.d_mask = d_mask;
  p.mask_bits = mask_bits;
  p.fail_list = w.fail_list;
  p.final_cands = w.final_cands;
  p.stream = stream;
  sh.last_launches = static_cast<int>(g_launches.load() - launches0);
  if (pend) return PX_OK;
  bool changed = false;
  return finish_flat_search(h, sh, p, &changed);
}

// Instrumentation: the first tensor-core candidate pass alone (query
// conversion, K1, split merge; the rescoring runs too but its results are
// not used). Leaves each query's merged approximate candidates in *merged
// ([nq][*cands], sorted by approximate key) inside the shard's workspace.
px_status first_pass_candidates(const px_flat* h, FlatShard& sh, int metric, const float* d_q, int64_t nq,
                                int k, cudaStream_t stream, const uint64_t** merged, int* cands, int* pass) {
  if (gemm_cap_for(k) <= 0 || h->ld % 32 != 0 || sh.hl == nullptr || sh.n < 1)
    return set_error(PX_EUNSUPPORTED, "the tensor-core path cannot serve this request (k or an empty shard)");
  if (nq > (int64_t(1) << 30)) return set_error(PX_EUNSUPPORTED, "too many queries in one call");
  const PassKind kind = first_pass_for(h, k);
  SearchPlan plan;
  plan_gemm(sh, nq, k, kind, h->sample_mode, plan);
  Carver c;
  TensorWs w;
  carve_tensor_ws(c, plan, nq, h->ld, h->ldb, k, kind, w);
  cudaError_t e = sh.ws.reserve(c.used);
  if (e != cudaSuccess) return cuda_status(e, "search workspace allocation");
  c = Carver(sh.ws.ptr);
  carve_tensor_ws(c, plan, nq, h->ld, h->ldb, k, kind, w);
  int n_fail = 0;
  bool inexact = false;
  px_status s = tensor_pass(h, sh, plan, metric, d_q, nq, k, nullptr, kind, w, false, stream, &n_fail, &inexact);
  if (s != PX_OK) return s;
  *merged = w.merged;
  *cands = plan.cands;
  *pass = kind;
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
