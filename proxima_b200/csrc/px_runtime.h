// Host-side runtime structures shared by the C ABI translation units.
#pragma once

#include <atomic>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/px.h"
#include "px_kernels.h"

namespace px {

extern thread_local std::string g_last_error;
constexpr int kShardFlags = 8;  // words of FlatShard::flag
px_status set_error(px_status s, const std::string& msg);
px_status cuda_status(cudaError_t e, const char* what);
bool all_finite(const float* p, int64_t count);
int device_sm_count(int dev);
size_t device_smem_optin(int dev);  // opt-in shared memory per block (bytes)
px_status resolve_devices(const int32_t* devices, int32_t ndev, std::vector<int>& out);
void split_rows(int64_t n, int parts, std::vector<int64_t>& begin, std::vector<int64_t>& count);

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev);
  ~DeviceGuard();
};

// Grow-only device allocation (freed explicitly by the owner).
struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  cudaError_t reserve(size_t need);
  void release();
};

// Grow-only page-locked host allocation.
struct HostBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  px_status reserve(size_t need);
  void release();
};
bool is_pinned(const void* p);

struct Carver {
  void* base = nullptr;
  size_t used = 0;
  Carver() = default;
  explicit Carver(void* b) : base(b) {}
  void* take(size_t bytes);
};

// Maps shard-local rows to global ids: one (local_begin, global_begin) pair
// per add() run that reached this shard.
struct Segments {
  std::vector<int64_t> local, global;
  DevBuf dev;
  bool dirty = true;
  px_status sync_device();
  IdSegments view(int64_t id_offset) const;
  void local_mask(const uint8_t* global_mask, int64_t n_local, std::vector<uint8_t>& out) const;
  // Calls fn(local_begin, global_begin, count) for each run of this shard's
  // rows whose global ids fall in [start, end).
  template <class Fn>
  px_status for_range(int64_t n_local, int64_t start, int64_t end, Fn&& fn) const {
    for (size_t i = 0; i < local.size(); ++i) {
      const int64_t lb = local[i];
      const int64_t le = (i + 1 < local.size()) ? local[i + 1] : n_local;
      const int64_t gb = global[i], ge = gb + (le - lb);
      const int64_t s = gb > start ? gb : start, e = ge < end ? ge : end;
      if (s < e) {
        px_status st = fn(lb + (s - gb), s, e - s);
        if (st != PX_OK) return st;
      }
    }
    return PX_OK;
  }
};

}  // namespace px

struct FlatShard {
  int device = 0;
  int sms = 148;
  cudaStream_t stream = nullptr;
  float* x = nullptr;      // fp32 rows, stride ld
  float* hl = nullptr;     // tf32 split, stride 2*ld: per 16-element chunk hi x16 then lo x16
  float* norms = nullptr;  // squared norms
  void* xb = nullptr;      // bf16 rows, stride ldb (a multiple of 64), zero padded
  int64_t n = 0, cap = 0;
  int* flag = nullptr;     // [0] lo plane nonzero, [1] some value inexact in bf16,
                           // [2] max squared norm, [3] max ||x - bf16(x)||,
                           // [4] max ||x - tf32_hi(x)|| (float bits); written by appends
  bool lo_nonzero = false;
  bool bf_inexact = false;
  float max_norm_sq = 0.f;
  float bf_resid = 0.f;    // upper bounds on the rows' largest representation errors
  float tf_resid = 0.f;
  cudaEvent_t ev_start = nullptr, ev_stop = nullptr;  // brackets the dominant kernel when profiling
  cudaEvent_t ev_done = nullptr;  // this shard's results are in the gather buffer (own device)
  int last_path = 0, last_fallback = 0, last_refined = 0, last_launches = 0, last_pass = -1;
  int last_sample_tiles = 0;
  bool last_profiled = false;
  px::Segments segs;
  px::DevBuf ws;           // search workspace
  px::DevBuf stage;        // uploads (queries, rows, masks, outputs)
  px::DevBuf ws2;          // three-pass refinement workspace
  px::DevBuf fb;           // certificate-fallback workspace
  int64_t* out_ids = nullptr;  // results of the last search (inside stage)
  float* out_dists = nullptr;
  int* counters_h = nullptr;   // page-locked copy of a tensor pass's device counters (4 ints)
  // Totals since the last px_flat_profile_totals reset; the last profiled
  // search's kernel time is added when the events are next needed.
  bool prof_pending = false;
  double tot_ms = 0.0;
  int64_t tot_profiled = 0, tot_searches = 0, tot_fallback = 0, tot_refined = 0;

  px_status ensure_capacity(int64_t need, int ld, int ldb);
  px_status append_device(const float* d_src, int64_t count, int d, int ld, int ldb, int64_t global_begin);
  void release();
};

// Device-0 buffers for gathering the shards' lists in a multi-device handle.
struct GatherBuf {
  int device = -1;
  size_t cap = 0;
  float* keys = nullptr;
  int64_t* ids = nullptr;
  float* out_dists = nullptr;
  int64_t* out_ids = nullptr;
  cudaEvent_t events[8] = {};
  px_status ensure(int dev, size_t entries);
  void release_all();
};

// A captured small-batch search (query upload, exact scan, merge, emit,
// result download) with the staging and workspace buffers it owns. Besides
// those it depends only on the shard's rows and segment table, which change
// only through an add or reserve; those clear the handle's graphs first.
struct FlatSearchGraph {
  int64_t nq = 0, n = 0, id_offset = 0, rows_per_cta = 0;
  int k = 0, metric = 0, natural = 0, group = 0, ncta = 0;
  cudaGraphExec_t exec = nullptr;
  void* pinned = nullptr;  // page-locked queries and results (owned)
  void* dev = nullptr;     // device queries, results and scan workspace (owned)
  uint64_t last_use = 0;
};

struct px_flat {
  int dim = 0;
  int ld = 0;   // fp32 / split-plane row stride: dim rounded up to 32
  int ldb = 0;  // bf16 plane row stride: dim rounded up to 64 (plus 64 for a small-dim L2 index's folded norms)
  int metric = 0;
  int64_t total = 0;
  int64_t id_offset = 0;
  int path_mode = PX_PATH_AUTO;
  int sample_mode = PX_SAMPLE_AUTO;
  std::vector<FlatShard> shards;
  GatherBuf gather;
  px::HostBuf pinned;  // staging for pageable host buffers
  std::vector<FlatSearchGraph> graphs;  // single-shard small-batch replays (shard 0's device)
  uint64_t graph_clock = 0;
  std::mutex mu;
};

namespace px {

enum class FlatPath { Exact = 0, Gemm = 1 };

struct SearchPlan {
  FlatPath path = FlatPath::Exact;
  // exact scan
  int group = 1;
  int ncta = 1;
  int64_t rows_per_cta = 0;
  // tensor-core path
  int cap = 0, cands = 0, T = 0, S = 0, nb = 0, tiles_per_split = 0, n_items = 0, grid = 0;
  int lists = 0;  // candidate lists per query: S, or 4 * S on CTA pairs
  int seed_S = 0;  // single-tile splits of the bf16 pass's sample pass (0: none)
  int64_t q_rows = 0;
  size_t ws_bytes = 0;
  uint64_t* partial = nullptr;
  uint64_t* final_cands = nullptr;
};

extern std::atomic<int64_t> g_launches;
extern std::atomic<int> g_profiling;

px_status plan_flat_search(const px_flat* h, const FlatShard& sh, int64_t nq, int k, bool masked,
                           SearchPlan& plan);
// A tensor-core search whose certificate has not been read back yet: its
// candidates are in plan.final_cands, provisionally (every query certified).
struct TensorPending {
  bool active = false;
  int metric = 0, k = 0, first = 0;
  int64_t nq = 0, launches0 = 0;
  const float* d_q = nullptr;
  const uint8_t* d_mask = nullptr;
  const uint32_t* mask_bits = nullptr;
  int* fail_list = nullptr;
  uint64_t* final_cands = nullptr;
  cudaStream_t stream = nullptr;
};
// With pend == nullptr the search completes before it returns. Otherwise a
// tensor-core search returns after enqueueing its rescoring and the copy of
// its certificate counters (pend->active): the caller may enqueue work on
// the candidates (the emit), then must call finish_flat_search, which waits
// for the stream and runs the refinement or the exact scan for uncertified
// queries; *changed then says whether the candidates were rewritten.
px_status run_flat_search(const px_flat* h, FlatShard& sh, SearchPlan& plan, int metric,
                          const float* d_q, int64_t nq, int k, const uint8_t* d_mask,
                          cudaStream_t stream, void* ws = nullptr, TensorPending* pend = nullptr);
px_status finish_flat_search(const px_flat* h, FlatShard& sh, TensorPending& pend, bool* changed);
// Adds the last profiled search's kernel time to the shard's totals (waits
// for its stop event); called before the events are recorded again.
px_status flush_search_profile(FlatShard& sh);
px_status first_pass_candidates(const px_flat* h, FlatShard& sh, int metric, const float* d_q, int64_t nq,
                                int k, cudaStream_t stream, const uint64_t** merged, int* cands, int* pass);

}  // namespace px
