// Merges of sorted top-k lists and the conversion to caller outputs.
//
// The reference keeps one heap per query and converts its sorted contents to
// natural distances with -1 / f32::MAX / f32::MIN padding
// (crates/core/src/flat.rs:139-147, pq.rs:332-346). Here the per-CTA (or
// per-GPU) sorted lists are merged on the device and converted in one pass.
#include "px_common.cuh"
#include "px_kernels.h"

namespace px {

namespace {

constexpr int kMergeWarps = 4;

// Per-warp shared memory for a staged copy of one query's lists (the
// tournament's refills then read shared memory, not a dependent global load
// per step); larger lists merge straight from global memory.
constexpr size_t kMergeStageBytes = 40 * 1024;
// From this many output words on, the merge selects by value search
// (merge_select_kernel) rather than popping one word per tournament step.
constexpr int kMergeSelectMinK = 128;
// Shared memory the threshold merge (merge_heads_kernel) may take per block.
constexpr size_t kMergeHeadsMaxSmem = 200 * 1024;

// Copies n words to shared memory, 16 loads in flight per lane (a plain
// load-store loop would wait out a global-memory latency per word).
__device__ __forceinline__ void stage_words(uint64_t* dst, const uint64_t* __restrict__ src, int n, int lane) {
  constexpr int kInFlight = 16;
  for (int i0 = 0; i0 < n; i0 += 32 * kInFlight) {
    uint64_t v[kInFlight];
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const int i = i0 + u * 32 + lane;
      v[u] = i < n ? __ldg(src + i) : 0ull;
    }
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const int i = i0 + u * 32 + lane;
      if (i < n) dst[i] = v[u];
    }
  }
}

// Ascending bitonic sort of n words (a power of two, at least 2) in shared
// memory by one warp. (Loading all of a lane's pairs of a stage before
// storing any, in registers sized for n = 1,024, measured slower: it cut
// the warps per SM and did the largest sort's work for every n.)
__device__ __forceinline__ void warp_bitonic_sort(uint64_t* a, int n, int lane) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int p = lane; p < n / 2; p += 32) {
        // Pair p: positions lo_i, lo_i + stride (stride a power of two).
        const int lo_i = ((p & ~(stride - 1)) << 1) | (p & (stride - 1));
        const int hi_i = lo_i + stride;
        const bool up = (lo_i & size) == 0;
        const uint64_t x = a[lo_i], y = a[hi_i];
        if ((x > y) == up) {
          a[lo_i] = y;
          a[hi_i] = x;
        }
      }
      __syncwarp();
    }
  }
}

// One warp per query: a k-step tournament over `nlists` sorted lists. Each
// lane owns lists lane, lane+32, ...; it caches the smallest of its heads and
// rescans only after its own list advanced. STAGED: the query's lists are
// first copied to shared memory with coalesced loads.
template <bool STAGED>
__global__ void __launch_bounds__(kMergeWarps * 32)
merge_lists_kernel(const uint64_t* __restrict__ lists, int64_t nq, int nlists, int list_len,
                   int k, uint64_t* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* heads = reinterpret_cast<uint64_t*>(smem_raw) + static_cast<size_t>(warp) * nlists;
  int* pos = reinterpret_cast<int*>(reinterpret_cast<uint64_t*>(smem_raw) +
                                    static_cast<size_t>(kMergeWarps) * nlists) +
             static_cast<size_t>(warp) * nlists;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * kMergeWarps + warp;
  if (q >= nq) return;
  const uint64_t* ql = lists + q * static_cast<int64_t>(nlists) * list_len;
  if constexpr (STAGED) {
    // After heads ([warps][nlists] u64) and pos ([warps][nlists] int),
    // rounded up to 16 bytes.
    const size_t fixed = (static_cast<size_t>(kMergeWarps) * nlists * (sizeof(uint64_t) + sizeof(int)) + 15) & ~size_t(15);
    uint64_t* stage = reinterpret_cast<uint64_t*>(smem_raw + fixed) +
                      static_cast<size_t>(warp) * nlists * list_len;
    stage_words(stage, ql, nlists * list_len, lane);
    __syncwarp();
    ql = stage;
  }

  uint64_t best = PX_EMPTY;
  int best_list = -1;
  for (int l = lane; l < nlists; l += 32) {
    uint64_t h = list_len > 0 ? ql[static_cast<int64_t>(l) * list_len] : PX_EMPTY;
    heads[l] = h;
    pos[l] = 0;
    if (h < best) {
      best = h;
      best_list = l;
    }
  }
  __syncwarp();
  for (int j = 0; j < k; ++j) {
    uint64_t v = best;
    int src = lane;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      uint64_t ov = __shfl_xor_sync(0xffffffffu, v, off);
      int os = __shfl_xor_sync(0xffffffffu, src, off);
      if (ov < v || (ov == v && os < src)) {
        v = ov;
        src = os;
      }
    }
    if (lane == 0) out[q * k + j] = v;
    if (v == PX_EMPTY) {
      for (int jj = j + 1 + lane; jj < k; jj += 32) out[q * k + jj] = PX_EMPTY;
      return;
    }
    if (lane == src) {
      int l = best_list;
      int p = ++pos[l];
      heads[l] = p < list_len ? ql[static_cast<int64_t>(l) * list_len + p] : PX_EMPTY;
      best = PX_EMPTY;
      best_list = -1;
      for (int ll = lane; ll < nlists; ll += 32) {
        uint64_t h = heads[ll];
        if (h < best) {
          best = h;
          best_list = ll;
        }
      }
    }
    __syncwarp();
  }
}

// Number of words <= v in a sorted list of len words (an upper bound).
__device__ __forceinline__ int count_le_sorted(const uint64_t* L, int len, uint64_t v) {
  int lo = 0, hi = len;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (L[mid] <= v) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// One warp per query: the k smallest words of `nlists` sorted lists by a
// threshold instead of a k-step tournament (whose k dependent warp
// reductions dominate small searches). The query's lists are staged in shared
// memory and their heads sorted; H, the k-th smallest head, bounds the
// answer, since k distinct words (those heads) are <= H. Only the lists whose
// head is <= H can hold words <= H -- exactly k lists, the words of a query
// being distinct -- so at most min(nlists, k) * list_len words qualify; they
// are gathered (exclusive scan of the lanes' counts) and sorted, and the
// first k are the answer. With fewer than k lists (or fewer than k non-empty
// ones) every real word qualifies. Shared memory per warp: the staged lists,
// hp words of heads and cp words of gathered candidates (powers of two, at
// most 1,024).
__global__ void __launch_bounds__(kMergeWarps * 32)
merge_heads_kernel(const uint64_t* __restrict__ lists, int64_t nq, int nlists, int list_len, int k, int hp,
                   int cp, uint64_t* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = nlists * list_len;
  uint64_t* stage = reinterpret_cast<uint64_t*>(smem_raw) + static_cast<size_t>(warp) * (total + hp + cp);
  uint64_t* heads = stage + total;
  uint64_t* cand = heads + hp;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * kMergeWarps + warp;
  if (q >= nq) return;
  stage_words(stage, lists + q * static_cast<int64_t>(total), total, lane);
  __syncwarp();
  uint64_t H = PX_EMPTY;
  if (nlists >= k) {
    for (int l = lane; l < hp; l += 32) heads[l] = l < nlists ? stage[l * list_len] : PX_EMPTY;
    __syncwarp();
    warp_bitonic_sort(heads, hp, lane);
    H = heads[k - 1];
  }
  // PX_EMPTY is the largest word: with H == PX_EMPTY count the real words.
  const uint64_t lim = H == PX_EMPTY ? PX_EMPTY - 1 : H;
  int mine = 0;
  for (int l = lane; l < nlists; l += 32) mine += count_le_sorted(stage + l * list_len, list_len, lim);
  int incl = mine;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  // <= cp by the argument above; the clamps only keep a violation of it
  // inside the buffer.
  const int count = min(__shfl_sync(0xffffffffu, incl, 31), cp);
  int at = incl - mine;
  for (int l = lane; l < nlists; l += 32) {
    const uint64_t* L = stage + l * list_len;
    const int c = count_le_sorted(L, list_len, lim);
    for (int i = 0; i < c && at < cp; ++i) cand[at++] = L[i];
  }
  int n2 = 32;
  while (n2 < count) n2 <<= 1;
  for (int i = count + lane; i < n2; i += 32) cand[i] = PX_EMPTY;
  __syncwarp();
  warp_bitonic_sort(cand, n2, lane);
  for (int j = lane; j < k; j += 32) out[q * k + j] = j < n2 ? cand[j] : PX_EMPTY;
}

// One warp per query, for large k: the k smallest words of `nlists` sorted
// lists, without a k-step tournament. The query's lists are staged in shared
// memory; the k-th smallest word T is found bit by bit, counting the words
// <= a trial value with a binary search in each list (32 steps over the key
// half; 32 more over the row half only when the boundary key repeats, since
// all words of a query are distinct: distinct rows). The words <= T are then
// gathered and sorted with a warp bitonic sort.
__global__ void __launch_bounds__(kMergeWarps * 32)
merge_select_kernel(const uint64_t* __restrict__ lists, int64_t nq, int nlists, int list_len, int k, int kp,
                    uint64_t* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = nlists * list_len;
  uint64_t* stage = reinterpret_cast<uint64_t*>(smem_raw) + static_cast<size_t>(warp) * (total + kp);
  uint64_t* sel = stage + total;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * kMergeWarps + warp;
  if (q >= nq) return;
  const uint64_t* ql = lists + q * static_cast<int64_t>(total);
  stage_words(stage, ql, total, lane);
  __syncwarp();
  auto count_le = [&](uint64_t v) {
    int c = 0;
    for (int l = lane; l < nlists; l += 32) c += count_le_sorted(stage + l * list_len, list_len, v);
    return __reduce_add_sync(0xffffffffu, c);
  };
  // Real (non-empty) words: PX_EMPTY is the largest word.
  const int real = count_le(PX_EMPTY - 1);
  const int kk = real < k ? real : k;
  uint64_t t = 0;  // the threshold: exactly kk words are <= t
  if (kk > 0) {
    uint32_t hi = 0;  // smallest key half with at least kk words at or below it
    for (int b = 31; b >= 0; --b) {
      const uint32_t trial = hi | ((1u << b) - 1u);
      if (count_le((static_cast<uint64_t>(trial) << 32) | 0xFFFFFFFFull) < kk) hi |= 1u << b;
    }
    t = (static_cast<uint64_t>(hi) << 32) | 0xFFFFFFFFull;
    if (count_le(t) != kk) {  // the boundary key repeats: resolve on the row half
      uint32_t lo = 0;
      for (int b = 31; b >= 0; --b) {
        const uint32_t trial = lo | ((1u << b) - 1u);
        if (count_le((static_cast<uint64_t>(hi) << 32) | trial) < kk) lo |= 1u << b;
      }
      t = (static_cast<uint64_t>(hi) << 32) | lo;
    }
  }
  // Gather the kk words <= t: each lane's lists' prefixes, at offsets from an
  // exclusive scan of the lanes' counts.
  int mine = 0;
  if (kk > 0)
    for (int l = lane; l < nlists; l += 32) mine += count_le_sorted(stage + l * list_len, list_len, t);
  int incl = mine;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  int at = incl - mine;
  if (kk > 0) {
    for (int l = lane; l < nlists; l += 32) {
      const uint64_t* L = stage + l * list_len;
      const int c = count_le_sorted(L, list_len, t);
      for (int i = 0; i < c && at < kp; ++i) sel[at++] = L[i];  // at most kk (<= kp) words qualify
    }
  }
  __syncwarp();
  for (int i = kk + lane; i < kp; i += 32) sel[i] = PX_EMPTY;
  __syncwarp();
  warp_bitonic_sort(sel, kp, lane);  // kp: a power of two, 128 .. 1,024
  for (int j = lane; j < k; j += 32) out[q * k + j] = sel[j];
}

__device__ __forceinline__ int64_t map_row(uint32_t row, const IdSegments& s) {
  int lo = 0, hi = s.nseg - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (s.local_begin[mid] <= static_cast<int64_t>(row)) lo = mid; else hi = mid - 1;
  }
  return s.global_begin[lo] + (static_cast<int64_t>(row) - s.local_begin[lo]) + s.id_offset;
}

__global__ void emit_kernel(const uint64_t* __restrict__ cands, int64_t total, bool l2, bool natural,
                            IdSegments segs, int64_t* __restrict__ out_ids,
                            float* __restrict__ out_dists) {
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  uint64_t c = cands[i];
  if (c == PX_EMPTY) {
    out_ids[i] = -1;
    out_dists[i] = natural ? pad_dist(l2) : 3.40282347e+38f;
  } else {
    out_ids[i] = map_row(cand_row(c), segs);
    float key = cand_key(c);
    out_dists[i] = natural ? natural_dist(key, l2) : key;
  }
}

// One thread per query: G-way merge of per-shard sorted (key, id) lists.
// Shard g's lists start key_stride / id_stride bytes after shard g-1's.
__global__ void merge_shards_kernel(const char* __restrict__ keys, int64_t key_stride,
                                    const char* __restrict__ ids, int64_t id_stride,
                                    int nshard, int64_t nq, int k, bool l2, bool natural,
                                    float* __restrict__ out_dists, int64_t* __restrict__ out_ids) {
  int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  int pos[8];
  for (int g = 0; g < nshard; ++g) pos[g] = 0;
  for (int j = 0; j < k; ++j) {
    int win = -1;
    uint32_t wk = 0;
    int64_t wid = 0;
    for (int g = 0; g < nshard; ++g) {
      if (pos[g] >= k) continue;
      const int64_t e = q * k + pos[g];
      const int64_t id = reinterpret_cast<const int64_t*>(ids + g * id_stride)[e];
      if (id < 0) continue;
      const uint32_t o = key_to_ord(reinterpret_cast<const float*>(keys + g * key_stride)[e]);
      if (win < 0 || o < wk || (o == wk && id < wid)) {
        win = g;
        wk = o;
        wid = id;
      }
    }
    if (win < 0) {
      out_ids[q * k + j] = -1;
      out_dists[q * k + j] = natural ? pad_dist(l2) : 3.40282347e+38f;
    } else {
      ++pos[win];
      float key = ord_to_key(wk);
      out_ids[q * k + j] = wid;
      out_dists[q * k + j] = natural ? natural_dist(key, l2) : key;
    }
  }
}

}  // namespace

cudaError_t launch_merge_lists(const uint64_t* lists, int64_t nq, int nlists, int list_len, int k,
                               uint64_t* out, cudaStream_t stream) {
  if (nq == 0 || k == 0) return cudaSuccess;
  const size_t fixed =
      (static_cast<size_t>(kMergeWarps) * nlists * (sizeof(uint64_t) + sizeof(int)) + 15) & ~size_t(15);
  const size_t stage = sizeof(uint64_t) * static_cast<size_t>(nlists) * list_len;
  const bool staged = stage <= kMergeStageBytes;
  // Threshold merge: heads and gathered candidates each at most 1,024 words.
  {
    int hp = 32, cp = 32;
    while (hp < nlists) hp <<= 1;
    const int64_t cmax = static_cast<int64_t>(nlists < k ? nlists : k) * list_len;
    while (cp < cmax) cp <<= 1;
    const size_t hsmem = static_cast<size_t>(kMergeWarps) * (stage + sizeof(uint64_t) * (hp + cp));
    if (staged && list_len > 0 && hp <= 1024 && cp <= 1024 && hsmem <= kMergeHeadsMaxSmem) {
      cudaError_t e = cudaFuncSetAttribute(merge_heads_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(hsmem));
      if (e != cudaSuccess) return e;
      const int64_t blocks = (nq + kMergeWarps - 1) / kMergeWarps;
      merge_heads_kernel<<<static_cast<unsigned>(blocks), kMergeWarps * 32, hsmem, stream>>>(
          lists, nq, nlists, list_len, k, hp, cp, out);
      return cudaGetLastError();
    }
  }
  // Large k: select by value search instead of a k-step tournament.
  if (staged && k >= kMergeSelectMinK && k <= 1024) {
    int kp = 1;
    while (kp < k) kp <<= 1;
    const size_t smem = static_cast<size_t>(kMergeWarps) * (stage + sizeof(uint64_t) * kp);
    cudaError_t e = cudaFuncSetAttribute(merge_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const int64_t blocks = (nq + kMergeWarps - 1) / kMergeWarps;
    merge_select_kernel<<<static_cast<unsigned>(blocks), kMergeWarps * 32, smem, stream>>>(lists, nq, nlists,
                                                                                          list_len, k, kp, out);
    return cudaGetLastError();
  }
  const size_t smem = fixed + (staged ? kMergeWarps * stage : 0);
  auto kern = staged ? merge_lists_kernel<true> : merge_lists_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int64_t blocks = (nq + kMergeWarps - 1) / kMergeWarps;
  kern<<<static_cast<unsigned>(blocks), kMergeWarps * 32, smem, stream>>>(lists, nq, nlists, list_len, k, out);
  return cudaGetLastError();
}

cudaError_t launch_emit(const uint64_t* cands, int64_t nq, int k, bool l2, bool natural,
                        IdSegments segs, int64_t* out_ids, float* out_dists, cudaStream_t stream) {
  const int64_t total = nq * k;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  emit_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0, stream>>>(
      cands, total, l2, natural, segs, out_ids, out_dists);
  return cudaGetLastError();
}

cudaError_t launch_merge_shards(const float* keys, const int64_t* ids, int nshard, int64_t nq, int k,
                                bool l2, bool natural, float* out_dists, int64_t* out_ids,
                                cudaStream_t stream) {
  return launch_merge_shards_strided(keys, static_cast<int64_t>(sizeof(float)) * nq * k, ids,
                                     static_cast<int64_t>(sizeof(int64_t)) * nq * k, nshard, nq, k, l2, natural,
                                     out_dists, out_ids, stream);
}

cudaError_t launch_merge_shards_strided(const float* keys, int64_t key_stride, const int64_t* ids,
                                        int64_t id_stride, int nshard, int64_t nq, int k, bool l2, bool natural,
                                        float* out_dists, int64_t* out_ids, cudaStream_t stream) {
  if (nq == 0 || k == 0) return cudaSuccess;
  if (nshard < 1 || nshard > 8) return cudaErrorInvalidValue;
  const int threads = 128;
  merge_shards_kernel<<<static_cast<unsigned>((nq + threads - 1) / threads), threads, 0, stream>>>(
      reinterpret_cast<const char*>(keys), key_stride, reinterpret_cast<const char*>(ids), id_stride, nshard, nq,
      k, l2, natural, out_dists, out_ids);
  return cudaGetLastError();
}

}  // namespace px
