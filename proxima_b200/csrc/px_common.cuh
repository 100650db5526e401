// Shared device helpers for the proxima_b200 kernels.
//
// Candidate encoding. Every top-k list on the device holds 64-bit words
//   cand = (total_order(key) << 32) | local_row
// where total_order maps an f32 key to a u32 whose unsigned order is exactly
// f32::total_cmp (the order the reference's Cand uses: flat.rs:28-31,
// pq.rs:211-215). Unsigned compares of cand therefore order by key first and,
// for equal keys, by row -- the tie rule of this library (smaller id first).
// An empty slot holds PX_EMPTY (all ones), larger than any real candidate.
#pragma once

#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

#define PX_EMPTY 0xFFFFFFFFFFFFFFFFull

namespace px {

__host__ __device__ __forceinline__ uint32_t f2u(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  return b;
}

__host__ __device__ __forceinline__ float u2f(uint32_t b) {
  float x;
  memcpy(&x, &b, 4);
  return x;
}

__host__ __device__ __forceinline__ uint32_t key_to_ord(float key) {
  uint32_t b = f2u(key);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__host__ __device__ __forceinline__ float ord_to_key(uint32_t o) {
  uint32_t b = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
  return u2f(b);
}

__host__ __device__ __forceinline__ uint64_t pack_cand(float key, uint32_t row) {
  return (static_cast<uint64_t>(key_to_ord(key)) << 32) | row;
}

__host__ __device__ __forceinline__ float cand_key(uint64_t c) {
  return ord_to_key(static_cast<uint32_t>(c >> 32));
}

__host__ __device__ __forceinline__ uint32_t cand_row(uint64_t c) {
  return static_cast<uint32_t>(c & 0xFFFFFFFFu);
}

// x rounded to tf32 (10 stored mantissa bits), to nearest with ties away from
// zero: the hi part of the three-pass split.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Natural distance reported to callers (flat.rs:142, 146; pq.rs:335-345).
__device__ __forceinline__ float natural_dist(float key, bool l2) {
  return l2 ? __fsqrt_rn(key) : -key;
}

__device__ __forceinline__ float pad_dist(bool l2) {
  return l2 ? 3.40282347e+38f : -3.40282347e+38f;
}

// Exact reference arithmetic (distance.rs:4-39): 8 lane accumulators, each a
// rounded multiply then a rounded add (no FMA contraction), lanes summed left
// to right, then the remainder. The intrinsics pin every rounding so nvcc's
// default --fmad=true cannot contract them.
template <bool L2>
__device__ __forceinline__ float lane_term(float a, float b) {
  if (L2) {
    float d = __fsub_rn(a, b);
    return __fmul_rn(d, d);
  } else {
    return __fmul_rn(a, b);
  }
}

// Full exact key of (q, x) over `len` elements read from generic pointers.
template <bool L2>
__device__ __forceinline__ float exact_dot_or_l2(const float* __restrict__ q,
                                                 const float* __restrict__ x, int len) {
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const int chunks = len >> 3;
  for (int c = 0; c < chunks; ++c) {
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[l] = __fadd_rn(acc[l], lane_term<L2>(q[c * 8 + l], x[c * 8 + l]));
  }
  float s = acc[0];
#pragma unroll
  for (int l = 1; l < 8; ++l) s = __fadd_rn(s, acc[l]);
  for (int i = chunks * 8; i < len; ++i) s = __fadd_rn(s, lane_term<L2>(q[i], x[i]));
  return s;
}

// Key as FlatIndex::scan forms it: squared L2, or the negated inner product.
template <bool L2>
__device__ __forceinline__ float exact_key(const float* __restrict__ q, const float* __restrict__ x,
                                           int len) {
  float s = exact_dot_or_l2<L2>(q, x, len);
  return L2 ? s : -s;
}

__device__ __forceinline__ float4 ldg_stream4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

// In-place ascending bitonic sort of `count` segments of `seg` u64 words each
// (seg a power of two), cooperatively by all `nthreads` threads of the block.
// Caller synchronises before and after.
__device__ __forceinline__ void block_bitonic_sort(uint64_t* data, int seg, int count, int tid,
                                                   int nthreads) {
  const int half = seg >> 1;
  const int total_pairs = half * count;
  for (int size = 2; size <= seg; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int p = tid; p < total_pairs; p += nthreads) {
        const int s = p / half;
        const int e = p - s * half;
        const int lo = 2 * stride * (e / stride) + (e % stride);
        const int hi = lo + stride;
        uint64_t* base = data + static_cast<size_t>(s) * seg;
        const bool up = (lo & size) == 0;
        uint64_t a = base[lo], b = base[hi];
        if ((a > b) == up) {
          base[lo] = b;
          base[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

// Block-level top-k over G independent candidate streams (one per query).
//
// Threads offer packed candidates; a candidate is kept only if it beats the
// stream's current threshold (the k-th best seen at the last compaction).
// Kept candidates are appended to a per-stream buffer of BUF words with one
// shared-memory atomic. The owner calls `maybe_compact` once per iteration
// (all threads, after a __syncthreads) with `reserve` = the most candidates
// one iteration can append per stream; a buffer whose fill could overflow in
// the next iteration is sorted and cut back to its k best, which also
// tightens the threshold. `compact_all` sorts every buffer so that its first
// k words are the stream's top-k (PX_EMPTY-padded).
template <int G, int BUF>
struct BlockTopK {
  uint64_t* buf;  // [G][BUF]
  int* cnt;       // [G]
  uint64_t* thr;  // [G]

  __device__ void init(uint64_t* smem_buf, int* smem_cnt, uint64_t* smem_thr, int tid, int nthreads) {
    buf = smem_buf;
    cnt = smem_cnt;
    thr = smem_thr;
    for (int i = tid; i < G; i += nthreads) {
      cnt[i] = 0;
      thr[i] = PX_EMPTY;
    }
  }

  __device__ __forceinline__ void offer(int g, uint64_t cand, uint64_t threshold) {
    if (cand < threshold) {
      int p = atomicAdd(&cnt[g], 1);
      buf[g * BUF + p] = cand;
    }
  }

  // k <= 32: warp w keeps stream w's k best in ascending order, with k rounds
  // of a warp-wide minimum over the entries at or above `lo`, where lo is one
  // past the last word taken. A stream's words are distinct (each row is
  // offered to a stream once), so the rounds take the k smallest in order.
  // About k*cnt/32 shared loads per lane, against a full bitonic sort of BUF
  // words per stream. Used for buffers of 1024 words and more; on smaller
  // ones the block-wide sort is shorter than one warp's serial rounds.
  __device__ void select_small(int k, int tid, int nthreads) {
    const int lane = tid & 31;
    for (int g = tid >> 5; g < G; g += nthreads >> 5) {
      uint64_t* b = buf + g * BUF;
      const int n = cnt[g];
      uint64_t mine = PX_EMPTY;  // lane r ends holding the r-th smallest
      uint64_t lo = 0;
      for (int r = 0; r < k; ++r) {
        uint64_t m = PX_EMPTY;
        for (int e = lane; e < n; e += 32) {
          const uint64_t v = b[e];
          if (v >= lo && v < m) m = v;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const uint64_t x = __shfl_xor_sync(0xffffffffu, m, o);
          m = x < m ? x : m;
        }
        if (lane == r) mine = m;
        if (m == PX_EMPTY) break;  // warp-uniform: fewer than k entries
        lo = m + 1;
      }
      const uint64_t kth = __shfl_sync(0xffffffffu, mine, k - 1);
      __syncwarp();
      if (lane < k) b[lane] = mine;
      if (lane == 0) {
        const int c = n < k ? n : k;
        cnt[g] = c;
        thr[g] = (c == k) ? kth : PX_EMPTY;
      }
    }
    __syncthreads();
  }

  // Sorts every stream's buffer and keeps its k best. All threads.
  __device__ void compact_all(int k, int tid, int nthreads) {
    if (BUF >= 1024 && k <= 32) {
      select_small(k, tid, nthreads);
      return;
    }
    for (int i = tid; i < G * BUF; i += nthreads) {
      int g = i / BUF, e = i - g * BUF;
      if (e >= cnt[g]) buf[i] = PX_EMPTY;
    }
    __syncthreads();
    block_bitonic_sort(buf, BUF, G, tid, nthreads);
    for (int g = tid; g < G; g += nthreads) {
      int c = cnt[g] < k ? cnt[g] : k;
      cnt[g] = c;
      thr[g] = (c == k) ? buf[g * BUF + k - 1] : PX_EMPTY;
    }
    __syncthreads();
  }

  // All threads; call after a __syncthreads that follows the offers.
  __device__ void maybe_compact(int k, int reserve, int tid, int nthreads) {
    bool need = false;
#pragma unroll
    for (int g = 0; g < G; ++g) need |= cnt[g] > BUF - reserve;
    __syncthreads();  // every thread has read cnt before compact_all rewrites it
    if (need) compact_all(k, tid, nthreads);
  }
};

}  // namespace px
