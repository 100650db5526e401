// K5: exact rescoring and certification of tensor-core candidates.
//
// Input: per query the CAP best candidates by the approximate key of the
// tensor-core pass, merged over all splits and sorted. Each candidate is
// rescored with the reference's exact arithmetic (distance.rs:4-39 via
// exact_key), the CAP exact keys are ranked (ties by row), and the first k
// are the answer -- provided no row outside the candidate set can beat the
// k-th. That is certified with a rigorous bound eps on |approx - exact|:
//   every non-candidate x has approx(x) >= A, the largest approximate key
//   among the candidates (or less: the largest key of a full split list, or
//   the starting threshold of a seeded pass), hence exact(x) >= A - eps; the
//   result is exact if exact_k < A - eps (strict, so no outside row can even
//   tie).
// A query whose certificate fails is listed for the exact streaming scan.
//
// eps is a worst-case bound, evaluated in double precision, with three parts.
//
// 1. Representation. The pass multiplies rounded copies q~, x~ of the query
//    and the rows. Exactly, q.x - q~.x~ = (q - q~).x + q~.(x - x~), so by
//    Cauchy-Schwarz
//        |q.x - q~.x~| <= ||q - q~|| * max||x|| + ||q~|| * max||x - x~||.
//    The query terms are computed here from the query itself (with the same
//    rounding the conversion kernel applies: bf16 round-to-nearest-even, or
//    tf32 round-to-nearest-away); max||x - x~|| is an upper bound the shard
//    build keeps (k_prep.cu). Both are zero for data exact in the pass's
//    format (e.g. small integers). For the three-pass tf32 sum
//    qh.xh + qh.xl + ql.xh the dropped terms are qh.rx + ql.(x - xh) + rq.x
//    (rx, rq: the tf32 rounding of the lo parts), each at most
//    2^-22 * sum|q_i x_i| (+ 2^-33), so 4 * 2^-22 * S bounds them, with
//    S = ||q|| * max||x|| >= sum|q_i x_i|.
// 2. Accumulation. The tensor core's products of bf16 or tf32 values are
//    exact in fp32. The sums are modelled as any sequence of steps, each
//    adding c >= 1 products to the fp32 accumulator with every operand
//    aligned to the largest one and cut to 24 significant bits (at most one
//    unit in the last place of the largest operand lost per operand), then
//    the sum rounded or cut to 24 bits (another unit). Every operand and
//    partial sum is at most M = sum of the magnitudes of all products, so a
//    step loses at most (c + 2) * 2^-23 * M, i.e. at most 3 * 2^-23 * M per
//    product whatever the hardware's grouping: the model assumes only that
//    no operand keeps fewer than 24 bits relative to the largest operand of
//    its step. M = S (x 1.01 for the rounded copies' own growth); a folded L2
//    pass accumulates 2 q~.x~ - ||x||^2 (its norm as three exact bf16 values
//    in the rows' padding), so M = 2.02 S + max||x||^2 there. Products that
//    underflow fp32 add at most 2^-120 * (1 + ||q|| + max||x||) each.
// 3. Reference and epilogue rounding: the reference key's own fp32 rounding
//    (8-lane order, relative (d/8 + 10) * 2^-23 of the sum of the terms'
//    magnitudes), the fp32 row norms, and the epilogue's rounding of the
//    approximate key (|A| * 2^-22).
// Magnitudes near the exponent range (where the bf16 pieces or the partial
// sums could overflow) are never certified.
#include <cuda_bf16.h>

#include "px_common.cuh"
#include "px_kernels.h"

namespace px {

namespace {

constexpr int kRescoreWarps = 4;
constexpr int kMaxCands = 256;
// Candidate rows staged per warp and round: as many as fit in ~16 KB, a
// multiple of four between 4 and 16 (one 4-candidate step per 8-lane group).
// Rows too long for 8 of them (d > 480) are not staged: four rows per round
// is what the direct loads already keep in flight, and the staging area
// would only cut the warps per SM.
constexpr int kRowStageBytes = 16 * 1024;

// Floats per staged row: d rounded up to 32, plus 8, so the four rows of a
// step start in four different 8-bank slices.
__host__ __device__ __forceinline__ int staged_row_floats(int d) { return ((d + 31) & ~31) + 8; }
__host__ __device__ __forceinline__ int staged_rows(int d) {
  const int g = (kRowStageBytes / (4 * staged_row_floats(d))) & ~3;
  return g < 4 ? 4 : (g > 16 ? 16 : g);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// STAGE: candidate rows go through shared memory (below); otherwise (rows too
// long for it) each lane fetches kBatch of its elements before adding them.
template <bool L2, bool STAGE>
__global__ void __launch_bounds__(kRescoreWarps * 32)
rescore_kernel(const RescoreArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dq = (a.d + 3) & ~3;
  float* s_q = reinterpret_cast<float*>(smem_raw) + warp * dq;
  uint64_t* s_c = reinterpret_cast<uint64_t*>(reinterpret_cast<float*>(smem_raw) + kRescoreWarps * dq) +
                  warp * 2 * kMaxCands;
  uint64_t* s_sorted = s_c + kMaxCands;
  const int ds = staged_row_floats(a.d);
  const int G = STAGE ? staged_rows(a.d) : 4;
  float* s_rows = reinterpret_cast<float*>(reinterpret_cast<uint64_t*>(reinterpret_cast<float*>(smem_raw) +
                                                                       kRescoreWarps * dq) +
                                           kRescoreWarps * 2 * kMaxCands) +
                  static_cast<size_t>(warp) * G * ds;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * kRescoreWarps + warp;
  if (q >= a.nq) return;

  const float* qv = a.queries + q * a.d;
  // ||q||^2, and for a bf16 or tf32 pass ||q' - q'~||^2 and ||q'~||^2, where
  // q' is what the query conversion rounds (2q for a folded L2 pass; the
  // doubling is exact) and q'~ its rounding. Squares of fp32 values and of
  // their exact rounding residuals are exact in double.
  const bool folded = a.norm_folded != 0;
  double qsq = 0.0, rq2 = 0.0, qt2 = 0.0;
  for (int i = lane; i < a.d; i += 32) {
    const float v = qv[i];
    s_q[i] = v;
    qsq += static_cast<double>(v) * v;
    const float u = folded ? __fmul_rn(2.0f, v) : v;
    float t = u;
    if (a.pass_kind == kPassBf16) t = __bfloat162float(__float2bfloat16_rn(u));
    else if (a.pass_kind == kPassTf32) t = tf32_rna(u);
    const double r = static_cast<double>(__fsub_rn(u, t));
    rq2 += r * r;
    qt2 += static_cast<double>(t) * t;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    qsq += __shfl_xor_sync(0xffffffffu, qsq, off);
    rq2 += __shfl_xor_sync(0xffffffffu, rq2, off);
    qt2 += __shfl_xor_sync(0xffffffffu, qt2, off);
  }
  __syncwarp();

  // The certificate's bound. lower_bound(a) is, in the reference's key space,
  // a lower bound on the exact key of every row whose approximate key is >= a
  // (eps as in the header; increasing in a).
  const double ref = (a.d / 8 + 10) * 0x1p-23;  // the reference's relative rounding
  const double qn = sqrt(qsq) * (1.0 + 0x1p-40);
  // Upper bound on every row's real norm: the shard keeps the largest fp32
  // norm, itself rounded in the reference's order.
  const double xn2 = static_cast<double>(a.max_norm_sq) * (1.0 + ref);
  const double xn = sqrt(xn2) * (1.0 + 0x1p-40);
  const double S = qn * xn;
  const bool q_lo = *a.q_lo_flag != 0;
  int npass = 1;
  double e_rep = 0.0;  // bound on |q'.x - (the pass's product of the rounded copies)|
  if (a.pass_kind == kPassBf16 || a.pass_kind == kPassTf32) {
    e_rep = (sqrt(rq2) * xn + sqrt(qt2) * static_cast<double>(a.x_resid)) * (1.0 + 0x1p-40);
  } else if (q_lo || a.x_lo_nonzero) {
    npass = 1 + (q_lo ? 1 : 0) + (a.x_lo_nonzero ? 1 : 0);
    e_rep = 4.0 * 0x1p-22 * S;
  }
  const int dk = folded ? a.d + 3 : a.d;  // K values with nonzero products
  const double products = static_cast<double>(npass) * dk + 2.0;
  const double M = folded ? 2.02 * S + xn2 : 1.01 * S;
  const double e_acc = 3.0 * 0x1p-23 * products * M + products * (1.0 + qn + xn) * 0x1p-120;
  const double qn2 = qn * qn;
  // Folded L2: the pass's key is -(2q~.x~ - ||x||^2) and e_rep already bounds
  // the doubled product; other L2 passes compute ||x||^2 - 2 q~.x~.
  const double e_fixed = L2 ? (folded ? e_rep + e_acc : 2.0 * (e_rep + e_acc)) + xn2 * ref +
                                  (qn + xn) * (qn + xn) * ref
                            : e_rep + e_acc + S * ref;
  const bool in_range = S < 0x1p100 && xn2 < 0x1p100;
  auto lower_bound = [&](double akey) {
    return L2 ? akey + qn2 - (e_fixed + (fabs(akey) + qn2) * 0x1p-22) : akey - (e_fixed + fabs(akey) * 0x1p-22);
  };

  // Every row outside the candidate set has an approximate key >=
  // min(A_cap, max of every full split list): when the per-split lists are
  // shorter than the merged set, a split can hide rows below A_cap.
  const uint64_t* mq = a.merged + q * a.cap;
  uint64_t last = mq[a.cap - 1];
  if (a.list_cap < a.cap) {
    uint64_t m = PX_EMPTY;
    const uint64_t* ql = a.lists + q * static_cast<int64_t>(a.nlists) * a.list_cap;
    for (int j = lane; j < a.nlists; j += 32) {
      const uint64_t lmax = ql[static_cast<int64_t>(j) * a.list_cap + a.list_cap - 1];
      m = lmax < m ? lmax : m;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const uint64_t o = __shfl_xor_sync(0xffffffffu, m, off);
      m = o < m ? o : m;
    }
    last = m < last ? m : last;
  }
  // A seeded pass admitted only keys <= its starting threshold: every row it
  // left out has a larger approximate key.
  if (a.seed != nullptr) {
    const uint64_t s = a.seed[q * a.seed_k + a.seed_k - 1];
    last = s < last ? s : last;
  }

  // Exact keys, four candidates at a time, in approximate-key order: thread l
  // of a group of eight runs the reference's lane-l accumulator
  // (acc_l += term(x[8c + l], q[8c + l]), c = 0, 1, ...) on its own, so each
  // accumulator is the same sequential chain as the reference's, and the
  // group reads 32 contiguous bytes of the row per step. The lanes are then
  // summed left to right and the remainder added, as distance.rs does.
  // The rows are random gathers: G of them at a time are copied to shared
  // memory with every 16-byte piece in flight at once (one memory latency
  // per G candidates instead of one per four), and the chains read them
  // there.
  // Early exit: once `done` candidates are scored, every unscored candidate
  // and every row outside the set has an approximate key >= a* = min(the
  // next candidate's, last), hence an exact key >= lower_bound(a*). If k
  // scored keys lie strictly below that, no other row can reach the top k
  // (not even tie), so the top k of the scored ones is the answer, certified.
  const int grp = lane >> 3, l = lane & 7, g0 = lane & ~7;
  const int chunks = a.d >> 3;
  int scored = a.cap;
  bool early = false;
  const int pieces = (a.d + 3) >> 2;  // 16-byte pieces per row (rows are 128-byte aligned, ld >= d rounded to 32)
  const uint32_t rows_addr = static_cast<uint32_t>(__cvta_generic_to_shared(s_rows));
  for (int j0 = 0; j0 < a.cap; j0 += 4) {
    if (STAGE && j0 % G == 0) {
      // Stage candidates j0 .. j0 + G - 1 (the ones that exist).
      __syncwarp();  // the previous group's rows are no longer read
      for (int i = lane; i < G * pieces; i += 32) {
        const int r = i / pieces, pc = i - r * pieces;
        const int jr = j0 + r;
        const uint64_t cr = jr < a.cap ? mq[jr] : PX_EMPTY;
        if (cr != PX_EMPTY)
          cp_async16(rows_addr + static_cast<uint32_t>((r * ds + pc * 4) * 4),
                     a.base + static_cast<int64_t>(cand_row(cr)) * a.ld + pc * 4);
      }
      cp_async_wait_all();
      __syncwarp();
    }
    const int j = j0 + grp;
    const uint64_t c = j < a.cap ? mq[j] : PX_EMPTY;
    const bool valid = c != PX_EMPTY;
    const uint32_t row = valid ? cand_row(c) : 0u;
    const float* x = STAGE ? s_rows + (j % G) * ds : a.base + static_cast<int64_t>(row) * a.ld;
    float acc = 0.f;
    if (valid) {
      if constexpr (STAGE) {
#pragma unroll 8
        for (int cc = 0; cc < chunks; ++cc) acc = __fadd_rn(acc, lane_term<L2>(s_q[cc * 8 + l], x[cc * 8 + l]));
      } else {
        constexpr int kBatch = 48;
        for (int c0 = 0; c0 < chunks; c0 += kBatch) {
          float xv[kBatch];
#pragma unroll
          for (int b = 0; b < kBatch; ++b) xv[b] = c0 + b < chunks ? __ldg(x + (c0 + b) * 8 + l) : 0.f;
#pragma unroll
          for (int b = 0; b < kBatch; ++b)
            if (c0 + b < chunks) acc = __fadd_rn(acc, lane_term<L2>(s_q[(c0 + b) * 8 + l], xv[b]));
        }
      }
    }
    float sum = __shfl_sync(0xffffffffu, acc, g0);
#pragma unroll
    for (int m = 1; m < 8; ++m) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, acc, g0 + m));
    if (l == 0 && j < a.cap) {
      uint64_t e = PX_EMPTY;
      if (valid) {
        for (int i = chunks * 8; i < a.d; ++i) sum = __fadd_rn(sum, lane_term<L2>(s_q[i], x[i]));
        e = pack_cand(L2 ? sum : -sum, row);
      }
      s_c[j] = e;
    }
    __syncwarp();
    const int done = j0 + 4;
    if (done >= a.k && done < a.cap && in_range) {
      const uint64_t next = mq[done];
      if (next == PX_EMPTY) {  // the rest of the merged list is empty
        scored = done;
        break;
      }
      const uint64_t astar = next < last ? next : last;
      const double T = lower_bound(static_cast<double>(cand_key(astar)));
      int below = 0;
      for (int i = lane; i < done; i += 32)
        below += (s_c[i] != PX_EMPTY && static_cast<double>(cand_key(s_c[i])) < T) ? 1 : 0;
      if (__reduce_add_sync(0xffffffffu, below) >= a.k) {
        scored = done;
        early = true;
        break;
      }
    }
  }
  __syncwarp();
  // Rank sort of the scored candidates (values are distinct except PX_EMPTY;
  // equal ones rank by index).
  for (int j = lane; j < scored; j += 32) {
    const uint64_t v = s_c[j];
    int rank = 0;
    for (int i = 0; i < scored; ++i) {
      const uint64_t u = s_c[i];
      rank += (u < v) || (u == v && i < j);
    }
    s_sorted[rank] = v;
  }
  __syncwarp();

  int ok = 1;
  if (!early) {
    const uint64_t kth = s_sorted[a.k - 1];
    if (last != PX_EMPTY && kth == PX_EMPTY) {
      // Fewer than k candidates, yet a full list may hide rows: not certified.
      ok = 0;
    } else if (last != PX_EMPTY) {
      const double bound = lower_bound(static_cast<double>(cand_key(last)));
      ok = (static_cast<double>(cand_key(kth)) < bound && in_range) ? 1 : 0;
    }
  }
  for (int j = lane; j < a.k; j += 32) a.out[q * a.k + j] = s_sorted[j];
  if (lane == 0) {
    a.status[q] = ok ? 0 : 1;
    if (!ok) {
      const int pos = atomicAdd(a.n_fail, 1);
      a.fail_list[pos] = static_cast<int>(q);
    }
  }
}

__global__ void gather_rows_kernel(const float* __restrict__ src, int d, const int* __restrict__ idx,
                                   int count, float* __restrict__ dst) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(count) * d) return;
  const int r = static_cast<int>(i / d), e = static_cast<int>(i - static_cast<int64_t>(r) * d);
  dst[i] = src[static_cast<int64_t>(idx[r]) * d + e];
}

__global__ void scatter_cands_kernel(const uint64_t* __restrict__ src, int k, const int* __restrict__ idx,
                                     int count, uint64_t* __restrict__ dst) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(count) * k) return;
  const int r = static_cast<int>(i / k), j = static_cast<int>(i - static_cast<int64_t>(r) * k);
  dst[static_cast<int64_t>(idx[r]) * k + j] = src[i];
}

}  // namespace

cudaError_t launch_rescore(const RescoreArgs& a, cudaStream_t stream) {
  if (a.nq == 0) return cudaSuccess;
  if (a.cap > kMaxCands || a.k > a.cap) return cudaErrorInvalidValue;
  const int dq = (a.d + 3) & ~3;
  const size_t base_smem = sizeof(float) * kRescoreWarps * dq + sizeof(uint64_t) * kRescoreWarps * 2 * kMaxCands;
  const size_t staged_smem =
      base_smem + sizeof(float) * kRescoreWarps * staged_rows(a.d) * staged_row_floats(a.d);
  // Rows are staged in 16-byte pieces (ld a multiple of 4, the base 16-byte
  // aligned), when the staged rows fit.
  const bool stage = a.ld % 4 == 0 && reinterpret_cast<uintptr_t>(a.base) % 16 == 0 && staged_rows(a.d) >= 8 &&
                     staged_smem <= 200 * 1024;
  const size_t smem = stage ? staged_smem : base_smem;
  const unsigned blocks = static_cast<unsigned>((a.nq + kRescoreWarps - 1) / kRescoreWarps);
  auto kern = a.l2 ? (stage ? rescore_kernel<true, true> : rescore_kernel<true, false>)
                   : (stage ? rescore_kernel<false, true> : rescore_kernel<false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  kern<<<blocks, kRescoreWarps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const float* src, int d, const int* idx, int count, float* dst,
                               cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(count) * d;
  if (total == 0) return cudaSuccess;
  gather_rows_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(src, d, idx, count, dst);
  return cudaGetLastError();
}

cudaError_t launch_scatter_cands(const uint64_t* src, int k, const int* idx, int count, uint64_t* dst,
                                 cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(count) * k;
  if (total == 0) return cudaSuccess;
  scatter_cands_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(src, k, idx, count, dst);
  return cudaGetLastError();
}

}  // namespace px
