// K5: exact rescoring and certification of tensor-core candidates.
//
// Input: per query the CAP best candidates by the approximate key of the
// tensor-core pass, merged over all splits and sorted. Each candidate is
// rescored with the reference's exact arithmetic (distance.rs:4-39 via
// exact_key), the CAP exact keys are ranked (ties by row), and the first k
// are the answer -- provided no row outside the candidate set can beat the
// k-th. That is certified with a rigorous bound eps on |approx - exact|:
//   every non-candidate x has approx(x) >= A, the largest approximate key
//   among the candidates, hence exact(x) >= A - eps; the result is exact if
//   exact_k < A - eps (strict, so no outside row can even tie).
// A query whose certificate fails is listed for the exact streaming scan.
//
// eps is a worst-case bound, in double precision, built from
//   S = ||q|| * max_x ||x|| >= sum_i |q_i x_i|        (Cauchy-Schwarz)
// the representation error of the pass's operands (zero when they are exact:
// (2^-8 + 2^-18) * S for bf16 copies, (2^-10 + 2^-22) * S for tf32 hi values
// alone, 4 * 2^-22 * S for the three-pass tf32 sum), an allowance of
// 2 * 2^-22 * S per tensor-core accumulation step (one per 8 values of K and
// pass), and the rounding of the reference arithmetic and of the norms.
// An L2 pass with folded norms accumulates 2 q.x - ||x||^2 (the norm as three
// exact bf16 values in the rows' padding): the same terms doubled, so the
// same bound on the key, plus the per-step allowance on the norm's share of
// the partial sums, 2 * 2^-22 * max ||x||^2 per step, over three more K
// values. Magnitudes near the exponent range (where the bf16 pieces or the
// partial sums could overflow) are never certified.
#include "px_common.cuh"
#include "px_kernels.h"

namespace px {

namespace {

constexpr int kRescoreWarps = 4;
constexpr int kMaxCands = 256;

template <bool L2>
__global__ void __launch_bounds__(kRescoreWarps * 32)
rescore_kernel(const RescoreArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dq = (a.d + 3) & ~3;
  float* s_q = reinterpret_cast<float*>(smem_raw) + warp * dq;
  uint64_t* s_c = reinterpret_cast<uint64_t*>(reinterpret_cast<float*>(smem_raw) + kRescoreWarps * dq) +
                  warp * 2 * kMaxCands;
  uint64_t* s_sorted = s_c + kMaxCands;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * kRescoreWarps + warp;
  if (q >= a.nq) return;

  const float* qv = a.queries + q * a.d;
  double qsq = 0.0;
  for (int i = lane; i < a.d; i += 32) {
    const float v = qv[i];
    s_q[i] = v;
    qsq += static_cast<double>(v) * v;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) qsq += __shfl_xor_sync(0xffffffffu, qsq, off);
  __syncwarp();

  // Exact keys, four candidates at a time: thread l of a group of eight runs
  // the reference's lane-l accumulator (acc_l += term(x[8c + l], q[8c + l]),
  // c = 0, 1, ...) on its own, so each accumulator is the same sequential
  // chain as the reference's, and the group reads 32 contiguous bytes of the
  // row per step. The lanes are then summed left to right and the remainder
  // added, as distance.rs does.
  const uint64_t* mq = a.merged + q * a.cap;
  const int grp = lane >> 3, l = lane & 7, g0 = lane & ~7;
  const int chunks = a.d >> 3;
  for (int j0 = 0; j0 < a.cap; j0 += 4) {
    const int j = j0 + grp;
    const uint64_t c = j < a.cap ? mq[j] : PX_EMPTY;
    const bool valid = c != PX_EMPTY;
    const uint32_t row = valid ? cand_row(c) : 0u;
    const float* x = a.base + static_cast<int64_t>(row) * a.ld;
    float acc = 0.f;
    if (valid) {
#pragma unroll 4
      for (int cc = 0; cc < chunks; ++cc) acc = __fadd_rn(acc, lane_term<L2>(s_q[cc * 8 + l], x[cc * 8 + l]));
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
  }
  __syncwarp();
  // Rank sort (values are distinct except PX_EMPTY; equal ones rank by index).
  for (int j = lane; j < a.cap; j += 32) {
    const uint64_t v = s_c[j];
    int rank = 0;
    for (int i = 0; i < a.cap; ++i) {
      const uint64_t u = s_c[i];
      rank += (u < v) || (u == v && i < j);
    }
    s_sorted[rank] = v;
  }
  __syncwarp();

  // Certificate. Every row outside the candidate set has an approximate key
  // >= min(A_cap, max of every full split list): when the per-split lists
  // are shorter than the merged set, a split can hide rows below A_cap.
  int ok = 1;
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
  const uint64_t kth = s_sorted[a.k - 1];
  if (last != PX_EMPTY && kth == PX_EMPTY) {
    // Fewer than k candidates, yet a full list may hide rows: not certified.
    ok = 0;
  } else if (last != PX_EMPTY) {
    const double qn = sqrt(qsq);
    const double xn = static_cast<double>(a.max_norm);
    const bool q_lo = *a.q_lo_flag != 0;
    int npass = 1;
    double rep = 0.0;  // representation error per product, relative to |q_i x_i|
    if (a.pass_kind == kPassBf16) {
      // Each bf16 value is within 2^-9 of its fp32 value: (1 + 2^-9)^2 - 1.
      if (*a.q_bf_flag != 0 || a.x_bf_inexact) rep = 0x1p-8 + 0x1p-18;
    } else if (q_lo || a.x_lo_nonzero) {
      if (a.pass_kind == kPassTf32) {
        // hi x hi alone: each hi is within 2^-11 of its value.
        rep = 0x1p-10 + 0x1p-22;
      } else {
        // Three-pass sum: the dropped lo x lo term and the tf32 rounding of
        // each lo.
        npass = 1 + (q_lo ? 1 : 0) + (a.x_lo_nonzero ? 1 : 0);
        rep = 4.0 * 0x1p-22;
      }
    }
    const int dk = a.norm_folded ? a.d + 3 : a.d;  // K values with nonzero products
    const double steps = static_cast<double>(npass) * ((dk + 7) / 8) + 2.0;
    const double S = qn * xn;
    const double e_dot = S * (rep + 2.0 * steps * 0x1p-22);
    const double ref = (a.d / 8 + 10) * 0x1p-23;
    const double A = static_cast<double>(cand_key(last));
    const double Ek = static_cast<double>(cand_key(kth));
    double bound;
    if (L2) {
      const double qn2 = qn * qn;
      double eps = 2.0 * e_dot + xn * xn * ref + (qn + xn) * (qn + xn) * ref + (fabs(A) + qn2) * 0x1p-22;
      if (a.norm_folded) eps += 2.0 * steps * 0x1p-22 * xn * xn + 0x1p-120;
      bound = A + qn2 - eps;
    } else {
      const double eps = e_dot + S * ref + fabs(A) * 0x1p-22;
      bound = A - eps;
    }
    ok = (Ek < bound && S < 0x1p100 && xn * xn < 0x1p100) ? 1 : 0;
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
  const size_t smem = sizeof(float) * kRescoreWarps * dq + sizeof(uint64_t) * kRescoreWarps * 2 * kMaxCands;
  const unsigned blocks = static_cast<unsigned>((a.nq + kRescoreWarps - 1) / kRescoreWarps);
  if (a.l2) {
    cudaError_t e = cudaFuncSetAttribute(rescore_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    rescore_kernel<true><<<blocks, kRescoreWarps * 32, smem, stream>>>(a);
  } else {
    cudaError_t e = cudaFuncSetAttribute(rescore_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    rescore_kernel<false><<<blocks, kRescoreWarps * 32, smem, stream>>>(a);
  }
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
