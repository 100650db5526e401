// K2: exact streaming scan for small query batches.
//
// Restates FlatIndex::scan (crates/core/src/flat.rs:106-148) on the device:
// every key is computed in the reference's exact arithmetic
// (distance.rs:4-39), so the keys are bit-identical to the CPU's and the
// top-k needs no rescoring. The kernel streams the shard once per group of G
// queries with 128-bit loads, which makes it HBM-bound for G <= 2 and
// FP32-issue-bound above that.
//
// Thread mapping: two threads per base row. Thread half h of row r reads
// lanes 4h..4h+3 of every 8-float chunk (one float4 per chunk), so a warp
// reads 16 rows x 32 contiguous bytes per load -- whole 32-byte sectors --
// and each thread owns four of the reference's eight lane accumulators.
// After the chunk loop the pair combines its lanes in the reference's left
// to right order through one shuffle exchange.
#include "px_common.cuh"
#include "px_kernels.h"

namespace px {

namespace {

constexpr int kExactThreads = 256;
constexpr int kRowsPerIter = kExactThreads / 2;

template <int G, int BUF, bool L2>
__global__ void __launch_bounds__(kExactThreads)
exact_scan_kernel(const float* __restrict__ base, int64_t n, int ld, int d,
                  const float* __restrict__ queries, int dq, int nq, int k, int64_t rows_per_cta,
                  const uint8_t* __restrict__ mask, uint64_t* __restrict__ partial) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* s_buf = reinterpret_cast<uint64_t*>(smem_raw);            // G*BUF
  uint64_t* s_thr = s_buf + G * BUF;  // G words, padded to an even count                                  // G
  int* s_cnt = reinterpret_cast<int*>(s_thr + ((G + 1) & ~1));                     // G
  float* s_q = reinterpret_cast<float*>(s_cnt + ((G + 3) & ~3));      // G*dq, 16B aligned

  const int tid = threadIdx.x;
  const int q0 = blockIdx.y * G;
  const int gcount = min(G, nq - q0);

  BlockTopK<G, BUF> topk;
  topk.init(s_buf, s_cnt, s_thr, tid, kExactThreads);
  for (int i = tid; i < G * dq; i += kExactThreads) {
    int g = i / dq, e = i - g * dq;
    s_q[i] = (g < gcount && e < d) ? queries[static_cast<int64_t>(q0 + g) * d + e] : 0.f;
  }
  __syncthreads();

  const int64_t row_begin = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
  const int64_t row_end = min(n, row_begin + rows_per_cta);
  const int half = tid & 1;
  const int chunks = d >> 3;
  const int rem_begin = chunks * 8;

  uint64_t thr[G];
#pragma unroll
  for (int g = 0; g < G; ++g) thr[g] = PX_EMPTY;

  for (int64_t it = row_begin; it < row_end; it += kRowsPerIter) {
    const int64_t r = it + (tid >> 1);
    const bool valid = r < row_end && (mask == nullptr || mask[r] != 0);
    float acc[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[g][i] = 0.f;

    if (valid) {
      const float* xrow = base + r * ld + half * 4;
      const float* qh = s_q + half * 4;
#pragma unroll 8  // eight 16-byte loads in flight per thread
      for (int c = 0; c < chunks; ++c) {
        float4 x = ldg_stream4(xrow + c * 8);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float4 q = *reinterpret_cast<const float4*>(qh + g * dq + c * 8);
          acc[g][0] = __fadd_rn(acc[g][0], lane_term<L2>(q.x, x.x));
          acc[g][1] = __fadd_rn(acc[g][1], lane_term<L2>(q.y, x.y));
          acc[g][2] = __fadd_rn(acc[g][2], lane_term<L2>(q.z, x.z));
          acc[g][3] = __fadd_rn(acc[g][3], lane_term<L2>(q.w, x.w));
        }
      }
    }
    // Lanes 4..7 live in the partner thread; fold them in the reference order.
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float p0 = __shfl_xor_sync(0xffffffffu, acc[g][0], 1);
      float p1 = __shfl_xor_sync(0xffffffffu, acc[g][1], 1);
      float p2 = __shfl_xor_sync(0xffffffffu, acc[g][2], 1);
      float p3 = __shfl_xor_sync(0xffffffffu, acc[g][3], 1);
      if (half == 0 && valid && g < gcount) {
        float s = acc[g][0];
        s = __fadd_rn(s, acc[g][1]);
        s = __fadd_rn(s, acc[g][2]);
        s = __fadd_rn(s, acc[g][3]);
        s = __fadd_rn(s, p0);
        s = __fadd_rn(s, p1);
        s = __fadd_rn(s, p2);
        s = __fadd_rn(s, p3);
        const float* xr = base + r * ld;
        for (int i = rem_begin; i < d; ++i) s = __fadd_rn(s, lane_term<L2>(s_q[g * dq + i], xr[i]));
        const float key = L2 ? s : -s;
        topk.offer(g, pack_cand(key, static_cast<uint32_t>(r)), thr[g]);
      }
    }
    __syncthreads();
    topk.maybe_compact(k, kRowsPerIter, tid, kExactThreads);
#pragma unroll
    for (int g = 0; g < G; ++g) thr[g] = s_thr[g];
  }

  __syncthreads();
  topk.compact_all(k, tid, kExactThreads);
  const int ncta = gridDim.x;
  for (int i = tid; i < gcount * k; i += kExactThreads) {
    int g = i / k, j = i - g * k;
    partial[(static_cast<int64_t>(q0 + g) * ncta + blockIdx.x) * k + j] = s_buf[g * BUF + j];
  }
}

template <int G, int BUF>
size_t exact_smem_bytes(int dq) {
  return sizeof(uint64_t) * (G * BUF + ((G + 1) & ~1)) + sizeof(int) * ((G + 3) & ~3) + sizeof(float) * G * dq;
}

template <int G, int BUF>
cudaError_t launch_exact_g(const ExactScanArgs& a, cudaStream_t stream) {
  const int dq = (a.d + 3) & ~3;
  const size_t smem = exact_smem_bytes<G, BUF>(dq);
  dim3 grid(a.ncta, (a.nq + G - 1) / G);
  if (a.l2) {
    auto kern = exact_scan_kernel<G, BUF, true>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kExactThreads, smem, stream>>>(a.base, a.n, a.ld, a.d, a.queries, dq, a.nq, a.k,
                                                 a.rows_per_cta, a.mask, a.partial);
  } else {
    auto kern = exact_scan_kernel<G, BUF, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kExactThreads, smem, stream>>>(a.base, a.n, a.ld, a.d, a.queries, dq, a.nq, a.k,
                                                 a.rows_per_cta, a.mask, a.partial);
  }
  return cudaGetLastError();
}

template <int BUF>
cudaError_t launch_exact_buf(const ExactScanArgs& a, cudaStream_t stream) {
  switch (a.group) {
    case 1: return launch_exact_g<1, BUF>(a, stream);
    case 2: return launch_exact_g<2, BUF>(a, stream);
    case 4: return launch_exact_g<4, BUF>(a, stream);
    default: return launch_exact_g<8, BUF>(a, stream);
  }
}

}  // namespace

int exact_max_k() { return 1024 - kRowsPerIter; }

int exact_group_for(int64_t nq, int k, int d, size_t smem_limit) {
  int g = nq <= 1 ? 1 : (nq <= 2 ? 2 : (nq <= 4 ? 4 : 8));
  while (g > 0 && exact_smem_for(g, k, d) > smem_limit) g >>= 1;
  return g;
}

size_t exact_smem_for(int group, int k, int d) {
  const int dq = (d + 3) & ~3;
  const int buf = exact_buf_for(k);
  return sizeof(uint64_t) * (group * buf + ((group + 1) & ~1)) + sizeof(int) * ((group + 3) & ~3) +
         sizeof(float) * group * dq;
}

int exact_buf_for(int k) {
  if (k + kRowsPerIter <= 256) return 256;
  if (k + kRowsPerIter <= 512) return 512;
  return 1024;
}

cudaError_t launch_exact_scan(const ExactScanArgs& a, cudaStream_t stream) {
  switch (exact_buf_for(a.k)) {
    case 256: return launch_exact_buf<256>(a, stream);
    case 512: return launch_exact_buf<512>(a, stream);
    default: return launch_exact_buf<1024>(a, stream);
  }
}

}  // namespace px
