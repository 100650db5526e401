// Shard and query preparation for the tensor-core path.
//
// The fp32 rows are kept as given (the exact rescoring and the streaming scan
// read them); beside them each row is split for the 3xTF32 contraction:
//   hi = tf32_rna(x),  lo = tf32_rna(x - hi)      (x - hi is exact in fp32)
// so that q.x ~= qhi.xhi + qhi.xlo + qlo.xhi with an error of a few 2^-22
// relative per product. The split plane interleaves the two halves per
// 16-element chunk -- [hi x16 | lo x16], 128 bytes -- so one 128-byte TMA row
// brings both to shared memory (half the L2 requests of separate planes);
// a 64-byte box over the same plane reads the hi halves alone. Rows are
// padded with zeros to a multiple of 32 floats, which leaves every dot
// product unchanged. A bf16 copy (round to nearest even, rows padded with
// zeros to a multiple of 64 so one 128-byte TMA row is one K slice) feeds the
// first candidate pass for small k; a flag records whether any value is not
// exactly representable in bf16. `norms` holds the squared L2 norm of each
// row for the approximate key ||x||^2 - 2 q.x.
//
// Folded L2 norms: where a row's bf16 padding has room (d + 3 <= ldb), the
// bf16 copy of a shard row also carries its fp32 ||x||^2 in columns d, d+1,
// d+2, split into three bf16 values whose sum is exact. Round-to-nearest
// splitting leaves a remainder of at most 16 significant bits after the
// first piece and at most 8 after the second, so the third is exact (for
// norms above 2^-100, below which bf16 subnormals could drop bits). A query
// converted for a folded L2 pass holds 2q (exact doubling) and -1 in those
// columns, so its bf16 product with a row is 2 q.x - ||x||^2, the negated L2
// key, and the inner-product epilogue serves the L2 pass. Any other query
// holds zeros there, which leaves its products unchanged.
#include <cuda_bf16.h>

#include "px_common.cuh"
#include "px_kernels.h"

namespace px {

namespace {

// An upper bound, as a float, on the square root of a sum of squares that
// was accumulated in double (each square exact, at most a few dozen adds):
// the relative margin dwarfs double rounding, and both conversions round up.
__device__ __forceinline__ float sqrt_up(double sum_sq) {
  return __double2float_ru(__dsqrt_ru(sum_sq * (1.0 + 0x1p-40)));
}

// One warp per row.
// fold_query: convert query rows for a folded L2 pass (see above).
// resid (shard rows): resid[0] / resid[1] are raised (float bits) to an upper
// bound on ||x - bf16(x)|| / ||x - tf32_hi(x)|| over the row's d values, the
// per-row representation errors the certificate of a bf16 / tf32 candidate
// pass bounds the shard's contribution by.
__global__ void prepare_rows_kernel(const float* __restrict__ src, int64_t n, int d, int ld, int ldb,
                                    float* __restrict__ dst, float* __restrict__ hl,
                                    __nv_bfloat16* __restrict__ xb, float* __restrict__ norms,
                                    int* __restrict__ lo_nonzero, int* __restrict__ bf_inexact,
                                    int* __restrict__ max_norm_sq, bool fold_query, int* __restrict__ resid) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  bool nz = false, bz = false;
  // x - bf16(x) and x - tf32(x) are exact in fp32, and their squares exact in
  // double.
  double rb = 0.0, rt = 0.0;
  const int width = ldb > ld ? ldb : ld;
  for (int e = lane; e < width; e += 32) {
    float x = e < d ? src[row * d + e] : 0.f;
    if (e < ld) {
      if (dst) dst[row * ld + e] = x;
      if (hl) {
        const float h = tf32_rna(x);
        const float r = __fsub_rn(x, h);
        const float l = tf32_rna(r);
        float* p = hl + row * 2 * ld + (e >> 4) * 32 + (e & 15);
        p[0] = h;
        p[16] = l;
        nz |= (l != 0.f);
        rt += static_cast<double>(r) * r;
      }
    }
    if (xb && e < ldb) {
      const float xv = !fold_query ? x : (e < d ? __fmul_rn(2.0f, x) : (e < d + 3 ? -1.0f : 0.0f));
      const __nv_bfloat16 b = __float2bfloat16_rn(xv);
      xb[row * ldb + e] = b;
      const float r = __fsub_rn(xv, __bfloat162float(b));
      bz |= (r != 0.f);
      rb += static_cast<double>(r) * r;
    }
  }
  __syncwarp();
  const bool any_nz = __any_sync(0xffffffffu, nz);
  const bool any_bz = __any_sync(0xffffffffu, bz);
  if (lo_nonzero && any_nz && lane == 0) atomicOr(lo_nonzero, 1);
  if (bf_inexact && any_bz && lane == 0) atomicOr(bf_inexact, 1);
  if (resid) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      rb += __shfl_xor_sync(0xffffffffu, rb, off);
      rt += __shfl_xor_sync(0xffffffffu, rt, off);
    }
    // Non-negative floats order like their bit patterns as ints.
    if (lane == 0) {
      atomicMax(resid, __float_as_int(sqrt_up(rb)));
      atomicMax(resid + 1, __float_as_int(sqrt_up(rt)));
    }
  }
  if ((norms || max_norm_sq) && lane == 0) {
    // Squared norm in the reference's 8-lane order (l2_sqr(x, 0)).
    const float* x = (dst ? dst + row * ld : src + row * d);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const int chunks = d >> 3;
    for (int c = 0; c < chunks; ++c)
#pragma unroll
      for (int l = 0; l < 8; ++l) acc[l] = __fadd_rn(acc[l], __fmul_rn(x[c * 8 + l], x[c * 8 + l]));
    float s = acc[0];
#pragma unroll
    for (int l = 1; l < 8; ++l) s = __fadd_rn(s, acc[l]);
    for (int i = chunks * 8; i < d; ++i) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
    if (norms) norms[row] = s;
    if (max_norm_sq) atomicMax(max_norm_sq, __float_as_int(s));  // s >= 0: int order = float order
    if (xb && d + 3 <= ldb) {  // shard row: the folded norm (the warp's zero padding is ordered before)
      const __nv_bfloat16 h = __float2bfloat16_rn(s);
      const float r1 = __fsub_rn(s, __bfloat162float(h));
      const __nv_bfloat16 m = __float2bfloat16_rn(r1);
      xb[row * ldb + d] = h;
      xb[row * ldb + d + 1] = m;
      xb[row * ldb + d + 2] = __float2bfloat16_rn(__fsub_rn(r1, __bfloat162float(m)));
    }
  }
}

__global__ void pack_mask_kernel(const uint8_t* __restrict__ mask, int64_t n, uint32_t* __restrict__ bits) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (w * 32 >= n) return;
  uint32_t b = 0;
  for (int j = 0; j < 32; ++j) {
    const int64_t r = w * 32 + j;
    if (r < n && mask[r] != 0) b |= 1u << j;
  }
  bits[w] = b;
}

__global__ void zero_rows_kernel(float* __restrict__ p, int64_t begin, int64_t end, int ld) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x + begin * ld;
  if (i < end * ld) p[i] = 0.f;
}

}  // namespace

cudaError_t launch_pack_mask(const uint8_t* mask, int64_t n, uint32_t* bits, cudaStream_t stream) {
  const int64_t words = (n + 31) / 32;
  if (words == 0) return cudaSuccess;
  pack_mask_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, stream>>>(mask, n, bits);
  return cudaGetLastError();
}

cudaError_t launch_prepare_rows(const float* src, int64_t n, int d, int ld, int ldb, float* dst, float* hl,
                                void* xb, float* norms, int* lo_nonzero, int* bf_inexact, int* max_norm_sq,
                                cudaStream_t stream, bool fold_query, int* resid) {
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks = (n * 32 + threads - 1) / threads;
  prepare_rows_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      src, n, d, ld, ldb, dst, hl, static_cast<__nv_bfloat16*>(xb), norms, lo_nonzero, bf_inexact,
      max_norm_sq, fold_query, resid);
  return cudaGetLastError();
}

cudaError_t launch_split_queries(const float* q, int64_t nq, int d, int ld, int ldb, int64_t rows_alloc,
                                 float* hl, void* qb, int* lo_nonzero, int* bf_inexact, cudaStream_t stream,
                                 bool fold_l2) {
  cudaError_t e = launch_prepare_rows(q, nq, d, ld, ldb, nullptr, hl, qb, nullptr, lo_nonzero, bf_inexact,
                                      nullptr, stream, fold_l2);
  if (e != cudaSuccess) return e;
  if (rows_alloc > nq) {
    const int threads = 256;
    if (hl) {
      const int64_t count = (rows_alloc - nq) * 2 * ld;
      const unsigned blocks = static_cast<unsigned>((count + threads - 1) / threads);
      zero_rows_kernel<<<blocks, threads, 0, stream>>>(hl, nq, rows_alloc, 2 * ld);
    }
    if (qb) {
      // ldb is a multiple of 64: the bf16 padding rows are whole float pairs.
      const int64_t count = (rows_alloc - nq) * (ldb / 2);
      const unsigned blocks = static_cast<unsigned>((count + threads - 1) / threads);
      zero_rows_kernel<<<blocks, threads, 0, stream>>>(static_cast<float*>(qb), nq, rows_alloc, ldb / 2);
    }
  }
  return cudaGetLastError();
}

}  // namespace px
