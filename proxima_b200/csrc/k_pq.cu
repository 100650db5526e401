// PQ asymmetric-distance scan (K3 LUT build, K4 scan) and the nearest-centroid
// kernel used by PQ encoding and k-means assignment.
//
// Arithmetic restated from crates/core/src/pq.rs:
//   adc_table  (pq.rs:123-136): table[sub*ksub + c] = l2_sqr(q_sub, centroid)
//                               or -inner_product, exact 8-lane order;
//   scan       (pq.rs:314-323): key = 0.0; key += table[sub*ksub + code[sub]]
//                               for sub = 0..m-1, sequential f32 adds;
//   encode_into(pq.rs:107-121) and the kmeans assignment (pq.rs:155-167):
//                               argmin over centroids with strict '<', so the
//                               first of equal distances wins.
// All three are bit-exact with the CPU.
#include "px_common.cuh"
#include "px_kernels.h"

namespace px {

namespace {

constexpr int kPqThreads = 512;       // 16 warps: enough to hide the LUT-gather latency
constexpr int kPqRowsPerIter = 512;   // kSlots (threads / G) x G rows per thread
// Candidate buffer of the m = 16, 8-query scan for k <= 32: 1,024 rows per
// iteration (the most one iteration can add per query) plus 32. Its
// compactions are warp selections, which need no power-of-two size.
constexpr int kPqWideBuf = 1056;

// 32-bit shared-memory load (the LUT gathers are the kernel's hot loop).
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

// The same load, free for the compiler to schedule and to fold constant
// offsets into. Only for addresses that depend on data loaded after the
// table's __syncthreads (a code byte), so it cannot move above it.
__device__ __forceinline__ float lds_f32_sched(uint32_t addr) {
  float v;
  asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

// Four adjacent table entries (one code, four queries) in one 16-byte load;
// same scheduling freedom and the same condition on the address.
__device__ __forceinline__ float4 lds_f32x4_sched(uint32_t addr) {
  float4 v;
  asm("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// Two fp32 additions in one instruction (Blackwell's add.rn.f32x2): each half
// is rounded to nearest-even on its own, exactly as add.rn.f32 rounds it, so
// the packed sums are bit-identical to two __fadd_rn.
__device__ __forceinline__ uint64_t fadd2(uint64_t acc, float x, float y) {
  uint64_t b, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(x), "f"(y));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(acc), "l"(b));
  return r;
}
__device__ __forceinline__ float lo_f32(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float hi_f32(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }

__global__ void pq_lut_kernel(const float* __restrict__ books, int m, int ksub, int dsub, bool l2,
                              const float* __restrict__ queries, float* __restrict__ lut) {
  const int q = blockIdx.x;
  const int dim = m * dsub;
  const float* qv = queries + static_cast<int64_t>(q) * dim;
  float* out = lut + static_cast<int64_t>(q) * m * ksub;
  for (int i = threadIdx.x; i < m * ksub; i += blockDim.x) {
    const int sub = i / ksub;
    const float* cen = books + static_cast<int64_t>(i) * dsub;
    const float* qs = qv + sub * dsub;
    out[i] = l2 ? exact_key<true>(qs, cen, dsub) : exact_key<false>(qs, cen, dsub);
  }
}

// One CTA scans `rows_per_cta` codes for G queries. Shared-memory LUT layout
// is [sub][code][G]: the G threads that share a code read G consecutive words,
// so a warp's gathers touch at most 32/G distinct 32-word rows.
// M > 0: m == M (a multiple of 16) and ksub == 256, so table offsets and
// code byte positions are compile-time constants; M == 0: any m and ksub.
// M == 16 with G == 8 (the common case) takes the skewed schedule below, over
// a [sub/8][code][sub%8][query] table; with BUF == kPqWideBuf (k <= 32) it
// covers 1,024 rows per iteration instead of 512.
template <int G, int BUF, int M>
__global__ void __launch_bounds__(kPqThreads)
pq_scan_kernel(const uint8_t* __restrict__ codes, int64_t n, int m, int ksub,
               const float* __restrict__ lut, int nq, int k, int64_t rows_per_cta,
               const uint8_t* __restrict__ mask, uint64_t* __restrict__ partial) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* s_buf = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* s_thr = s_buf + G * BUF;  // G words, padded to an even count
  int* s_cnt = reinterpret_cast<int*>(s_thr + ((G + 1) & ~1));
  float* s_lut = reinterpret_cast<float*>(s_cnt + ((G + 3) & ~3));

  const int tid = threadIdx.x;
  const int q0 = blockIdx.y * G;
  const int gcount = min(G, nq - q0);
  const int table = m * ksub;

  BlockTopK<G, BUF> topk;
  topk.init(s_buf, s_cnt, s_thr, tid, kPqThreads);
  constexpr bool kSkewed = M == 16 && G == 8;
  if constexpr (kSkewed) {
    // [sub/8][code][sub%8][query]: a code's entries for eight subs and eight
    // queries fill 256 bytes, so sub s's 32 bytes sit in bank slice s % 4
    // whatever the code.
    for (int d = tid; d < G * table; d += kPqThreads) {
      const int g = d & 7, s = ((d >> 14) << 3) | ((d >> 3) & 7), c = (d >> 6) & 255;
      s_lut[d] = g < gcount ? lut[static_cast<int64_t>(q0 + g) * table + s * 256 + c] : 0.f;
    }
  } else {
    for (int i = tid; i < G * table; i += kPqThreads) {
      const int e = i / G, g = i - e * G;
      s_lut[i] = g < gcount ? lut[static_cast<int64_t>(q0 + g) * table + e] : 0.f;
    }
  }
  __syncthreads();

  const int g = tid % G;
  const int slot = tid / G;               // 0 .. kPqThreads/G - 1
  constexpr int kSlots = kPqThreads / G;  // codes per step
  const int64_t row_begin = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
  const int64_t row_end = min(n, row_begin + rows_per_cta);
  const bool vec16 = (m & 15) == 0;
  const uint32_t lut_addr = static_cast<uint32_t>(__cvta_generic_to_shared(s_lut));
  uint64_t thr = PX_EMPTY;

  if constexpr (kSkewed) {
    // Two threads per row, each serving four of the eight queries with one
    // 16-byte load per sub. A 16-byte shared load is served a quarter-warp
    // (four rows) at a time, and four random codes would collide in the four
    // 32-byte bank slices. So the four rows of a quarter-warp run skewed: the
    // row at position p is p steps behind, reading sub (i - p) % 16 at step
    // i, which is bank slice (i - p) % 4 -- four distinct slices, one
    // wavefront. Each thread streams its kRows rows' codes back to back; every
    // row still adds its subs in order 0..15 from 0.0, so keys are bit-exact.
    constexpr int kIterRows = BUF == kPqWideBuf ? 1024 : kPqRowsPerIter;
    constexpr int kRows = kIterRows / (kPqThreads / 2);
    constexpr int kWords = M * kRows / 4;  // code words of a thread's rows
    constexpr int kSkew = 3;
    constexpr int kSteps = M * kRows + kSkew;
    const int quad = tid & 1;
    const int qslot = tid >> 1;  // 0 .. kPqThreads/2 - 1
    const int p = qslot & 3;     // row position within the quarter-warp
    // off[t]: address of sub (t - p) % 16 for this thread's four queries.
    uint32_t off[M];
#pragma unroll
    for (int t = 0; t < M; ++t) {
      const int s = (t - p) & (M - 1);
      off[t] = lut_addr + static_cast<uint32_t>(quad * 16 + (s >> 3) * 65536 + (s & 7) * 32);
    }
    const uint32_t shift = 32u - 8u * static_cast<uint32_t>(p);
    uint64_t thr4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) thr4[j] = PX_EMPTY;
    // The next iteration's filter bytes and codes, fetched one iteration
    // ahead: every warp starts an iteration at the same barrier, so codes
    // loaded there would leave the SM idle for a global-memory round trip.
    uint4 nv[kRows];
    bool nok[kRows];
    auto fetch = [&](int64_t at) {
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        const int64_t row = at + r * (kPqThreads / 2) + qslot;
        nok[r] = row < row_end && (mask == nullptr || mask[row] != 0);
        nv[r] = nok[r] ? __ldg(reinterpret_cast<const uint4*>(codes + row * M)) : make_uint4(0, 0, 0, 0);
      }
    };
    if (row_begin < row_end) fetch(row_begin);
    for (int64_t it = row_begin; it < row_end; it += kIterRows) {
      bool ok[kRows];
      int64_t rr[kRows];
      uint32_t cw[kWords + 2];  // cw[1 + w] = code word w; zero on both sides
      cw[0] = 0u;
      cw[kWords + 1] = 0u;
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        rr[r] = it + r * (kPqThreads / 2) + qslot;
        ok[r] = nok[r];
        cw[1 + r * 4] = nv[r].x;
        cw[2 + r * 4] = nv[r].y;
        cw[3 + r * 4] = nv[r].z;
        cw[4 + r * 4] = nv[r].w;
      }
      if (it + kIterRows < row_end) fetch(it + kIterRows);
      // The code stream delayed by p bytes: byte i of sw is code byte i - p.
      uint32_t sw[kWords + 1];
#pragma unroll
      for (int w = 0; w <= kWords; ++w) sw[w] = __funnelshift_rc(cw[w], cw[w + 1], shift);
      // Queries (0, 1) and (2, 3) of the four as packed pairs: one f32x2
      // addition each per step.
      uint64_t k01 = 0, k23 = 0;  // +0.0f, +0.0f
      float fin[kRows][4];
#pragma unroll
      for (int i = 0; i < kSteps; ++i) {
        // code << 8 is the code's offset: 256 bytes per code.
        const uint32_t c8 = __byte_perm(sw[i >> 2], 0u, 0x4404u | (static_cast<uint32_t>(i & 3) << 4));
        const float4 t = lds_f32x4_sched(off[i & (M - 1)] + c8);
        if (i >= kSkew || i >= p) {  // before step p this thread's first row has not begun
          k01 = fadd2(k01, t.x, t.y);
          k23 = fadd2(k23, t.z, t.w);
        }
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          constexpr int kLast = M - 1;
          const int q = i - r * M - kLast;  // the position whose row r ends at step i
          if (q >= 0 && q <= kSkew && p == q) {
            fin[r][0] = lo_f32(k01);
            fin[r][1] = hi_f32(k01);
            fin[r][2] = lo_f32(k23);
            fin[r][3] = hi_f32(k23);
            k01 = 0;
            k23 = 0;
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kRows; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (ok[r] && quad * 4 + j < gcount)
            topk.offer(quad * 4 + j, pack_cand(fin[r][j], static_cast<uint32_t>(rr[r])), thr4[j]);
      __syncthreads();
      topk.maybe_compact(k, kIterRows, tid, kPqThreads);
#pragma unroll
      for (int j = 0; j < 4; ++j) thr4[j] = s_thr[quad * 4 + j];
    }
  } else
  for (int64_t it = row_begin; it < row_end; it += kPqRowsPerIter) {
    // Each thread scores G rows per iteration for its query g. The G rows'
    // codes are loaded first and their m-long addition chains interleaved
    // (G independent chains per thread); every chain keeps the reference's
    // sub order, so the keys stay bit-exact.
    bool ok[G];
    int64_t rr[G];
#pragma unroll
    for (int i = 0; i < G; ++i) {
      rr[i] = it + i * kSlots + slot;
      ok[i] = rr[i] < row_end && g < gcount && (mask == nullptr || mask[rr[i]] != 0);
    }
    float key[G];
#pragma unroll
    for (int i = 0; i < G; ++i) key[i] = 0.0f;
    if constexpr (M > 0) {
      const uint32_t lbase = lut_addr + static_cast<uint32_t>(g * 4);
#pragma unroll
      for (int b = 0; b < M; b += 16) {
        uint4 w[G];
#pragma unroll
        for (int i = 0; i < G; ++i)
          w[i] = ok[i] ? __ldg(reinterpret_cast<const uint4*>(codes + rr[i] * M + b)) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
          for (int bi = 0; bi < 4; ++bi) {
            const uint32_t lsub = lbase + static_cast<uint32_t>((b + wi * 4 + bi) * 256 * G * 4);
#pragma unroll
            for (int i = 0; i < G; ++i) {
              const uint32_t word = wi == 0 ? w[i].x : (wi == 1 ? w[i].y : (wi == 2 ? w[i].z : w[i].w));
              const uint32_t c = __byte_perm(word, 0u, 0x4440u | static_cast<uint32_t>(bi));
              key[i] = __fadd_rn(key[i], lds_f32_sched(lsub + c * (G * 4)));
            }
          }
        }
      }
    } else if (vec16) {
      for (int b = 0; b < m; b += 16) {
        uint4 w[G];
#pragma unroll
        for (int i = 0; i < G; ++i)
          w[i] = ok[i] ? __ldg(reinterpret_cast<const uint4*>(codes + rr[i] * m + b)) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
          for (int bi = 0; bi < 4; ++bi) {
            const int sub = b + wi * 4 + bi;
            const uint32_t lsub = lut_addr + static_cast<uint32_t>((sub * ksub * G + g) * 4);
#pragma unroll
            for (int i = 0; i < G; ++i) {
              const uint32_t word = wi == 0 ? w[i].x : (wi == 1 ? w[i].y : (wi == 2 ? w[i].z : w[i].w));
              const uint32_t c = (word >> (8 * bi)) & 0xFFu;
              key[i] = __fadd_rn(key[i], lds_f32(lsub + c * (G * 4)));
            }
          }
        }
      }
    } else {
      for (int sub = 0; sub < m; ++sub) {
        const uint32_t lsub = lut_addr + static_cast<uint32_t>((sub * ksub * G + g) * 4);
#pragma unroll
        for (int i = 0; i < G; ++i) {
          const uint32_t c = ok[i] ? codes[rr[i] * m + sub] : 0u;
          key[i] = __fadd_rn(key[i], lds_f32(lsub + c * (G * 4)));
        }
      }
    }
#pragma unroll
    for (int i = 0; i < G; ++i)
      if (ok[i]) topk.offer(g, pack_cand(key[i], static_cast<uint32_t>(rr[i])), thr);
    __syncthreads();
    topk.maybe_compact(k, kPqRowsPerIter, tid, kPqThreads);
    thr = s_thr[g];
  }

  __syncthreads();
  topk.compact_all(k, tid, kPqThreads);
  const int ncta = gridDim.x;
  for (int i = tid; i < gcount * k; i += kPqThreads) {
    const int gg = i / k, j = i - gg * k;
    partial[(static_cast<int64_t>(q0 + gg) * ncta + blockIdx.x) * k + j] = s_buf[gg * BUF + j];
  }
}

template <int G, int BUF, int M>
cudaError_t launch_pq_gm(const PqScanArgs& a, cudaStream_t stream) {
  const size_t smem = pq_smem_for(G, a.m, a.ksub, a.k);
  auto kern = pq_scan_kernel<G, BUF, M>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.ncta, (a.nq + G - 1) / G);
  kern<<<grid, kPqThreads, smem, stream>>>(a.codes, a.n, a.m, a.ksub, a.lut, a.nq, a.k,
                                           a.rows_per_cta, a.mask, a.partial);
  return cudaGetLastError();
}

template <int G, int BUF>
cudaError_t launch_pq_g(const PqScanArgs& a, cudaStream_t stream) {
  if (a.ksub == 256) {
    if (a.m == 16) return launch_pq_gm<G, BUF, 16>(a, stream);
    if (a.m == 32) return launch_pq_gm<G, BUF, 32>(a, stream);
  }
  return launch_pq_gm<G, BUF, 0>(a, stream);
}

template <int BUF>
cudaError_t launch_pq_buf(const PqScanArgs& a, cudaStream_t stream) {
  switch (a.group) {
    case 1: return launch_pq_g<1, BUF>(a, stream);
    case 2: return launch_pq_g<2, BUF>(a, stream);
    case 4: return launch_pq_g<4, BUF>(a, stream);
    default: return launch_pq_g<8, BUF>(a, stream);
  }
}

int pq_buf_for(int group, int m, int ksub, int k) {
  if (group == 8 && m == 16 && ksub == 256 && k <= 32) return kPqWideBuf;
  if (k + kPqRowsPerIter <= 1024) return 1024;
  return 2048;
}

// Nearest centroid: grid.y = subspace, one thread per vector. All threads of
// a warp walk the same centroids, so centroid reads are broadcasts.
__global__ void nearest_centroid_kernel(const float* __restrict__ vectors, int64_t n, int m,
                                        int dsub, int ksub, const float* __restrict__ books,
                                        uint32_t* __restrict__ out_assign,
                                        uint8_t* __restrict__ out_codes) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int sub = blockIdx.y;
  if (i >= n) return;
  const float* v = vectors + i * static_cast<int64_t>(m) * dsub + sub * dsub;
  const float* book = books + static_cast<int64_t>(sub) * ksub * dsub;
  uint32_t best = 0;
  float best_d = 3.40282347e+38f;
  for (int c = 0; c < ksub; ++c) {
    const float dist = exact_dot_or_l2<true>(v, book + static_cast<int64_t>(c) * dsub, dsub);
    if (dist < best_d) {
      best_d = dist;
      best = static_cast<uint32_t>(c);
    }
  }
  if (out_assign) out_assign[i * m + sub] = best;
  if (out_codes) out_codes[i * m + sub] = static_cast<uint8_t>(best);
}

}  // namespace

int pq_max_k() { return 2048 - kPqRowsPerIter; }

int pq_rows_per_iter(int group, int m, int ksub, int k) {
  return pq_buf_for(group, m, ksub, k) == kPqWideBuf ? 1024 : kPqRowsPerIter;
}

size_t pq_smem_for(int group, int m, int ksub, int k) {
  const int buf = pq_buf_for(group, m, ksub, k);
  return sizeof(uint64_t) * (group * buf + ((group + 1) & ~1)) + sizeof(int) * ((group + 3) & ~3) +
         sizeof(float) * static_cast<size_t>(group) * m * ksub;
}

int pq_group_for(int m, int ksub, int64_t nq, int k) {
  const size_t budget = 200 * 1024;
  int g = 8;
  while (g > 1 && (pq_smem_for(g, m, ksub, k) > budget || g / 2 >= nq)) g >>= 1;
  return g;
}

cudaError_t launch_pq_lut(const float* books, int m, int ksub, int dsub, bool l2,
                          const float* queries, int nq, float* lut, cudaStream_t stream) {
  if (nq == 0) return cudaSuccess;
  pq_lut_kernel<<<nq, 256, 0, stream>>>(books, m, ksub, dsub, l2, queries, lut);
  return cudaGetLastError();
}

cudaError_t launch_pq_scan(const PqScanArgs& a, cudaStream_t stream) {
  const int buf = pq_buf_for(a.group, a.m, a.ksub, a.k);
  if (buf == kPqWideBuf) return launch_pq_gm<8, kPqWideBuf, 16>(a, stream);
  if (buf == 1024) return launch_pq_buf<1024>(a, stream);
  return launch_pq_buf<2048>(a, stream);
}

cudaError_t launch_nearest_centroid(const float* vectors, int64_t n, int m, int dsub, int ksub,
                                    const float* books, uint32_t* out_assign, uint8_t* out_codes,
                                    cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const int threads = 128;
  dim3 grid(static_cast<unsigned>((n + threads - 1) / threads), m);
  nearest_centroid_kernel<<<grid, threads, 0, stream>>>(vectors, n, m, dsub, ksub, books,
                                                        out_assign, out_codes);
  return cudaGetLastError();
}

}  // namespace px
