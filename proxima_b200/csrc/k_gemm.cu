// K1: batched exact-kNN candidate generation on the 5th-generation tensor
// cores, with the top-k selection fused into the epilogue.
//
// The query x base distance matrix is a dense contraction; this kernel
// computes it tile by tile in TMEM and never writes it to HBM. Operands are
// the tf32 split planes of the queries and the shard (hi = tf32(x),
// lo = tf32(x - hi), interleaved per 16-element chunk); each output tile
// accumulates
//     qhi.xhi + qhi.xlo + qlo.xhi            (3xTF32, ~fp32 accurate)
// from 128-byte [hi|lo] TMA rows (128-byte swizzle), skipping a cross term
// whenever the corresponding lo plane is all zeros. A second variant reads
// only the 64-byte hi halves (64-byte swizzle) and multiplies qhi.xhi, and a
// third multiplies the bf16 copies of queries and rows (kind::f16, 128-byte
// rows of 64 elements) at twice the tf32 rate and half the bytes; both are
// exact for integer-valued data and otherwise carry a rounding error the
// certificate accounts for. The epilogue turns each
// accumulator into an approximate key (||x||^2 - 2 q.x for L2, -q.x for
// inner product) and keeps, per query, the CAP smallest keys in registers.
// Exactness is restored afterwards: the CAP candidates are rescored in the
// reference's arithmetic and certified against the error bound of this
// approximation (k_rescore.cu).
//
// CTA roles (64 + 128*QT threads, one CTA per SM):
//   warp 0      TMA producer: ring of {QT query tiles, one base tile} K-slices
//   warp 1      TMEM owner and MMA issuer (one elected thread)
//   warps 2..   QT epilogue warpgroups: TMEM -> registers -> per-query lists
// Two accumulator buffers (all 512 TMEM columns) let the epilogue drain tile
// t while the tensor core fills tile t+1.
//
// Work items are (query tile, contiguous run of base tiles); a persistent CTA
// walks items blockIdx.x, +gridDim.x, ... Items are ordered run-major, so
// the CTAs of one wave stream the same base tiles at the same time and share
// them through L2. Each item ends by writing its 128 sorted lists.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "px_common.cuh"
#include "px_kernels.h"
#include "px_tc.cuh"

namespace px {

namespace {

constexpr int BM = 128;  // queries per query tile (TMEM lanes)
constexpr uint32_t kTmemCols = 512;

// QT query tiles share each base tile of BN = 256 / QT rows. A stage row is
// 128 bytes -- [hi x16 | lo x16] tf32 (3xTF32) or 64 bf16 values -- with 4
// stages, or 64 bytes of hi values with 8 stages (tf32 hi-only). Either way
// the ring holds 192 KB, and the TMEM holds 2 buffers x QT accumulators x BN
// columns = 512 columns.
template <int QT, int KIND> struct Tile {
  static constexpr bool IL = KIND == kPass3xTf32;
  static constexpr bool BF = KIND == kPassBf16;
  static constexpr int BN = 256 / QT;
  static constexpr int ROW = KIND == kPassTf32 ? 64 : 128;  // bytes per tile row per stage
  static constexpr int STAGES = KIND == kPassTf32 ? 8 : 4;
  static constexpr int KEL = BF ? 64 : 16;    // K elements per stage
  static constexpr int KCOORD = BF ? 64 : 32; // plane columns per stage
  static constexpr int A_TILE = BM * ROW;
  static constexpr int B_TILE = BN * ROW;
  static constexpr int STAGE_BYTES = QT * A_TILE + B_TILE;
  static constexpr int NBARS = 2 * STAGES + 2 + 2 + 1;  // full, empty, tmem full, tmem empty, done
  static constexpr int THREADS = 64 + 128 * QT;  // TMA warp, MMA warp, QT epilogue warpgroups
  static constexpr size_t SMEM = 1024 + STAGES * STAGE_BYTES + NBARS * 8 + 16 + 128 * QT * 33 * 4;
};

__device__ __forceinline__ bool mbar_wait_quiet(uint32_t bar, uint32_t parity) {
  int dummy = 0;
  return tc::mbar_wait(bar, parity, &dummy);
}

__device__ __forceinline__ float min3f(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Largest of 32 raw accumulator words (as floats), the same tree with max.
__device__ __forceinline__ float max32u(const uint32_t (&v)[32]) {
  float a[10];
#pragma unroll
  for (int i = 0; i < 10; ++i)
    a[i] = max3f(__uint_as_float(v[3 * i]), __uint_as_float(v[3 * i + 1]), __uint_as_float(v[3 * i + 2]));
  const float b0 = max3f(a[0], a[1], a[2]);
  const float b1 = max3f(a[3], a[4], a[5]);
  const float b2 = max3f(a[6], a[7], a[8]);
  const float b3 = max3f(a[9], __uint_as_float(v[30]), __uint_as_float(v[31]));
  return fmaxf(max3f(b0, b1, b2), b3);
}

// Smallest of 32 keys: a depth-4 tree of three-input minimums (16 ops).
__device__ __forceinline__ float min32(const float (&k)[32]) {
  float a[10];
#pragma unroll
  for (int i = 0; i < 10; ++i) a[i] = min3f(k[3 * i], k[3 * i + 1], k[3 * i + 2]);
  const float b0 = min3f(a[0], a[1], a[2]);
  const float b1 = min3f(a[3], a[4], a[5]);
  const float b2 = min3f(a[6], a[7], a[8]);
  const float b3 = min3f(a[9], k[30], k[31]);
  return fminf(min3f(b0, b1, b2), b3);
}

// Replaces the list's largest entry by cand and finds the new largest key.
// The scan compares keys only (the words' high halves): among entries with
// the largest key it keeps the first, and the threshold becomes the largest
// word with that key, so a later candidate with an equal key may replace an
// equal one. Either way every row the list drops has a key >= the list's
// largest key, which is all the certificate relies on; words stay distinct.
template <int CAP>
__device__ __forceinline__ void list_insert(uint64_t (&L)[CAP], uint64_t& thr, int& maxpos,
                                            uint64_t cand) {
#pragma unroll
  for (int j = 0; j < CAP; ++j) L[j] = (j == maxpos) ? cand : L[j];
  uint32_t hi = static_cast<uint32_t>(L[0] >> 32);
  maxpos = 0;
#pragma unroll
  for (int j = 1; j < CAP; ++j) {
    const uint32_t h = static_cast<uint32_t>(L[j] >> 32);
    if (h > hi) {
      hi = h;
      maxpos = j;
    }
  }
  thr = (static_cast<uint64_t>(hi) << 32) | 0xFFFFFFFFull;
}

template <int CAP>
__device__ __forceinline__ void list_sort(uint64_t (&L)[CAP]) {
#pragma unroll
  for (int size = 2; size <= CAP; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < CAP; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const uint64_t a = L[i], b = L[j];
          const bool sw = up ? (a > b) : (a < b);
          L[i] = sw ? b : a;
          L[j] = sw ? a : b;
        }
      }
    }
  }
}

// One top-CAP candidate list of an epilogue thread: unsorted words, the
// largest of them (thr, PX_EMPTY while not full) and its position, thr's key
// as a float for the column tests, and the key the list admits while it is
// not full (open_key).
template <int CAP>
struct TopList {
  uint64_t L[CAP];
  uint64_t thr;
  float thr_key;
  float open_key;
  int maxpos;

  // start_key: +inf (accept everything), a sample pass's k-th key, or -inf
  // for a padding query row.
  __device__ __forceinline__ void reset(float start_key) {
#pragma unroll
    for (int j = 0; j < CAP; ++j) L[j] = PX_EMPTY;
    thr = PX_EMPTY;
    thr_key = start_key;
    open_key = start_key;
    maxpos = 0;
  }
};

// The key a query's lists start from. Without a seed every list is open
// (+inf). With one, seed[qidx][seed_k - 1] is the seed_k-th best word a
// sample pass found (seed_k >= k): seed_k real rows have keys <= its key, so
// no row above it can be in the top k, and the lists admit only keys <= it
// (fewer than seed_k sample candidates: open). A padding query row (past nq) has all-zero products,
// hence equal keys that would all pass and take the rare insertion path on
// every step: -inf lets nothing in.
__device__ __forceinline__ float list_start_key(const GemmTopkArgs& p, int64_t qidx) {
  if (qidx >= p.nq) return __int_as_float(0xff800000);
  if (p.seed != nullptr) {
    const uint64_t w = p.seed[qidx * p.seed_k + p.seed_k - 1];
    if (w != PX_EMPTY) return cand_key(w);
  }
  return __int_as_float(0x7f800000);
}

// Approximate keys of 32 accumulator columns (base rows rbase ..): -q.x, or
// ||x||^2 - 2 q.x with the row norms (padded to whole 256-row tiles, so every
// chunk of a tile is in bounds).
template <bool L2>
__device__ __forceinline__ void chunk_keys(const uint32_t (&v)[32], const GemmTopkArgs& p, int64_t rbase,
                                           float (&key)[32]) {
  if (L2) {
    const float4* nrm = reinterpret_cast<const float4*>(p.norms + rbase);
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
      const float4 nv = __ldg(nrm + j4);
      key[4 * j4 + 0] = fmaf(-2.0f, __uint_as_float(v[4 * j4 + 0]), nv.x);
      key[4 * j4 + 1] = fmaf(-2.0f, __uint_as_float(v[4 * j4 + 1]), nv.y);
      key[4 * j4 + 2] = fmaf(-2.0f, __uint_as_float(v[4 * j4 + 2]), nv.z);
      key[4 * j4 + 3] = fmaf(-2.0f, __uint_as_float(v[4 * j4 + 3]), nv.w);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) key[j] = -__uint_as_float(v[j]);
  }
}

__device__ __forceinline__ uint32_t low_bits(int n) {
  return n <= 0 ? 0u : (n >= 32 ? 0xffffffffu : (1u << n) - 1u);
}

// Inserts one column (key, row) if it beats the list's threshold.
template <int CAP>
__device__ __forceinline__ void insert_one(TopList<CAP>& T, float key, int64_t row) {
  const uint64_t cand = pack_cand(key, static_cast<uint32_t>(row));
  if (cand < T.thr) {
    list_insert<CAP>(T.L, T.thr, T.maxpos, cand);
    T.thr_key = T.thr == PX_EMPTY ? T.open_key : cand_key(T.thr);
  }
}

// Inserts the columns of `pass` (keys in slot[0..31], rows rbase ..) that
// beat the running threshold into the top-CAP list.
template <int CAP>
__device__ __forceinline__ void insert_passing(TopList<CAP>& T, uint32_t pass, const float* slot, int64_t rbase) {
  while (pass) {
    const int j = __ffs(pass) - 1;
    pass &= pass - 1;
    const float kj = slot[j];
    if (kj <= T.thr_key) {
      const uint64_t cand = pack_cand(kj, static_cast<uint32_t>(rbase + j));
      if (cand < T.thr) {
        list_insert<CAP>(T.L, T.thr, T.maxpos, cand);
        T.thr_key = T.thr == PX_EMPTY ? T.open_key : cand_key(T.thr);
      }
    }
  }
}

// Drains NCOL accumulator columns (base rows row0 ..) of this thread's TMEM
// lane, 64 columns per step: two TMEM loads in flight and one wait,
// approximate keys, two independent three-input min trees that reject the 64
// columns in the common case, and the exact per-column test and insertion
// otherwise. The first 32 columns of every step go to list A, the second 32
// to list B (A and B may be the same list). taddr: the lane's TMEM address of
// column 0; slot: 32 floats of this thread in shared memory, touched only on
// the rare path.
template <int CAP, bool L2, int NCOL>
__device__ __forceinline__ void drain_columns(TopList<CAP>& A, TopList<CAP>& B, uint32_t taddr, int64_t row0,
                                              int valid_cols, const GemmTopkArgs& p, float* slot) {
  static_assert(NCOL % 64 == 0, "columns are drained 64 at a time");
#pragma unroll 1
  for (int c = 0; c < NCOL / 64; ++c) {
    __syncwarp();  // tcgen05.ld is .sync.aligned
    uint32_t v0[32], v1[32];
    tc::tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c * 64), v0);
    tc::tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c * 64 + 32), v1);
    tc::tmem_ld_wait();
    const int64_t rbase = row0 + c * 64;
    const int nvalid = valid_cols - c * 64;
    if (nvalid <= 0) continue;
    const bool whole = nvalid >= 64 && p.mask_bits == nullptr;
    float m0, m1;
    if (!L2) {
      // Inner product: the keys are -v, and -max(v) == min(-v) exactly, so
      // the common case needs no negated keys at all.
      m0 = -max32u(v0);
      m1 = -max32u(v1);
      if (whole && !(m0 <= A.thr_key) && !(m1 <= B.thr_key)) continue;
    }
    float k0[32], k1[32];
    chunk_keys<L2>(v0, p, rbase, k0);
    chunk_keys<L2>(v1, p, rbase + 32, k1);
    // Common case: nothing in the 64 columns beats its list's threshold.
    // Partial or filtered steps take the exact per-column test; otherwise
    // only a half whose minimum can pass does.
    if (L2) {
      m0 = min32(k0);
      m1 = min32(k1);
      if (whole && !(m0 <= A.thr_key) && !(m1 <= B.thr_key)) continue;
    }
    uint32_t pass0 = 0, pass1 = 0;
    if (!whole || m0 <= A.thr_key) {
#pragma unroll
      for (int j = 0; j < 32; ++j) pass0 |= (k0[j] <= A.thr_key ? 1u : 0u) << j;
    }
    if (!whole || m1 <= B.thr_key) {
#pragma unroll
      for (int j = 0; j < 32; ++j) pass1 |= (k1[j] <= B.thr_key ? 1u : 0u) << j;
    }
    pass0 &= low_bits(nvalid);
    pass1 &= low_bits(nvalid - 32);
    if (p.mask_bits) {  // rbase is a multiple of 64
      pass0 &= __ldg(p.mask_bits + (rbase >> 5));
      pass1 &= __ldg(p.mask_bits + (rbase >> 5) + 1);
    }
    // Rare path. In a whole block a single passing column is the block's
    // minimum (it passes whenever anything does), whose key m is already at
    // hand: insert it directly. Otherwise the half's keys go through this
    // thread's shared-memory slot so they can be indexed.
    if (pass0) {
      if (whole && (pass0 & (pass0 - 1)) == 0) {
        insert_one<CAP>(A, m0, rbase + __ffs(pass0) - 1);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) slot[j] = k0[j];
        insert_passing<CAP>(A, pass0, slot, rbase);
      }
    }
    if (pass1) {
      if (whole && (pass1 & (pass1 - 1)) == 0) {
        insert_one<CAP>(B, m1, rbase + 32 + __ffs(pass1) - 1);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) slot[j] = k1[j];
        insert_passing<CAP>(B, pass1, slot, rbase + 32);
      }
    }
  }
}

template <int CAP, bool L2, int QT, int KIND>
__global__ void __launch_bounds__(Tile<QT, KIND>::THREADS, 1)
gemm_topk_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_x,
                 const GemmTopkArgs p) {
  using TL = Tile<QT, KIND>;
  constexpr bool IL = TL::IL;
  constexpr bool SW128 = KIND != kPassTf32;
  constexpr int BN = TL::BN;
  constexpr int STAGES = TL::STAGES;
  constexpr int STAGE_BYTES = TL::STAGE_BYTES;
  constexpr int B_OFF = QT * TL::A_TILE;  // base tile after the QT query tiles
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + TL::NBARS);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  float* s_keys = reinterpret_cast<float*>(s_tmem + 4);  // (128 * QT) x 33 epilogue key slots

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t smem_base = tc::smem_addr(smem);
  auto full_bar = [&](int s) { return tc::smem_addr(&bars[s]); };
  auto empty_bar = [&](int s) { return tc::smem_addr(&bars[STAGES + s]); };
  auto tfull_bar = [&](int a) { return tc::smem_addr(&bars[2 * STAGES + a]); };
  auto tempty_bar = [&](int a) { return tc::smem_addr(&bars[2 * STAGES + 2 + a]); };
  const uint32_t done_bar = tc::smem_addr(&bars[2 * STAGES + 4]);

  const bool q_lo = IL && *p.q_lo_flag != 0;
  const bool x_lo = IL && p.x_lo_nonzero != 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(full_bar(s), 1);
      tc::mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(tfull_bar(a), 1);
      tc::mbar_init(tempty_bar(a), 4 * QT);
    }
    tc::mbar_init(done_bar, 1);
    *s_abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tm_q);
    tc::prefetch_tmap(&tm_x);
  }
  if (warp == 1) {
    tc::tmem_alloc(tc::smem_addr(s_tmem), kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  const int KC = TL::BF ? p.ldb / TL::KEL : p.ld / TL::KEL;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) {
        issued[s] = false;
        issued_phase[s] = 0;
      }
      const uint32_t bytes = STAGE_BYTES;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        const int qp = item % p.T;  // group of QT query tiles
        const int split = item / p.T;
        const int t0 = split * p.split_stride;
        const int t1 = min(p.nb, t0 + p.tiles_per_split);
        for (int t = t0; ok && t < t1; ++t) {
          for (int kc = 0; kc < KC; ++kc) {
            if (!tc::mbar_wait(empty_bar(stage), phase ^ 1, s_abort)) {
              ok = false;
              break;
            }
            const uint32_t sbase = smem_base + stage * STAGE_BYTES;
            tc::mbar_arrive_expect_tx(full_bar(stage), bytes);
            // Slice kc starts at column 32*kc of an interleaved tf32 row, or
            // 64*kc of a bf16 row.
#pragma unroll
            for (int q = 0; q < QT; ++q)
              tc::tma_load_2d(sbase + q * TL::A_TILE, &tm_q, full_bar(stage), kc * TL::KCOORD,
                              (qp * QT + q) * BM);
            tc::tma_load_2d(sbase + B_OFF, &tm_x, full_bar(stage), kc * TL::KCOORD, t * BN);
            issued[stage] = true;
            issued_phase[stage] = phase;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      // Every issued load must land before this CTA's shared memory goes away.
#pragma unroll
      for (int s = 0; s < STAGES; ++s)
        if (issued[s]) mbar_wait_quiet(full_bar(s), issued_phase[s]);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = TL::BF ? tc::idesc_bf16(BM, BN) : tc::idesc_tf32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
        const int split = item / p.T;
        const int t0 = split * p.split_stride;
        const int t1 = min(p.nb, t0 + p.tiles_per_split);
        for (int t = t0; ok && t < t1; ++t) {
          if (!tc::mbar_wait(tempty_bar(acc), acc_phase ^ 1, s_abort)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          for (int kc = 0; kc < KC; ++kc) {
            if (!tc::mbar_wait(full_bar(stage), phase, s_abort)) {
              ok = false;
              break;
            }
            tc::tc_fence_after();
            const uint32_t sbase = smem_base + stage * STAGE_BYTES;
            const uint64_t b_desc =
                SW128 ? tc::sw128_kmajor_desc(sbase + B_OFF) : tc::sw64_kmajor_desc(sbase + B_OFF);
#pragma unroll
            for (int q = 0; q < QT; ++q) {
              const uint32_t d_tmem = tmem_base + static_cast<uint32_t>((acc * QT + q) * BN);
              const uint32_t a_addr = sbase + q * TL::A_TILE;
              const uint64_t a_desc = SW128 ? tc::sw128_kmajor_desc(a_addr) : tc::sw64_kmajor_desc(a_addr);
              if constexpr (TL::BF) {
                // Four K steps of 16 bf16 values (32 bytes) per 128-byte row.
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                  const uint64_t off = static_cast<uint64_t>(kk * 32) >> 4;
                  tc::mma_bf16(d_tmem, a_desc + off, b_desc + off, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
                }
              } else {
#pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                  // Descriptor start addresses move in 16-byte units: K step kk
                  // of the hi half sits at 32*kk bytes, of the lo half 64 later.
                  const uint64_t hi = static_cast<uint64_t>(kk * 32) >> 4;
                  const uint64_t lo = static_cast<uint64_t>(64 + kk * 32) >> 4;
                  const uint32_t accumulate = (kc > 0 || kk > 0) ? 1u : 0u;
                  tc::mma_tf32(d_tmem, a_desc + hi, b_desc + hi, idesc, accumulate);
                  if (IL) {
                    if (x_lo) tc::mma_tf32(d_tmem, a_desc + hi, b_desc + lo, idesc, 1u);
                    if (q_lo) tc::mma_tf32(d_tmem, a_desc + lo, b_desc + hi, idesc, 1u);
                  }
                }
              }
            }
            tc::mma_commit(empty_bar(stage));
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          tc::mma_commit(tfull_bar(acc));
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
      }
      // All issued MMAs must be complete before TMEM is released.
      tc::mma_commit(done_bar);
      mbar_wait_quiet(done_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int wg = (warp - 2) >> 2;  // which query tile of the group
    const int quarter = warp & 3;    // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    float* slot = s_keys + (wg * 128 + row_in_tile) * 33;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
      const int qp = item % p.T;
      const int split = item / p.T;
      const int t0 = split * p.split_stride;
      const int t1 = min(p.nb, t0 + p.tiles_per_split);
      const int64_t qidx = static_cast<int64_t>(qp * QT + wg) * BM + row_in_tile;
      TopList<CAP> T;
      T.reset(list_start_key(p, qidx));
      for (int t = t0; t < t1; ++t) {
        // Warp-uniform decision: the tcgen05.ld below is .sync.aligned.
        const bool got = __all_sync(0xffffffffu, tc::mbar_wait(tfull_bar(acc), acc_phase, s_abort));
        if (!got) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const int64_t row0 = static_cast<int64_t>(t) * BN;
        // Columns of this tile that are real rows (the last tile may be short).
        const int valid_cols = p.n - row0 < BN ? static_cast<int>(p.n - row0) : BN;
        const uint32_t col0 = static_cast<uint32_t>((acc * QT + wg) * BN);
        drain_columns<CAP, L2, BN>(T, T, lane_addr + col0, row0, valid_cols, p, slot);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(tempty_bar(acc));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) break;
      list_sort<CAP>(T.L);
      if (qidx < p.nq) {
        uint64_t* out = p.partial + (qidx * p.S + split) * CAP;
#pragma unroll
        for (int j = 0; j < CAP; ++j) out[j] = T.L[j];
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem_base, kTmemCols);
  if (threadIdx.x == 0 && *s_abort) atomicOr(p.err, 1);
}

// ---------------------------------------------------------------------------
// The bf16 pass on CTA pairs (tcgen05 cta_group::2).
//
// A cluster of two CTAs computes 256 queries x 256 base rows per tile: each
// CTA stages its 128 query rows and 128 of the base rows (K slices of 64 bf16
// values, 128-byte swizzle), and the even CTA issues M = 256, N = 256 MMAs
// that read both CTAs' shared memory and write each CTA's TMEM (its 128
// queries x 256 columns). Per CTA that is 256 staged rows for 128 x 256
// outputs, against 384 rows for 256 x 128 outputs in the single-CTA kernel:
// 1.5x less operand traffic from L2 per output.
//
// Barriers (no TMA load uses multicast; the even CTA's tcgen05.commit signals
// the barrier at the same offset in both CTAs):
//   full[s]   even CTA; armed by its producer for both CTAs' bytes, and both
//             CTAs' TMA loads complete on it
//   empty[s]  each CTA; stage s consumed by the MMAs
//   tfull[a]  each CTA; accumulator a holds a finished tile
//   tempty[a] even CTA; 16 arrivals, the 8 epilogue warps of each CTA
//   done      each CTA; every MMA has completed
// Each CTA's two epilogue warpgroups drain 128 columns each of every tile, and
// each thread keeps two lists over alternate 32-column blocks, so every
// (query, split) has four lists. The epilogue's rare insertion path
// indexes its keys through a 33-float shared-memory slot per thread (local
// memory spilled to DRAM on config 4's frequent refills). A seventh stage,
// or prefetching base slices into L2 ahead of the ring, measured slower.
namespace pairk {
constexpr int PM = 128;                         // query rows per CTA (TMEM lanes)
constexpr int PH = 128;                         // base rows staged per CTA
constexpr int ROW = 128;                        // bytes per row per stage: 64 bf16
constexpr int STAGES = 6;
constexpr int A_TILE = PM * ROW;                // 16 KB
constexpr int STAGE_BYTES = A_TILE + PH * ROW;  // 32 KB
constexpr int NBARS = 2 * STAGES + 2 + 2 + 1;
constexpr int THREADS = 64 + 256;
constexpr size_t SMEM = 1024 + STAGES * STAGE_BYTES + NBARS * 8 + 16 + 256 * 33 * 4;
}  // namespace pairk

// Largest k the bf16 pass serves (its candidates then number 256, the most
// the rescoring takes; beyond, the bf16 bound is too wide to certify).
constexpr int kPairMaxK = 100;

template <bool L2, int CAP>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pairk::THREADS, 1)
gemm_topk_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_x,
                      const GemmTopkArgs p) {
  using namespace pairk;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  float* s_keys = reinterpret_cast<float*>(s_tmem + 4);  // 256 x 33 epilogue key slots

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t smem_base = tc::smem_addr(smem);
  auto full_bar = [&](int s) { return tc::smem_addr(&bars[s]); };
  auto empty_bar = [&](int s) { return tc::smem_addr(&bars[STAGES + s]); };
  auto tfull_bar = [&](int a) { return tc::smem_addr(&bars[2 * STAGES + a]); };
  auto tempty_bar = [&](int a) { return tc::smem_addr(&bars[2 * STAGES + 2 + a]); };
  const uint32_t done_bar = tc::smem_addr(&bars[2 * STAGES + 4]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(full_bar(s), 1);
      tc::mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(tfull_bar(a), 1);
      tc::mbar_init(tempty_bar(a), 16);
    }
    tc::mbar_init(done_bar, 1);
    *s_abort = 0;
    tc::fence_mbarrier_init_cluster();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tm_q);
    tc::prefetch_tmap(&tm_x);
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(tc::smem_addr(s_tmem), kTmemCols);
    tc::tmem_relinquish_pair();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // both CTAs' barriers are initialised before any use
  tc::tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int KC = p.ldb / 64;
  const int cluster = static_cast<int>(tc::cluster_id_x());
  const int nclusters = static_cast<int>(tc::nclusters_x());

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) {
        issued[s] = false;
        issued_phase[s] = 0;
      }
      bool ok = true;
      for (int item = cluster; ok && item < p.n_items; item += nclusters) {
        const int qg = item % p.T;
        const int split = item / p.T;
        const int t0 = split * p.split_stride;
        const int t1 = min(p.nb, t0 + p.tiles_per_split);
        for (int t = t0; ok && t < t1; ++t) {
          for (int kc = 0; kc < KC; ++kc) {
            if (!tc::mbar_wait(empty_bar(stage), phase ^ 1, s_abort)) {
              ok = false;
              break;
            }
            const uint32_t sbase = smem_base + stage * STAGE_BYTES;
            const uint32_t fb = tc::mapa_shared(full_bar(stage), 0);
            if (leader) tc::mbar_arrive_expect_tx(full_bar(stage), 2 * STAGE_BYTES);
            tc::tma_load_2d_pair(sbase, &tm_q, fb, kc * 64, qg * 256 + static_cast<int>(rank) * PM);
            tc::tma_load_2d_pair(sbase + A_TILE, &tm_x, fb, kc * 64, t * 256 + static_cast<int>(rank) * PH);
            issued[stage] = true;
            issued_phase[stage] = phase;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      // Both CTAs' loads complete on the even CTA's barriers: it waits for
      // every phase it armed before shared memory goes away; the odd CTA
      // leaves only after the closing cluster barrier.
      if (leader) {
#pragma unroll
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait_quiet(full_bar(s), issued_phase[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16(2 * PM, 2 * PH);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int item = cluster; ok && item < p.n_items; item += nclusters) {
        const int split = item / p.T;
        const int t0 = split * p.split_stride;
        const int t1 = min(p.nb, t0 + p.tiles_per_split);
        for (int t = t0; ok && t < t1; ++t) {
          if (!tc::mbar_wait(tempty_bar(acc), acc_phase ^ 1, s_abort)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * 2 * PH);
          for (int kc = 0; kc < KC; ++kc) {
            if (!tc::mbar_wait(full_bar(stage), phase, s_abort)) {
              ok = false;
              break;
            }
            tc::tc_fence_after();
            const uint32_t sbase = smem_base + stage * STAGE_BYTES;
            const uint64_t a_desc = tc::sw128_kmajor_desc(sbase);
            const uint64_t b_desc = tc::sw128_kmajor_desc(sbase + A_TILE);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t off = static_cast<uint64_t>(kk * 32) >> 4;
              tc::mma_bf16_pair(d_tmem, a_desc + off, b_desc + off, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
            }
            tc::mma_commit_pair_both(empty_bar(stage));
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          tc::mma_commit_pair_both(tfull_bar(acc));
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
      }
      // Every issued MMA completes before either CTA releases TMEM or
      // shared memory.
      tc::mma_commit_pair_both(done_bar);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int half = (warp - 2) >> 2;  // which 128 columns of each tile
    const int quarter = warp & 3;      // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    float* slot = s_keys + (half * 128 + row_in_tile) * 33;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int item = cluster; ok && item < p.n_items; item += nclusters) {
      const int qg = item % p.T;
      const int split = item / p.T;
      const int t0 = split * p.split_stride;
      const int t1 = min(p.nb, t0 + p.tiles_per_split);
      const int64_t qidx = static_cast<int64_t>(qg) * (2 * PM) + static_cast<int64_t>(rank) * PM + row_in_tile;
      // Two lists, over alternate 32-column blocks: the same number of
      // insertions as one list of twice the size, each at half the cost.
      const float start_key = list_start_key(p, qidx);
      TopList<CAP> TA, TB;
      TA.reset(start_key);
      TB.reset(start_key);
      for (int t = t0; t < t1; ++t) {
        const bool got = __all_sync(0xffffffffu, tc::mbar_wait(tfull_bar(acc), acc_phase, s_abort));
        if (!got) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const int64_t row0 = static_cast<int64_t>(t) * (2 * PH) + half * PH;
        if (L2 && t + 1 < t1 && lane < PH / 32) {
          // The next tile's 128 norms (four 128-byte lines, inside the
          // norms' 256-row padding) into L1, so the key computation of the
          // next tile does not wait on L2.
          const float* nx = p.norms + row0 + 2 * PH + lane * 32;
          asm volatile("prefetch.global.L1 [%0];" ::"l"(nx));
        }
        const int64_t rem = p.n - row0;
        const int valid_cols = rem < PH ? (rem < 0 ? 0 : static_cast<int>(rem)) : PH;
        const uint32_t col0 = static_cast<uint32_t>(acc * 2 * PH + half * PH);
        drain_columns<CAP, L2, PH>(TA, TB, lane_addr + col0, row0, valid_cols, p, slot);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cluster(tc::mapa_shared(tempty_bar(acc), 0));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) break;
      list_sort<CAP>(TA.L);
      list_sort<CAP>(TB.L);
      if (qidx < p.nq) {
        uint64_t* out = p.partial + ((qidx * p.S + split) * 2 + half) * 2 * CAP;
#pragma unroll
        for (int j = 0; j < CAP; ++j) out[j] = TA.L[j];
#pragma unroll
        for (int j = 0; j < CAP; ++j) out[CAP + j] = TB.L[j];
      }
    }
  }

  if (warp == 1 && lane == 0) mbar_wait_quiet(done_bar, 0);
  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // neither CTA leaves while the pair's MMAs or loads may touch it
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc_pair(tmem_base, kTmemCols);
  if (threadIdx.x == 0 && *s_abort) atomicOr(p.err, 1);
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

template <bool L2, int CAP>
cudaError_t launch_pair(const GemmTopkArgs& a, const CUtensorMap* maps, int grid, cudaStream_t stream) {
  auto kern = gemm_topk_pair_kernel<L2, CAP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(pairk::SMEM));
  if (e != cudaSuccess) return e;
  if (grid < 2 || grid % 2 != 0) return cudaErrorInvalidValue;
  kern<<<grid, pairk::THREADS, pairk::SMEM, stream>>>(maps[0], maps[1], a);
  return cudaGetLastError();
}

template <int CAP, bool L2, int QT, int KIND>
cudaError_t launch_typed(const GemmTopkArgs& a, const CUtensorMap* maps, int grid, cudaStream_t stream) {
  using TL = Tile<QT, KIND>;
  auto kern = gemm_topk_kernel<CAP, L2, QT, KIND>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(TL::SMEM));
  if (e != cudaSuccess) return e;
  kern<<<grid, TL::THREADS, TL::SMEM, stream>>>(maps[0], maps[1], a);
  return cudaGetLastError();
}

}  // namespace

// An interleaved split plane [rows x 2*ld] as a TMA tensor. il: boxes of 32
// floats (a whole [hi|lo] chunk, 128 bytes, 128-byte swizzle); otherwise 16
// floats (the hi half, 64 bytes, 64-byte swizzle). Rows past the end read as
// zeros.
cudaError_t encode_split_map(CUtensorMap* map, const float* plane, int64_t rows, int ld, int box_rows,
                             bool il) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = get_encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (rows < 1) rows = 1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(2 * ld), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(2 * ld) * sizeof(float)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(il ? 32 : 16), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(plane), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  il ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// A bf16 plane [rows x ldb] as a TMA tensor: boxes of 64 values (128 bytes,
// 128-byte swizzle) by box_rows rows. Rows past the end read as zeros.
cudaError_t encode_bf16_map(CUtensorMap* map, const void* plane, int64_t rows, int ldb, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = get_encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (rows < 1) rows = 1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(ldb), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldb) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(plane), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Candidates per list of the pair kernel; every (query, split, column half)
// has two lists, over alternate 32-column blocks. A list over R rows refills
// ~CAP * (1 + ln(R / CAP)) times at a cost linear in CAP, so two lists of CAP
// refill as often as one of 2 * CAP at half the cost per refill, while the
// merge needs only the best few per query from each of ~300 lists: 2 x 8
// keeps every k <= 16 certifiable unless 9 of a query's neighbours share one
// list (the certificate then sends the query on), larger k keep 2 x 16.
int gemm_pair_cap(int k) { return k <= 16 ? 8 : 16; }

// Candidates rescored per query after a bf16 pass. The certificate compares
// the k-th exact key with the largest approximate key among them, so more
// candidates widen the margin it can prove. On config 4's distribution
// (unit-norm rows, d = 768: a bound of 0.0039 on average; 20,000 simulated
// queries each): k = 10 leaves 0.08% uncertified with 32 and none with 64;
// k = 32 leaves 4.3% with 64 and none with 128; k = 50 none with 128;
// k = 100 56% with 160 and none with 256.
int gemm_pair_cands(int k) {
  if (k > kPairMaxK) return 0;
  if (k <= 16) return 64;
  if (k <= 50) return 128;
  return 256;
}


int gemm_pair_clusters(int device) {
  static int cached[64] = {};
  if (device < 0 || device >= 64) return 1;
  if (cached[device] > 0) return cached[device];
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  int clusters = 0;
  auto kern = gemm_topk_pair_kernel<false, 8>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pairk::SMEM)) ==
      cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sms / 2 * 2), 1, 1);
    cfg.blockDim = dim3(pairk::THREADS, 1, 1);
    cfg.dynamicSmemBytes = pairk::SMEM;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) clusters = 0;
  }
  cudaGetLastError();
  if (clusters <= 0) clusters = sms / 2;
  cached[device] = clusters;
  return clusters;
}

int gemm_cap_for(int k) {
  if (k <= 16) return 32;
  if (k <= 224) return 64;
  return 0;
}

// Candidates rescored per query after a tf32 pass (see gemm_pair_cands).
int gemm_cands_for(int k) {
  if (k <= 40) return 64;
  if (k <= 224) return (k + 32 + 31) / 32 * 32;
  return 0;
}

int gemm_qt_for(int k) { return gemm_cap_for(k) == 32 ? 2 : 1; }

int gemm_bn_for(int k) { return 256 / gemm_qt_for(k); }

cudaError_t launch_gemm_topk(const GemmTopkArgs& a, const void* q_plane, int64_t q_rows,
                             const void* x_plane, PassKind kind, int grid, cudaStream_t stream) {
  if (a.ld % 32 != 0 || a.ldb % 64 != 0) return cudaErrorInvalidValue;
  const int qt = gemm_qt_for(a.k);
  const int cap = gemm_cap_for(a.k);
  CUtensorMap maps[2];
  cudaError_t e;
  if (kind == kPassBf16) {
    // CTA pairs: each CTA stages 128 query rows and 128 base rows per slice.
    if (a.k > kPairMaxK) return cudaErrorInvalidValue;
    e = encode_bf16_map(&maps[0], q_plane, q_rows, a.ldb, pairk::PM);
    if (e == cudaSuccess) e = encode_bf16_map(&maps[1], x_plane, a.n, a.ldb, pairk::PH);
    if (e != cudaSuccess) return e;
    if (gemm_pair_cap(a.k) == 8)
      return a.l2 ? launch_pair<true, 8>(a, maps, grid, stream) : launch_pair<false, 8>(a, maps, grid, stream);
    return a.l2 ? launch_pair<true, 16>(a, maps, grid, stream) : launch_pair<false, 16>(a, maps, grid, stream);
  } else {
    const bool il = kind == kPass3xTf32;
    e = encode_split_map(&maps[0], static_cast<const float*>(q_plane), q_rows, a.ld, BM, il);
    if (e == cudaSuccess) e = encode_split_map(&maps[1], static_cast<const float*>(x_plane), a.n, a.ld, 256 / qt, il);
  }
  if (e != cudaSuccess) return e;
  if (cap == 32) {
    switch (kind) {
      case kPass3xTf32:
        return a.l2 ? launch_typed<32, true, 2, kPass3xTf32>(a, maps, grid, stream)
                    : launch_typed<32, false, 2, kPass3xTf32>(a, maps, grid, stream);
      case kPassTf32:
        return a.l2 ? launch_typed<32, true, 2, kPassTf32>(a, maps, grid, stream)
                    : launch_typed<32, false, 2, kPassTf32>(a, maps, grid, stream);
    }
  }
  if (cap == 64) {
    if (kind == kPass3xTf32)
      return a.l2 ? launch_typed<64, true, 1, kPass3xTf32>(a, maps, grid, stream)
                  : launch_typed<64, false, 1, kPass3xTf32>(a, maps, grid, stream);
    if (kind == kPassTf32)
      return a.l2 ? launch_typed<64, true, 1, kPassTf32>(a, maps, grid, stream)
                  : launch_typed<64, false, 1, kPassTf32>(a, maps, grid, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace px
