// Launch interfaces of the proxima_b200 kernels (internal to the library).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace px {

// ---- K2: exact streaming scan (k_exact.cu) --------------------------------
struct ExactScanArgs {
  const float* base;       // shard rows, row stride ld floats
  int64_t n;               // rows in the shard
  int ld;                  // row stride (floats), multiple of 4
  int d;                   // dimension
  const float* queries;    // nq x d, contiguous
  int nq;
  int k;
  int group;               // queries per CTA: 1, 2, 4 or 8
  int ncta;                // row splits (gridDim.x)
  int64_t rows_per_cta;
  const uint8_t* mask;     // optional per-row filter (nonzero = keep)
  bool l2;
  uint64_t* partial;       // [nq][ncta][k] sorted candidate lists
};
cudaError_t launch_exact_scan(const ExactScanArgs& a, cudaStream_t stream);
int exact_max_k();
// Queries per CTA for nq queries: 1, 2, 4 or 8, the largest whose shared
// memory (exact_smem_for) fits smem_limit bytes; 0 when even one does not.
int exact_group_for(int64_t nq, int k, int d, size_t smem_limit);
int exact_buf_for(int k);
size_t exact_smem_for(int group, int k, int d);

// ---- merges and output (k_merge.cu) ---------------------------------------
// Selects, per query, the k smallest of `nlists` sorted lists of packed
// candidates ([nq][nlists][list_len], PX_EMPTY-padded) into out [nq][k].
cudaError_t launch_merge_lists(const uint64_t* lists, int64_t nq, int nlists, int list_len, int k,
                               uint64_t* out, cudaStream_t stream);

// Converts packed candidates [nq][k] into caller ids / distances.
// natural: sqrt / negate as FlatIndex::scan reports (flat.rs:139-147);
// otherwise key space (squared L2, negated IP) as knn_gpu_search reports.
// Row -> global id through `nseg` segments (local_begin, global_begin) sorted
// by local_begin, plus id_offset.
struct IdSegments {
  const int64_t* local_begin;  // device, nseg
  const int64_t* global_begin; // device, nseg
  int nseg;
  int64_t id_offset;
};
cudaError_t launch_emit(const uint64_t* cands, int64_t nq, int k, bool l2, bool natural,
                        IdSegments segs, int64_t* out_ids, float* out_dists,
                        cudaStream_t stream);

// Cross-shard merge (K6): G sorted lists per query of (key, global id) pairs,
// layout [G][nq][k] in key space. Ties on key break by the smaller global id.
// Writes natural or key-space distances.
cudaError_t launch_merge_shards(const float* keys, const int64_t* ids, int nshard, int64_t nq,
                                int k, bool l2, bool natural, float* out_dists, int64_t* out_ids,
                                cudaStream_t stream);
// The same with shard g's keys at (char*)keys + g * key_stride and its ids at
// (char*)ids + g * id_stride (byte strides), e.g. records gathered by one
// collective.
cudaError_t launch_merge_shards_strided(const float* keys, int64_t key_stride, const int64_t* ids,
                                        int64_t id_stride, int nshard, int64_t nq, int k, bool l2, bool natural,
                                        float* out_dists, int64_t* out_ids, cudaStream_t stream);

// ---- PQ (k_pq.cu) ---------------------------------------------------------
// ADC tables (pq.rs:123-136): lut [nq][m][ksub].
cudaError_t launch_pq_lut(const float* books, int m, int ksub, int dsub, bool l2,
                          const float* queries, int nq, float* lut, cudaStream_t stream);

struct PqScanArgs {
  const uint8_t* codes;    // n x m
  int64_t n;
  int m;
  int ksub;
  const float* lut;        // [nq][m][ksub]
  int nq;
  int k;
  int group;               // queries per CTA
  int ncta;
  int64_t rows_per_cta;
  const uint8_t* mask;
  uint64_t* partial;       // [nq][ncta][k]
};
cudaError_t launch_pq_scan(const PqScanArgs& a, cudaStream_t stream);
int pq_group_for(int m, int ksub, int64_t nq, int k);
size_t pq_smem_for(int group, int m, int ksub, int k);
// Rows one scan iteration covers; a CTA's row range is a multiple of it.
int pq_rows_per_iter(int group, int m, int ksub, int k);
int pq_max_k();

// Nearest centroid per (vector, subspace) with the reference's strict '<'
// first-wins rule (pq.rs:107-121, 155-167). vectors: n x (m*dsub).
cudaError_t launch_nearest_centroid(const float* vectors, int64_t n, int m, int dsub, int ksub,
                                    const float* books, uint32_t* out_assign, uint8_t* out_codes,
                                    cudaStream_t stream);

// ---- shard preparation (k_prep.cu) ----------------------------------------
// Copies n rows of d floats into the shard (stride ld, zero padded), and
// writes the interleaved tf32 split plane `hl` (stride 2*ld: per 16-element
// chunk 16 hi values then 16 lo values), the bf16 plane `xb` (stride ldb, a
// multiple of 64) and the squared norms; any output may be null. lo_nonzero
// is raised when any lo element is nonzero, bf_inexact when any value
// differs from its bf16 rounding; max_norm_sq (float bits) is raised to the
// largest squared norm.
// Shard rows (norms non-null) also carry their squared norm, split exactly
// into three bf16 values, in bf16 columns d..d+2 when d + 3 <= ldb.
// resid (optional, two words of float bits): raised to upper bounds on the
// largest ||x - bf16(x)|| and ||x - tf32_hi(x)|| of the rows.
cudaError_t launch_prepare_rows(const float* src, int64_t n, int d, int ld, int ldb, float* dst, float* hl,
                                void* xb, float* norms, int* lo_nonzero, int* bf_inexact, int* max_norm_sq,
                                cudaStream_t stream, bool fold_query = false, int* resid = nullptr);
// Split plane and bf16 plane of nq query rows (either may be null),
// zero-filled up to rows_alloc rows. fold_l2: the bf16 rows hold 2q and -1 in
// columns d..d+2, so their product with a shard row is -(||x||^2 - 2 q.x).
cudaError_t launch_split_queries(const float* q, int64_t nq, int d, int ld, int ldb, int64_t rows_alloc,
                                 float* hl, void* qb, int* lo_nonzero, int* bf_inexact, cudaStream_t stream,
                                 bool fold_l2 = false);

// What a tensor-core candidate pass multiplies.
enum PassKind : int {
  kPass3xTf32 = 0,  // hi.hi + hi.lo + lo.hi of the tf32 split planes (~fp32)
  kPassTf32 = 1,    // hi.hi only
  kPassBf16 = 2,    // the bf16 planes
};

// ---- K1: tensor-core candidate generation (k_gemm.cu) ---------------------
struct GemmTopkArgs {
  int nq;
  int64_t n;            // shard rows
  int ld;               // row stride (floats), multiple of 32
  int ldb;              // bf16 plane row stride (elements), multiple of 64
  int k;
  int T;                // groups of gemm_qt_for(k) query tiles of 128
  int S;                // base splits
  int tiles_per_split;  // base tiles of gemm_bn_for(k) rows per split
  int split_stride;     // base tiles from one split's first tile to the next's
                        // (tiles_per_split, or more for a strided sample)
  int nb;               // base tiles
  int n_items;          // T * S
  bool l2;
  const float* norms;   // squared norms (L2)
  int x_lo_nonzero;     // shard lo plane in use
  const int* q_lo_flag; // device word: query lo plane in use
  uint64_t* partial;    // [nq][S][cap] sorted approximate candidates
  int* err;             // device word raised on a timed-out wait
  const uint32_t* mask_bits;  // optional filter, one bit per row (1 = may be returned)
  // Optional starting threshold per query ([nq][seed_k] sorted words of a
  // sample pass, seed_k >= k; its last word's key): the lists admit only
  // keys <= it. Null: every list starts open.
  const uint64_t* seed;
  int seed_k;
};
// Packs a byte mask (nonzero = keep) into one bit per row, 32 rows per word.
cudaError_t launch_pack_mask(const uint8_t* mask, int64_t n, uint32_t* bits, cudaStream_t stream);
int gemm_cap_for(int k);    // candidates kept per (query, split) in registers (0: unsupported)
int gemm_cands_for(int k);  // candidates per query after the split merge (<= 256)
int gemm_qt_for(int k);   // query tiles of 128 per CTA (2 for k <= 16, else 1)
int gemm_bn_for(int k);   // base rows per tile (256 / qt)
// CTA pairs of the bf16 pass's kernel that fit on `device` at once (each
// pair takes 256 queries x 256 base rows per tile, four lists per split).
int gemm_pair_clusters(int device);
int gemm_pair_cap(int k);    // candidates per list of the pair kernel (the bf16 pass)
int gemm_pair_cands(int k);  // candidates per query after a bf16 pass (0: k too large for it)
// q_plane / x_plane: the interleaved split planes (stride 2*ld) for the tf32
// passes, the bf16 planes (stride ldb) for kPassBf16, which serves
// gemm_pair_cands(k) > 0 only and runs on CTA pairs: grid is then an even
// number of CTAs, T counts groups of 256 queries, nb tiles of 256 rows, and
// partial holds four lists per split ([nq][S][2 column halves][2][cap]).
// kPassTf32 reads only
// the hi halves.
cudaError_t launch_gemm_topk(const GemmTopkArgs& a, const void* q_plane, int64_t q_rows,
                             const void* x_plane, PassKind kind, int grid, cudaStream_t stream);

// ---- K5: exact rescoring + certificate (k_rescore.cu) ---------------------
struct RescoreArgs {
  const uint64_t* merged;  // [nq][cap] sorted approximate candidates
  int64_t nq;
  int cap;                 // candidates per query (<= 256)
  int k;
  const uint64_t* lists;   // [nq][nlists][list_cap] per-split lists (for the bound)
  int nlists;
  int list_cap;
  const float* queries;    // nq x d
  const float* base;       // shard fp32 rows, stride ld
  int ld;
  int d;
  bool l2;
  float max_norm_sq;       // max over the shard of the rows' fp32 squared norms
  float x_resid;           // upper bound on max ||x - x~|| over the shard, x~ the rows as
                           // the pass multiplies them (bf16, or tf32 hi values)
  int x_lo_nonzero;
  const int* q_lo_flag;
  int pass_kind;           // PassKind of the candidate pass
  int norm_folded;         // L2 keys came from bf16 rows carrying ||x||^2 (2 q.x - ||x||^2)
  const uint64_t* seed;    // [nq][seed_k] the candidate pass's starting thresholds, or null
  int seed_k;
  uint64_t* out;           // [nq][k] exact candidates
  int* status;             // [nq] 0 = certified
  int* n_fail;             // count of uncertified queries
  int* fail_list;          // their indices
};
cudaError_t launch_rescore(const RescoreArgs& a, cudaStream_t stream);
cudaError_t launch_gather_rows(const float* src, int d, const int* idx, int count, float* dst,
                               cudaStream_t stream);
cudaError_t launch_scatter_cands(const uint64_t* src, int k, const int* idx, int count,
                                 uint64_t* dst, cudaStream_t stream);

}  // namespace px
