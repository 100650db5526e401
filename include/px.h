/*
 * px.h -- C ABI of libproxima_b200.so, the B200 (sm_100a) implementation of
 * Proxima's exact-kNN and PQ asymmetric-distance hot path.
 *
 * Two groups of entry points:
 *
 *  1. knn_gpu_create / knn_gpu_search / knn_gpu_free: the exact signatures
 *     and return conventions of the reference's CUDA satellite
 *     (crates/core/cuda/knn.cu:123-180, bound by crates/core/src/gpu.rs:10-15),
 *     so gpu.rs links against this library unchanged. Unlike the reference
 *     kernel (k <= 46, knn.cu:5,145) any 1 <= k <= PX_MAX_K is accepted.
 *
 *  2. px_*: the handle-based ABI that FlatIndex / PqIndex dispatch to. Sizes
 *     are 64-bit, outputs are natural distances with the reference's padding
 *     (id -1; FLT_MAX for L2, -FLT_MAX for inner product), and every call
 *     returns a px_status with a thread-local message in px_last_error().
 *     No call aborts or throws across the boundary.
 *
 * Threading: a handle may be searched from several threads at once (an
 * internal mutex serialises them); add/destroy must not race with searches.
 * All host buffers stay owned by the caller; the library copies inputs.
 */
#ifndef PROXIMA_B200_PX_H
#define PROXIMA_B200_PX_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PX_API __attribute__((visibility("default")))

/* Largest k any search accepts (the exact scan's shared-memory buffer). */
#define PX_MAX_K 768

typedef int32_t px_status;
enum {
  PX_OK = 0,
  PX_EINVAL = 1,      /* bad argument; message names it */
  PX_ECUDA = 2,       /* CUDA runtime/driver error */
  PX_ENOMEM = 3,      /* device or pinned host allocation failed */
  PX_ESTATE = 4,      /* call not valid in the handle's state */
  PX_ENCCL = 5,       /* NCCL error (multi-GPU merge) */
  PX_ETIMEOUT = 6,    /* a bounded device-side wait gave up */
  PX_EUNSUPPORTED = 7 /* valid request this build cannot serve */
};

/* Metric codes match gpu.rs:62-65 (0 = L2, 1 = inner product). */
enum { PX_METRIC_L2 = 0, PX_METRIC_IP = 1 };

/* Thread-local message of the last failed px_* call on this thread. */
PX_API const char* px_last_error(void);
PX_API const char* px_version(void);
/* Number of visible CUDA devices (0 when none); never fails. */
PX_API int32_t px_device_count(void);

/* ------------------------------------------------------------------------
 * Reference-compatible ABI (crates/core/cuda/knn.cu:123-180).
 * ------------------------------------------------------------------------ */
typedef struct PxGpuIndex PxGpuIndex;

/* Replaces knn_gpu_create (knn.cu:123): copies n x dim row-major floats to
 * the current CUDA device. NULL on failure. */
PX_API PxGpuIndex* knn_gpu_create(const float* base, int n, int dim);

/* Replaces knn_gpu_search (knn.cu:143): host queries (nq x dim), writes
 * nq x k ids and KEY-SPACE values (squared L2, or -inner product; padding:
 * id -1, key FLT_MAX). Returns 0, -1 for an invalid k (k < 1 or
 * k > PX_MAX_K), or a positive cudaError_t value. */
PX_API int knn_gpu_search(const PxGpuIndex* idx, const float* queries, int nq, int k, int metric,
                          long long* out_ids, float* out_keys);

/* Replaces knn_gpu_free (knn.cu:176). NULL is a no-op. */
PX_API void knn_gpu_free(PxGpuIndex* idx);

/* ------------------------------------------------------------------------
 * FlatIndex (crates/core/src/flat.rs) on one or more GPUs.
 * ------------------------------------------------------------------------ */
typedef struct px_flat px_flat;

/* FlatIndex::new (flat.rs:43). devices: ndev CUDA ordinals the base is
 * row-sharded across (NULL/0 = the current device). */
PX_API px_status px_flat_create(int32_t dim, int32_t metric, const int32_t* devices, int32_t ndev,
                                px_flat** out);
PX_API px_status px_flat_destroy(px_flat* h);

/* FlatIndex::add (flat.rs:72): appends n host rows (n x dim); rejects
 * non-finite values. Each call splits its rows into contiguous runs, one per
 * device, so ids keep the insertion order. */
PX_API px_status px_flat_add(px_flat* h, const float* rows, int64_t n);

/* Appends n rows that already live in device memory on the handle's single
 * device (handles with ndev == 1 only). Rows are not checked for NaN/Inf. */
PX_API px_status px_flat_add_device(px_flat* h, const float* d_rows, int64_t n);

/* Pre-sizes every shard for `n_total` rows in all (split as px_flat_add
 * splits), so that later adds up to that size do not reallocate. */
PX_API px_status px_flat_reserve(px_flat* h, int64_t n_total);

PX_API int64_t px_flat_size(const px_flat* h);
PX_API int32_t px_flat_dim(const px_flat* h);
PX_API int32_t px_flat_metric(const px_flat* h);

/* Copies rows [start, start + count) in id order back to the host
 * (count x dim floats), e.g. to save the index. */
PX_API px_status px_flat_read_rows(const px_flat* h, int64_t start, int64_t count, float* out);

/* Kernel path for flat searches: AUTO picks the exact streaming scan for
 * small batches and the tensor-core path otherwise; EXACT and
 * TENSOR force one (TENSOR fails with PX_EUNSUPPORTED where it cannot serve
 * the request, e.g. k > 224). TENSOR_3XTF32 is TENSOR with the first
 * candidate pass in 3xTF32 (~fp32-accurate candidates) instead of bf16/tf32.
 * Masks work on every path. Results are identical on every path. */
enum { PX_PATH_AUTO = 0, PX_PATH_EXACT = 1, PX_PATH_TENSOR = 2, PX_PATH_TENSOR_3XTF32 = 3 };
PX_API px_status px_flat_set_path(px_flat* h, int32_t mode);

/* The bf16 pass's sample pass (a first pass over 32 base tiles spread over
 * the shard, whose per-query thresholds the main pass's lists start from):
 * AUTO runs it on shards of at least 128 tiles of 256 rows whose splits are
 * at least 512 tiles long; ON on every shard of at least 128 tiles; OFF
 * never. Results are identical either way. */
enum { PX_SAMPLE_AUTO = 0, PX_SAMPLE_OFF = 1, PX_SAMPLE_ON = 2 };
PX_API px_status px_flat_set_sample_pass(px_flat* h, int32_t mode);

/* Per-search instrumentation (off by default). With profiling on, the
 * dominant kernel of each search is bracketed by CUDA events on the
 * launching stream; px_flat_last_profile waits for them and reports. */
typedef struct px_search_profile {
  int32_t path;             /* 0 exact scan, 1 tensor-core path, 2 PQ ADC scan */
  int32_t launches;         /* kernels the search launched on the first shard */
  int32_t fallback_queries; /* queries the certificate sent to the exact scan */
  int32_t profiled;         /* 1 if main_kernel_ms is valid */
  float main_kernel_ms;     /* device time of the dominant kernel */
  int32_t refined_queries;  /* queries re-run by the three-pass tensor-core pass */
  int32_t first_pass;       /* tensor-core path: operands of the first candidate
                               pass, 0 three-pass tf32, 1 tf32, 2 bf16; else -1 */
  int32_t sample_tiles;     /* base tiles of the bf16 pass's sample pass, which
                               sets the lists' starting thresholds (0: none) */
} px_search_profile;
PX_API void px_set_profiling(int32_t enable);
PX_API px_status px_flat_last_profile(const px_flat* h, px_search_profile* out);
/* Totals over the handle's searches (first shard) since the last reset, so a
 * benchmark loop need not read the profile after every search. */
typedef struct px_profile_totals {
  double main_kernel_ms;      /* summed device time of the profiled searches' dominant kernel */
  int64_t profiled_searches;  /* searches with profiling on */
  int64_t searches;
  int64_t fallback_queries;
  int64_t refined_queries;
} px_profile_totals;
PX_API px_status px_flat_profile_totals(px_flat* h, int32_t reset, px_profile_totals* out);
/* Total kernels launched by this library in this process. */
PX_API int64_t px_launch_count(void);

/* Adds `offset` to every id the handle returns (for a rank that holds rows
 * [offset, offset + size) of a base sharded across processes). */
PX_API px_status px_flat_set_id_offset(px_flat* h, int64_t offset);

/* FlatIndex::search_batch (flat.rs:150-191) / search (flat.rs:87): nq host
 * queries -> nq x k ids and natural distances (sqrt of squared L2, or +IP),
 * sorted ascending by key, ties by id. k == 0 is a no-op. */
PX_API px_status px_flat_search(const px_flat* h, const float* queries, int64_t nq, int32_t k,
                                int64_t* out_ids, float* out_dists);

/* FlatIndex::search_batch_filtered (flat.rs:193-231): mask has size()
 * bytes, nonzero = row may be returned. */
PX_API px_status px_flat_search_filtered(const px_flat* h, const float* queries, int64_t nq,
                                         int32_t k, const uint8_t* mask, int64_t* out_ids,
                                         float* out_dists);

/* Device-memory variant on a single-device handle: d_queries (nq x dim) and
 * both outputs live on the handle's device; runs on `stream` (a
 * cudaStream_t; NULL is CUDA's default stream, as for every `stream`
 * argument here). The exact path returns without waiting; the tensor-core
 * path waits on the host for that stream to finish each candidate pass (it
 * reads back how many queries the certificate left uncertified), then
 * enqueues the rest. Searches that share a handle share one workspace: keep
 * them on one stream. key_space != 0
 * writes squared-L2 / -IP keys (the form the cross-shard merge consumes)
 * instead of natural distances. */
PX_API px_status px_flat_search_device(const px_flat* h, const float* d_queries, int64_t nq,
                                       int32_t k, int32_t key_space, int64_t* d_out_ids,
                                       float* d_out_dists, void* stream);

/* Exact kNN that allocates nothing, for callers that may not allocate device
 * memory (a plugin handed a fixed arena by its host program, a service whose
 * allocator must own every byte). No counterpart in the reference. The caller
 * passes the base (d_base, n x dim row-major, dim a multiple of 4, 16-byte
 * aligned), the queries and both outputs, all in device memory on the current
 * device; results equal px_flat_search's (natural distances, ids 0..n-1).
 * Candidate lists live in a fixed 16 MiB device array inside the library
 * (held on every GPU that loads it); requests needing more (roughly
 * nq * k > 1M) are rejected with PX_EUNSUPPORTED, as are a dim and k whose
 * query row and candidate buffer exceed a block's shared memory (about
 * dim > 50,000). The array's address is tied to a CUDA context: the first
 * call in each context (the current one, whether the runtime's primary
 * context or the caller's own) looks it up and should come before any stream
 * capture in that context. Calls share the array: calls that overlap on the
 * GPU race. Runs on `stream` and returns without synchronising. */
PX_API px_status px_flat_search_noalloc(const float* d_base, int64_t n, int32_t dim, int32_t metric,
                                        const float* d_queries, int64_t nq, int32_t k,
                                        int64_t* d_out_ids, float* d_out_dists, void* stream);

/* Instrumentation, no counterpart in the reference: runs only the first
 * tensor-core candidate pass of a search (single-device handle, 1 <= k <=
 * 224, any path mode but EXACT treated as TENSOR) for nq host queries and
 * writes, per query, its merged candidates before exact rescoring: up to
 * max_cands ids (padding -1) with their APPROXIMATE keys as the pass computed
 * them (-q~.x~ for inner product; ||x||^2 - 2 q~.x~ for L2, without ||q||^2),
 * sorted by that key. *out_cands = candidates written per query, *out_pass =
 * the pass's operands (0 three-pass tf32, 1 tf32, 2 bf16). Tests use it to
 * measure the tensor cores' accumulation error against the bound the
 * certificate assumes. */
PX_API px_status px_flat_debug_candidates(const px_flat* h, const float* queries, int64_t nq, int32_t k,
                                          int32_t max_cands, int64_t* out_ids, float* out_keys,
                                          int32_t* out_cands, int32_t* out_pass);

/* Cross-shard merge on one device: keys/ids [nshard][nq][k] in key space,
 * each list sorted; writes the k best per query (ties by smaller id) as
 * natural distances (natural != 0) or keys. */
PX_API px_status px_merge_shards_device(int32_t device, const float* d_keys, const int64_t* d_ids,
                                        int32_t nshard, int64_t nq, int32_t k, int32_t metric,
                                        int32_t natural, float* d_out_dists, int64_t* d_out_ids,
                                        void* stream);

/* The same merge over shard RECORDS, the layout one collective moves: record
 * g (px_shard_record_bytes(nq, k) bytes, records back to back, 16-byte
 * aligned) holds shard g's ids [nq][k] (int64) followed by its keys [nq][k]
 * (float). A rank writes its record with px_flat_search_device (key_space =
 * 1, ids at the record's start, keys 8*nq*k bytes in), and one all-gather of
 * the records brings every shard's lists to every rank. */
PX_API int64_t px_shard_record_bytes(int64_t nq, int32_t k);
PX_API px_status px_merge_shard_records_device(int32_t device, const void* d_records, int32_t nshard, int64_t nq,
                                               int32_t k, int32_t metric, int32_t natural, float* d_out_dists,
                                               int64_t* d_out_ids, void* stream);

/* ------------------------------------------------------------------------
 * PqIndex (crates/core/src/pq.rs) on one or more GPUs.
 * ------------------------------------------------------------------------ */
typedef struct px_pq px_pq;

/* ProductQuantizer::train (pq.rs:54-105): bit-exact k-means codebooks.
 * Assignment steps run on `device`. out_codebooks: m * 2^nbits * (dim/m). */
PX_API px_status px_pq_train(const float* training, int64_t n, int32_t dim, int32_t m,
                             int32_t nbits, int32_t train_iters, int64_t train_sample,
                             uint64_t seed, int32_t device, float* out_codebooks);

/* PqIndex with given codebooks (m * 2^nbits * (dim/m) floats). */
PX_API px_status px_pq_create(int32_t dim, int32_t m, int32_t nbits, int32_t metric,
                              const float* codebooks, const int32_t* devices, int32_t ndev,
                              px_pq** out);
PX_API px_status px_pq_destroy(px_pq* h);

/* PqIndex::add (pq.rs:266-284): encodes n host vectors on the GPU and
 * appends their codes. */
PX_API px_status px_pq_add(px_pq* h, const float* vectors, int64_t n);
/* Appends n pre-encoded code rows (n x m bytes). */
PX_API px_status px_pq_add_codes(px_pq* h, const uint8_t* codes, int64_t n);
/* ProductQuantizer::encode_into (pq.rs:107-121) for n vectors -> n x m codes. */
PX_API px_status px_pq_encode(const px_pq* h, const float* vectors, int64_t n, uint8_t* out_codes);
PX_API int64_t px_pq_size(const px_pq* h);
/* Copies codes of rows [start, start + count) in id order back to the host
 * (count x m bytes). */
PX_API px_status px_pq_read_codes(const px_pq* h, int64_t start, int64_t count, uint8_t* out);
/* As px_flat_last_profile, for the last PQ search (path = 2, the ADC scan). */
PX_API px_status px_pq_last_profile(const px_pq* h, px_search_profile* out);

/* Device-memory variant of px_pq_search on a single-device handle, as
 * px_flat_search_device: d_queries (nq x dim) and both outputs on the
 * handle's device, enqueued on `stream` (NULL: the default stream) without
 * a host wait; key_space != 0 writes squared-L2 / -IP keys. */
PX_API px_status px_pq_search_device(const px_pq* h, const float* d_queries, int64_t nq, int32_t k,
                                     int32_t key_space, int64_t* d_out_ids, float* d_out_dists, void* stream);

/* PqIndex::search_batch (pq.rs:349-396) and its filtered form. */
PX_API px_status px_pq_search(const px_pq* h, const float* queries, int64_t nq, int32_t k,
                              int64_t* out_ids, float* out_dists);
PX_API px_status px_pq_search_filtered(const px_pq* h, const float* queries, int64_t nq,
                                       int32_t k, const uint8_t* mask, int64_t* out_ids,
                                       float* out_dists);

#ifdef __cplusplus
}
#endif

#endif /* PROXIMA_B200_PX_H */
