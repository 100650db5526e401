// Oracle: a CPU restatement of Proxima's exact-kNN and PQ-ADC hot path.
//
// TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and the
// cpu_baseline / reference leg of bench.py may load this library, and only as
// the checker (or the timed CPU baseline). The product (proxima_b200) never
// links, imports or calls it.
//
// Parity status: pinned against the reference's own known-answer and property
// tests (crates/core/src/{distance,flat,pq}.rs #[cfg(test)] blocks and
// tests/test_{engine,pq,filter}.py), restated in tests/test_oracle.py. The
// reference ships no golden vectors and its Rust crate cannot be compiled in
// this image (no cargo/rustc), so no output of the reference binary itself
// pins it.
//
// Every function cites the reference line it restates (paths relative to the
// reference project root). Floating-point order is reproduced exactly: this
// file must be compiled with -ffp-contract=off and without -ffast-math, so
// that every `a + b*c` is a rounded multiply followed by a rounded add, as in
// Rust (which never contracts to FMA).
//
// Tie order: FlatIndex::scan / PqIndex::scan keep a std::collections::BinaryHeap
// of candidates ordered by f32::total_cmp on the key only. The heap's sift
// order decides which of several equal keys survives at the k-th boundary and
// the order of equal keys in the output. BinaryHeap is Rust's standard library
// (not vendored in the reference; the crate needs Rust >= 1.87 for
// usize::is_multiple_of). Its published algorithm -- push = sift_up;
// pop = move last to root, sift_down_to_bottom, then sift_up;
// into_sorted_vec = repeated swap(0, end) + sift_down_range -- is restated in
// RustMaxHeap below so the oracle reproduces the reference's tie order too.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

constexpr int kLanes = 8;  // distance.rs:1

// f32::total_cmp as a signed-integer key (Rust core f32::total_cmp).
inline int32_t total_key(float x) {
  int32_t b;
  std::memcpy(&b, &x, 4);
  b ^= static_cast<int32_t>(static_cast<uint32_t>(b >> 31) >> 1);
  return b;
}

// distance.rs:4-20
float l2_sqr(const float* a, const float* b, int64_t len) {
  float acc[kLanes] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int64_t chunks = len / kLanes;
  for (int64_t c = 0; c < chunks; ++c) {
    for (int l = 0; l < kLanes; ++l) {
      float d = a[c * kLanes + l] - b[c * kLanes + l];
      float sq = d * d;
      acc[l] = acc[l] + sq;
    }
  }
  // acc.iter().sum(): a left fold. The fold seed (0.0 or -0.0 depending on
  // the Rust release) cannot change the result: no lane accumulator is ever
  // -0.0, so seed + acc[0] == acc[0] exactly.
  float sum = acc[0];
  for (int l = 1; l < kLanes; ++l) sum = sum + acc[l];
  for (int64_t i = chunks * kLanes; i < len; ++i) {
    float d = a[i] - b[i];
    float sq = d * d;
    sum = sum + sq;
  }
  return sum;
}

// distance.rs:24-39
float inner_product(const float* a, const float* b, int64_t len) {
  float acc[kLanes] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int64_t chunks = len / kLanes;
  for (int64_t c = 0; c < chunks; ++c) {
    for (int l = 0; l < kLanes; ++l) {
      float p = a[c * kLanes + l] * b[c * kLanes + l];
      acc[l] = acc[l] + p;
    }
  }
  float sum = acc[0];
  for (int l = 1; l < kLanes; ++l) sum = sum + acc[l];
  for (int64_t i = chunks * kLanes; i < len; ++i) {
    float p = a[i] * b[i];
    sum = sum + p;
  }
  return sum;
}

// flat.rs:11-32 / pq.rs:195-215: candidate ordered by key.total_cmp only.
struct Cand {
  float key;
  int64_t id;
};
inline int cmp(const Cand& a, const Cand& b) {
  int32_t x = total_key(a.key), y = total_key(b.key);
  return (x < y) ? -1 : (x > y ? 1 : 0);
}

// Rust std BinaryHeap<Cand> (a max-heap), restated.
class RustMaxHeap {
 public:
  explicit RustMaxHeap(size_t cap) { data_.reserve(cap); }
  size_t len() const { return data_.size(); }
  const Cand& peek() const { return data_[0]; }

  void push(Cand c) {
    size_t old_len = data_.size();
    data_.push_back(c);
    sift_up(0, old_len);
  }

  void pop() {
    Cand item = data_.back();
    data_.pop_back();
    if (!data_.empty()) {
      data_[0] = item;
      sift_down_to_bottom(0);
    }
  }

  std::vector<Cand> into_sorted_vec() {
    size_t end = data_.size();
    while (end > 1) {
      --end;
      std::swap(data_[0], data_[end]);
      sift_down_range(0, end);
    }
    return std::move(data_);
  }

 private:
  size_t sift_up(size_t start, size_t pos) {
    Cand elem = data_[pos];
    while (pos > start) {
      size_t parent = (pos - 1) / 2;
      if (cmp(elem, data_[parent]) <= 0) break;  // elem <= parent
      data_[pos] = data_[parent];
      pos = parent;
    }
    data_[pos] = elem;
    return pos;
  }

  void sift_down_to_bottom(size_t pos) {
    const size_t end = data_.size();
    const size_t start = pos;
    Cand elem = data_[pos];
    size_t child = 2 * pos + 1;
    const size_t lim = end >= 2 ? end - 2 : 0;
    while (end >= 2 && child <= lim) {
      child += (cmp(data_[child], data_[child + 1]) <= 0) ? 1 : 0;
      data_[pos] = data_[child];
      pos = child;
      child = 2 * pos + 1;
    }
    if (child == end - 1) {
      data_[pos] = data_[child];
      pos = child;
    }
    data_[pos] = elem;
    sift_up(start, pos);
  }

  size_t sift_down_range(size_t pos, size_t end) {
    Cand elem = data_[pos];
    size_t child = 2 * pos + 1;
    const size_t lim = end >= 2 ? end - 2 : 0;
    while (end >= 2 && child <= lim) {
      child += (cmp(data_[child], data_[child + 1]) <= 0) ? 1 : 0;
      if (cmp(elem, data_[child]) >= 0) {
        data_[pos] = elem;
        return pos;
      }
      data_[pos] = data_[child];
      pos = child;
      child = 2 * pos + 1;
    }
    if (child == end - 1 && cmp(elem, data_[child]) < 0) {
      data_[pos] = data_[child];
      pos = child;
    }
    data_[pos] = elem;
    return pos;
  }

  std::vector<Cand> data_;
};

// The heap step shared by flat.rs:131-136 and pq.rs:324-329.
inline void offer(RustMaxHeap& heap, size_t k, float key, int64_t id) {
  if (heap.len() < k) {
    heap.push(Cand{key, id});
  } else if (total_key(key) < total_key(heap.peek().key)) {
    heap.pop();
    heap.push(Cand{key, id});
  }
}

// flat.rs:139-147 / pq.rs:332-346: natural distances and padding.
void emit(RustMaxHeap& heap, bool l2, int64_t k, int64_t* out_ids, float* out_dists) {
  std::vector<Cand> sorted = heap.into_sorted_vec();
  int64_t j = 0;
  for (; j < static_cast<int64_t>(sorted.size()); ++j) {
    out_ids[j] = sorted[j].id;
    out_dists[j] = l2 ? std::sqrt(sorted[j].key) : -sorted[j].key;
  }
  for (; j < k; ++j) {
    out_ids[j] = -1;
    out_dists[j] = l2 ? 3.40282347e+38f : -3.40282347e+38f;  // f32::MAX / f32::MIN
  }
}

struct SplitMix {  // pq.rs:25-37
  uint64_t s;
  uint64_t next_u64() {
    s += 0x9E3779B97F4A7C15ull;
    uint64_t z = s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  uint64_t below(uint64_t n) { return next_u64() % n; }
};

// pq.rs:139-193
std::vector<float> kmeans(const float* data, int64_t n, int64_t d, int64_t k, int64_t iters,
                          uint64_t seed) {
  SplitMix rng{seed};
  std::vector<float> centroids(static_cast<size_t>(k * d), 0.0f);
  std::vector<int64_t> order(static_cast<size_t>(n));
  for (int64_t i = 0; i < n; ++i) order[i] = i;
  for (int64_t c = 0; c < k; ++c) {
    int64_t j = c + static_cast<int64_t>(rng.below(static_cast<uint64_t>(n - c)));
    std::swap(order[c], order[j]);
    int64_t idx = order[c];
    std::memcpy(&centroids[c * d], &data[idx * d], sizeof(float) * d);
  }
  std::vector<uint32_t> assign(static_cast<size_t>(n), 0);
  std::vector<float> sums(static_cast<size_t>(k * d), 0.0f);
  std::vector<uint32_t> counts(static_cast<size_t>(k), 0);
  for (int64_t it = 0; it < iters; ++it) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      const float* v = &data[i * d];
      uint32_t best = 0;
      float best_d = 3.40282347e+38f;
      for (int64_t c = 0; c < k; ++c) {
        float dist = l2_sqr(v, &centroids[c * d], d);
        if (dist < best_d) {
          best_d = dist;
          best = static_cast<uint32_t>(c);
        }
      }
      assign[i] = best;
    }
    std::fill(sums.begin(), sums.end(), 0.0f);
    std::fill(counts.begin(), counts.end(), 0u);
    for (int64_t i = 0; i < n; ++i) {
      int64_t c = assign[i];
      counts[c] += 1;
      const float* v = &data[i * d];
      float* s = &sums[c * d];
      for (int64_t j = 0; j < d; ++j) s[j] = s[j] + v[j];
    }
    for (int64_t c = 0; c < k; ++c) {
      if (counts[c] == 0) {
        int64_t idx = static_cast<int64_t>(rng.below(static_cast<uint64_t>(n)));
        std::memcpy(&centroids[c * d], &data[idx * d], sizeof(float) * d);
      } else {
        float inv = 1.0f / static_cast<float>(counts[c]);
        for (int64_t j = 0; j < d; ++j) centroids[c * d + j] = sums[c * d + j] * inv;
      }
    }
  }
  return centroids;
}

void set_threads(int num_threads) {
#ifdef _OPENMP
  if (num_threads > 0) omp_set_num_threads(num_threads);
#else
  (void)num_threads;
#endif
}

}  // namespace

extern "C" {

int ox_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

// flat.rs:238-250 (the tests' gen) == pq.rs:404-407 (SplitMix stream).
void ox_gen_uniform(uint64_t seed, int64_t count, float* out) {
  SplitMix s{seed};
  const float denom = static_cast<float>(UINT64_MAX);  // u64::MAX as f32 == 2^64
  for (int64_t i = 0; i < count; ++i) {
    float z = static_cast<float>(s.next_u64());
    out[i] = (z / denom) * 2.0f - 1.0f;
  }
}

uint64_t ox_splitmix_next(uint64_t* state) {
  SplitMix s{*state};
  uint64_t v = s.next_u64();
  *state = s.s;
  return v;
}

float ox_l2_sqr(const float* a, const float* b, int64_t len) { return l2_sqr(a, b, len); }
float ox_inner_product(const float* a, const float* b, int64_t len) {
  return inner_product(a, b, len);
}

// Exact key of (query, row) as FlatIndex::scan forms it (flat.rs:130).
void ox_flat_keys(const float* data, int64_t n, int64_t dim, int32_t metric, const float* query,
                  const int64_t* ids, int64_t count, float* out_keys) {
  for (int64_t i = 0; i < count; ++i) {
    int64_t id = ids ? ids[i] : i;
    const float* v = data + id * dim;
    (void)n;
    out_keys[i] = metric == 0 ? l2_sqr(query, v, dim) : -inner_product(query, v, dim);
  }
}

// flat.rs:106-148 (FlatIndex::scan); filter may be NULL (flat.rs:87-104).
void ox_flat_search(const float* data, int64_t n, int64_t dim, int32_t metric, const float* query,
                    int64_t k, const uint8_t* filter, int64_t* out_ids, float* out_dists) {
  if (k == 0) return;
  const bool l2 = metric == 0;
  RustMaxHeap heap(static_cast<size_t>(k + 1));
  for (int64_t i = 0; i < n; ++i) {
    if (filter && !filter[i]) continue;
    const float* v = data + i * dim;
    float key = l2 ? l2_sqr(query, v, dim) : -inner_product(query, v, dim);
    offer(heap, static_cast<size_t>(k), key, i);
  }
  emit(heap, l2, k, out_ids, out_dists);
}

// flat.rs:150-231 (search_batch / search_batch_filtered): a parallel loop
// over queries, each an independent scan.
void ox_flat_search_batch(const float* data, int64_t n, int64_t dim, int32_t metric,
                          const float* queries, int64_t nq, int64_t k, const uint8_t* filter,
                          int64_t* out_ids, float* out_dists, int32_t num_threads) {
  if (k == 0) return;
  set_threads(num_threads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t q = 0; q < nq; ++q) {
    ox_flat_search(data, n, dim, metric, queries + q * dim, k, filter, out_ids + q * k,
                   out_dists + q * k);
  }
}

// pq.rs:54-105 (ProductQuantizer::train). out_codebooks: m * 2^nbits * dsub.
void ox_pq_train(const float* training, int64_t n_all, int64_t dim, int64_t m, int64_t nbits,
                 int64_t train_iters, int64_t train_sample, uint64_t seed, float* out_codebooks) {
  const int64_t dsub = dim / m;
  const int64_t k = int64_t(1) << nbits;
  SplitMix rng{seed};
  int64_t n = n_all;
  if (train_sample > 0) n = std::min(std::max(train_sample, k), n_all);
  std::vector<int64_t> sample(static_cast<size_t>(n));
  if (n == n_all) {
    for (int64_t i = 0; i < n; ++i) sample[i] = i;
  } else {
    for (int64_t i = 0; i < n; ++i) sample[i] = static_cast<int64_t>(rng.below(n_all));
  }
  for (int64_t sub = 0; sub < m; ++sub) {
    std::vector<float> sub_data(static_cast<size_t>(n * dsub));
    for (int64_t i = 0; i < n; ++i) {
      std::memcpy(&sub_data[i * dsub], &training[sample[i] * dim + sub * dsub],
                  sizeof(float) * dsub);
    }
    uint64_t s = seed ^ (static_cast<uint64_t>(sub) * 0x9E3779B97F4A7C15ull);
    std::vector<float> book = kmeans(sub_data.data(), n, dsub, k, train_iters, s);
    std::memcpy(out_codebooks + sub * k * dsub, book.data(), sizeof(float) * k * dsub);
  }
}

// pq.rs:139-193, exposed for direct tests of the k-means restatement.
void ox_kmeans(const float* data, int64_t n, int64_t d, int64_t k, int64_t iters, uint64_t seed,
               float* out_centroids) {
  std::vector<float> c = kmeans(data, n, d, k, iters, seed);
  std::memcpy(out_centroids, c.data(), sizeof(float) * k * d);
}

// pq.rs:107-121 (encode_into), over n vectors (pq.rs:266-284 runs it per row).
void ox_pq_encode(const float* codebooks, int64_t dim, int64_t m, int64_t ksub,
                  const float* vectors, int64_t n, uint8_t* out_codes) {
  const int64_t dsub = dim / m;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float* v = vectors + i * dim;
    for (int64_t sub = 0; sub < m; ++sub) {
      const float* qs = v + sub * dsub;
      uint32_t best = 0;
      float best_d = 3.40282347e+38f;
      for (int64_t c = 0; c < ksub; ++c) {
        float d = l2_sqr(qs, codebooks + (sub * ksub + c) * dsub, dsub);
        if (d < best_d) {
          best_d = d;
          best = static_cast<uint32_t>(c);
        }
      }
      out_codes[i * m + sub] = static_cast<uint8_t>(best);
    }
  }
}

// pq.rs:123-136 (adc_table). table: m * ksub.
void ox_pq_adc_table(const float* codebooks, int64_t dim, int64_t m, int64_t ksub,
                     int32_t metric, const float* query, float* table) {
  const int64_t dsub = dim / m;
  for (int64_t sub = 0; sub < m; ++sub) {
    const float* qs = query + sub * dsub;
    for (int64_t c = 0; c < ksub; ++c) {
      const float* cen = codebooks + (sub * ksub + c) * dsub;
      table[sub * ksub + c] =
          metric == 0 ? l2_sqr(qs, cen, dsub) : -inner_product(qs, cen, dsub);
    }
  }
}

// pq.rs:299-347 (PqIndex::scan); filter may be NULL.
void ox_pq_search(const float* codebooks, int64_t dim, int64_t m, int64_t ksub, int32_t metric,
                  const uint8_t* codes, int64_t n, const float* query, int64_t k,
                  const uint8_t* filter, int64_t* out_ids, float* out_dists) {
  if (k == 0) return;
  std::vector<float> table(static_cast<size_t>(m * ksub));
  ox_pq_adc_table(codebooks, dim, m, ksub, metric, query, table.data());
  RustMaxHeap heap(static_cast<size_t>(k + 1));
  for (int64_t i = 0; i < n; ++i) {
    if (filter && !filter[i]) continue;
    const uint8_t* code = codes + i * m;
    float key = 0.0f;
    for (int64_t sub = 0; sub < m; ++sub) key = key + table[sub * ksub + code[sub]];
    offer(heap, static_cast<size_t>(k), key, i);
  }
  emit(heap, metric == 0, k, out_ids, out_dists);
}

// pq.rs:349-396 (search_batch_impl).
void ox_pq_search_batch(const float* codebooks, int64_t dim, int64_t m, int64_t ksub,
                        int32_t metric, const uint8_t* codes, int64_t n, const float* queries,
                        int64_t nq, int64_t k, const uint8_t* filter, int64_t* out_ids,
                        float* out_dists, int32_t num_threads) {
  if (k == 0) return;
  set_threads(num_threads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t q = 0; q < nq; ++q) {
    ox_pq_search(codebooks, dim, m, ksub, metric, codes, n, queries + q * dim, k, filter,
                 out_ids + q * k, out_dists + q * k);
  }
}

}  // extern "C"
