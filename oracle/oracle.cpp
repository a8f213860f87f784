// oracle.cpp -- CPU restatement of klearu-core's SLIDE path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
// engine in klearu_b200/csrc and the timed CPU baseline of bench.py.  Nothing
// in the product path links or calls it.
//
// It restates, in scalar f32 with the reference's loop and summation order
// (compiled with -ffp-contract=off: Rust never contracts a*b+c into an FMA),
// the following reference files (paths inside QuilibriumNetwork/klearu):
//   SimHash            crates/klearu-core/src/hash/simhash.rs:62-126
//   DWTA / WTA         crates/klearu-core/src/hash/dwta.rs:39-164, wta.rs:42-125
//   MinHash (DOPH)     crates/klearu-core/src/hash/minhash.rs:67-153
//   SRP                crates/klearu-core/src/hash/srp.rs:86-162
//   FIFO / reservoir   crates/klearu-core/src/bucket/fifo.rs:26-55, reservoir.rs:40-90
//   LshIndex           crates/klearu-core/src/lsh/index.rs:185-316
//   RebuildScheduler   crates/klearu-core/src/lsh/maintenance.rs:28-98
//   Sampling           crates/klearu-core/src/sampling/{vanilla,topk,threshold}.rs
//   Layer / Network    crates/klearu-core/src/network/layer.rs:30-308, net.rs:19-238
//   Adam / SGD         crates/klearu-core/src/optim/adam.rs:27-76, sgd.rs:17-58
//   HOGWILD            crates/klearu-core/src/optim/hogwild.rs:65-95
//   BF16 Mode 2        crates/klearu-accel/src/bf16/mod.rs:37-88
// and adds the modes the reference lacks: bf16 weight storage, batched
// gradient accumulation and a neuron-sharded output index.
//
// Random parameters (planes, windows, permutations, initial weights) are
// inputs: the reference draws them from rand 0.8.5 StdRng (ChaCha12), which is
// not available here, so seeded construction is parity-unpinned and both this
// oracle and the engine take the same explicit arrays.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <map>
#include <memory>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "../include/klearu_gpu.h"

namespace {

// ---------------------------------------------------------------------------
// bf16 (half 2.7.1 bf16::from_f32 / to_f32: round to nearest even, NaN kept)
// ---------------------------------------------------------------------------
inline uint16_t f32_to_bf16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x0040u);
  const uint32_t round_bit = 0x00008000u;
  if ((x & round_bit) != 0 && (x & (3 * round_bit - 1)) != 0) return (uint16_t)((x >> 16) + 1);
  return (uint16_t)(x >> 16);
}
inline float bf16_to_f32(uint16_t h) {
  uint32_t x = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

// f32::powi lowers to compiler-rt's __powisf2: square-and-multiply in f32.
inline float powi_f32(float a, int b) {
  const bool recip = b < 0;
  float r = 1.0f;
  while (true) {
    if (b & 1) r *= a;
    b /= 2;
    if (b == 0) break;
    a *= a;
  }
  return recip ? 1.0f / r : r;
}

// SipHash-1-3 with zero keys over two 8-byte little-endian words: what
// std::collections::hash_map::DefaultHasher computes for (usize, usize)
// (used by DwtaHash's sparse fallback, dwta.rs:131-134).  Written from the
// published SipHash specification (Aumasson & Bernstein).
inline uint64_t rotl(uint64_t x, int b) { return (x << b) | (x >> (64 - b)); }
struct Sip {
  uint64_t v0, v1, v2, v3;
  void round() {
    v0 += v1; v1 = rotl(v1, 13); v1 ^= v0; v0 = rotl(v0, 32);
    v2 += v3; v3 = rotl(v3, 16); v3 ^= v2;
    v0 += v3; v3 = rotl(v3, 21); v3 ^= v0;
    v2 += v1; v1 = rotl(v1, 17); v1 ^= v2; v2 = rotl(v2, 32);
  }
};
uint64_t siphash13_two_words(uint64_t a, uint64_t b) {
  Sip s{0x736f6d6570736575ULL, 0x646f72616e646f6dULL, 0x6c7967656e657261ULL,
        0x7465646279746573ULL};
  const uint64_t m[2] = {a, b};
  for (uint64_t w : m) {
    s.v3 ^= w;
    s.round();
    s.v0 ^= w;
  }
  const uint64_t last = (uint64_t)16 << 56;  // total length 16 bytes, no tail
  s.v3 ^= last;
  s.round();
  s.v0 ^= last;
  s.v2 ^= 0xff;
  s.round();
  s.round();
  s.round();
  return s.v0 ^ s.v1 ^ s.v2 ^ s.v3;
}

// SplitMix64 mixer of ReservoirBucket::deterministic_rand (reservoir.rs:36-44).
inline uint64_t splitmix_mod(uint64_t seed, uint64_t bound) {
  uint64_t z = seed + 0x9e3779b97f4a7c15ULL;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  z = z ^ (z >> 31);
  return z % bound;
}

// ---------------------------------------------------------------------------
// Inputs: a dense slice or a sorted sparse row.
// ---------------------------------------------------------------------------
struct SparseRow {
  const uint32_t* idx;
  const float* val;
  int nnz;
};

// ---------------------------------------------------------------------------
// Hash families (hash/*.rs)
// ---------------------------------------------------------------------------
struct Hash {
  int kind, d, k, L, w;
  int bpw = 0;                          // WTA/DWTA bits per window
  std::vector<int8_t> planes;           // SIMHASH [L][K][d]
  std::vector<uint32_t> windows;        // WTA/DWTA [L][K][w]
  std::vector<uint32_t> perms;          // MINHASH [L][d]
  std::vector<uint32_t> srp_rowptr, srp_idx;  // SRP rows (table*K + bit)
  std::vector<int8_t> srp_coef;
  int bin_size = 0;                     // MINHASH

  // simhash.rs:75-86 dot_ternary_dense
  float simhash_dot_dense(int t, int b, const float* x) const {
    const int8_t* p = &planes[((size_t)t * k + b) * d];
    float sum = 0.0f;
    for (int i = 0; i < d; ++i) {
      if (p[i] == 1) sum += x[i];
      else if (p[i] == -1) sum -= x[i];
    }
    return sum;
  }
  // simhash.rs:89-101 dot_ternary_sparse
  float simhash_dot_sparse(int t, int b, const SparseRow& r) const {
    const int8_t* p = &planes[((size_t)t * k + b) * d];
    float sum = 0.0f;
    for (int j = 0; j < r.nnz; ++j) {
      int8_t c = p[r.idx[j]];
      if (c == 1) sum += r.val[j];
      else if (c == -1) sum -= r.val[j];
    }
    return sum;
  }
  // srp.rs:93-104 dot_sparse_dense
  float srp_dot_dense(int t, int b, const float* x) const {
    const int row = t * k + b;
    float sum = 0.0f;
    for (uint32_t e = srp_rowptr[row]; e < srp_rowptr[row + 1]; ++e) {
      float v = x[srp_idx[e]];
      if (srp_coef[e] == 1) sum += v;
      else if (srp_coef[e] == -1) sum -= v;
    }
    return sum;
  }
  // srp.rs:108-133 dot_sparse_sparse (sorted merge)
  float srp_dot_sparse(int t, int b, const SparseRow& r) const {
    const int row = t * k + b;
    float sum = 0.0f;
    uint32_t i = srp_rowptr[row], iend = srp_rowptr[row + 1];
    int j = 0;
    while (i < iend && j < r.nnz) {
      uint32_t pi = srp_idx[i], si = r.idx[j];
      if (pi == si) {
        if (srp_coef[i] == 1) sum += r.val[j];
        else if (srp_coef[i] == -1) sum -= r.val[j];
        ++i;
        ++j;
      } else if (pi < si) {
        ++i;
      } else {
        ++j;
      }
    }
    return sum;
  }
  // dwta.rs:88-99 / wta.rs:91-102 argmax_dense
  int argmax_dense(const uint32_t* win, const float* x) const {
    int best_pos = 0;
    float best = -std::numeric_limits<float>::infinity();
    for (int p = 0; p < w; ++p) {
      float v = x[win[p]];
      if (v > best) {
        best = v;
        best_pos = p;
      }
    }
    return best_pos;
  }
  // dwta.rs:104-137 argmax_sparse (binary search + SipHash fallback)
  int argmax_sparse(const uint32_t* win, const SparseRow& r, int t, int kk) const {
    int best_pos = -1;
    float best = -std::numeric_limits<float>::infinity();
    for (int p = 0; p < w; ++p) {
      const uint32_t* it = std::lower_bound(r.idx, r.idx + r.nnz, win[p]);
      if (it != r.idx + r.nnz && *it == win[p]) {
        float v = r.val[it - r.idx];
        if (v > best) {
          best = v;
          best_pos = p;
        }
      }
    }
    if (best_pos >= 0) return best_pos;
    return (int)(siphash13_two_words((uint64_t)t, (uint64_t)kk) % (uint64_t)w);
  }
  // minhash.rs:67-153
  uint64_t minhash(const std::vector<uint32_t>& nz, int t) const {
    std::vector<uint32_t> mins(k, 0xffffffffu);
    const uint32_t* perm = &perms[(size_t)t * d];
    for (uint32_t dim : nz) {
      uint32_t pm = perm[dim];
      size_t bin = pm / (uint32_t)bin_size;
      if ((int)bin < k) mins[bin] = std::min(mins[bin], pm);
    }
    bool all_empty = true;
    for (uint32_t v : mins) all_empty &= (v == 0xffffffffu);
    if (all_empty) {
      std::fill(mins.begin(), mins.end(), 0u);
    } else {
      for (int i = 0; i < k; ++i) {
        if (mins[i] == 0xffffffffu) {
          int j = (i + 1) % k;
          while (mins[j] == 0xffffffffu) j = (j + 1) % k;
          mins[i] = mins[j];
        }
      }
    }
    const uint64_t PRIME = 0x517cc1b727220a95ULL;
    const uint64_t mask = k >= 64 ? ~0ULL : ((1ULL << k) - 1);
    uint64_t h = 0, pp = 1;
    for (uint32_t m : mins) {
      h += (uint64_t)m * pp;
      pp *= PRIME;
    }
    return h & mask;
  }

  uint64_t hash_dense(const float* x, int t, float* min_abs) const {
    uint64_t h = 0;
    float mn = std::numeric_limits<float>::infinity();
    switch (kind) {
      case KL_HASH_SIMHASH:
      case KL_HASH_SRP:
        for (int b = 0; b < k; ++b) {
          float dot = kind == KL_HASH_SIMHASH ? simhash_dot_dense(t, b, x) : srp_dot_dense(t, b, x);
          if (dot >= 0.0f) h |= 1ULL << b;
          mn = std::min(mn, std::fabs(dot));
        }
        break;
      case KL_HASH_WTA:
      case KL_HASH_DWTA: {
        int shift = 0;
        for (int kk = 0; kk < k; ++kk) {
          h |= (uint64_t)argmax_dense(&windows[((size_t)t * k + kk) * w], x) << shift;
          shift += bpw;
        }
        break;
      }
      case KL_HASH_MINHASH: {
        std::vector<uint32_t> nz;
        for (int i = 0; i < d; ++i)
          if (x[i] != 0.0f) nz.push_back((uint32_t)i);
        h = minhash(nz, t);
        break;
      }
    }
    if (min_abs) *min_abs = mn;
    return h;
  }

  uint64_t hash_sparse(const SparseRow& r, int t, float* min_abs) const {
    uint64_t h = 0;
    float mn = std::numeric_limits<float>::infinity();
    switch (kind) {
      case KL_HASH_SIMHASH:
      case KL_HASH_SRP:
        for (int b = 0; b < k; ++b) {
          float dot = kind == KL_HASH_SIMHASH ? simhash_dot_sparse(t, b, r) : srp_dot_sparse(t, b, r);
          if (dot >= 0.0f) h |= 1ULL << b;
          mn = std::min(mn, std::fabs(dot));
        }
        break;
      case KL_HASH_WTA: {  // wta.rs:115-118: to_dense then hash_dense
        std::vector<float> dense(d, 0.0f);
        for (int j = 0; j < r.nnz; ++j) dense[r.idx[j]] = r.val[j];
        return hash_dense(dense.data(), t, min_abs);
      }
      case KL_HASH_DWTA: {
        int shift = 0;
        for (int kk = 0; kk < k; ++kk) {
          h |= (uint64_t)argmax_sparse(&windows[((size_t)t * k + kk) * w], r, t, kk) << shift;
          shift += bpw;
        }
        break;
      }
      case KL_HASH_MINHASH: {  // minhash.rs:150-152: every stored index
        std::vector<uint32_t> nz(r.idx, r.idx + r.nnz);
        h = minhash(nz, t);
        break;
      }
    }
    if (min_abs) *min_abs = mn;
    return h;
  }
};

Hash* make_hash(int kind, int d, int k, int L, int w, const kl_hash_params* p) {
  auto* h = new Hash();
  h->kind = kind;
  h->d = d;
  h->k = k;
  h->L = L;
  h->w = w;
  switch (kind) {
    case KL_HASH_SIMHASH:
      h->planes.assign(p->planes, p->planes + (size_t)L * k * d);
      break;
    case KL_HASH_WTA:
    case KL_HASH_DWTA:
      h->windows.assign(p->windows, p->windows + (size_t)L * k * w);
      h->bpw = 1;
      if (w > 1) {
        h->bpw = 0;
        while ((1 << h->bpw) < w) ++h->bpw;
      }
      break;
    case KL_HASH_MINHASH:
      h->perms.assign(p->perms, p->perms + (size_t)L * d);
      h->bin_size = (d + k - 1) / k;
      break;
    case KL_HASH_SRP: {
      h->srp_rowptr.assign(p->srp_rowptr, p->srp_rowptr + L * k + 1);
      uint32_t nnz = h->srp_rowptr[L * k];
      h->srp_idx.assign(p->srp_idx, p->srp_idx + nnz);
      h->srp_coef.assign(p->srp_coef, p->srp_coef + nnz);
      break;
    }
    default:
      delete h;
      return nullptr;
  }
  return h;
}

// ---------------------------------------------------------------------------
// Buckets (bucket/fifo.rs, bucket/reservoir.rs) as fixed arrays, so that the
// racy HOGWILD baseline can never touch freed memory.
// ---------------------------------------------------------------------------
struct Bucket {
  uint32_t* data;
  int cap;
  int len = 0;
  uint64_t count = 0;

  void insert_fifo(uint32_t id) {  // fifo.rs:27-33
    if (len >= cap) {
      std::memmove(data, data + 1, sizeof(uint32_t) * (cap - 1));
      len = cap - 1;
    }
    data[len++] = id;
  }
  void insert_reservoir(uint32_t id) {  // reservoir.rs:50-67
    count += 1;
    if (len < cap) {
      data[len++] = id;
    } else {
      uint64_t seed = count * 0x517cc1b727220a95ULL + (uint64_t)id;
      uint64_t j = splitmix_mod(seed, count);
      if (j < (uint64_t)cap) {
        uint64_t slot = splitmix_mod(seed + 1, (uint64_t)cap);
        data[slot] = id;
      }
    }
  }
  bool remove(uint32_t id) {  // fifo.rs:35-42 / reservoir.rs:69-76 (swap_remove)
    int n = std::min(len, cap);
    for (int p = 0; p < n; ++p) {
      if (data[p] == id) {
        data[p] = data[n - 1];
        len = n - 1;
        return true;
      }
    }
    return false;
  }
  void clear(bool reservoir) {
    len = 0;
    if (reservoir) count = 0;
  }
};

// ---------------------------------------------------------------------------
// LshIndex (lsh/index.rs:178-316)
// ---------------------------------------------------------------------------
struct Index {
  std::shared_ptr<Hash> hash;
  int type, cap, L, nb;
  std::vector<uint32_t> store;
  std::vector<Bucket> buckets;  // [L][nb]

  Index(std::shared_ptr<Hash> h, int bucket_type, int capacity)
      : hash(std::move(h)), type(bucket_type), cap(capacity) {
    L = hash->L;
    nb = 1 << hash->k;
    store.assign((size_t)L * nb * cap, 0);
    buckets.resize((size_t)L * nb);
    for (size_t i = 0; i < buckets.size(); ++i) {
      buckets[i].data = &store[i * cap];
      buckets[i].cap = cap;
    }
  }
  Bucket& bucket(int t, uint64_t code) { return buckets[(size_t)t * nb + (code & (uint64_t)(nb - 1))]; }
  void bucket_insert(Bucket& b, uint32_t id) {
    if (type == KL_BUCKET_FIFO) b.insert_fifo(id);
    else b.insert_reservoir(id);
  }
  void insert(uint32_t id, const float* x) {  // index.rs:257-262
    for (int t = 0; t < L; ++t) bucket_insert(bucket(t, hash->hash_dense(x, t, nullptr)), id);
  }
  void insert_sparse(uint32_t id, const SparseRow& r) {
    for (int t = 0; t < L; ++t) bucket_insert(bucket(t, hash->hash_sparse(r, t, nullptr)), id);
  }
  void remove_with_weights(uint32_t id, const float* x) {
    for (int t = 0; t < L; ++t) bucket(t, hash->hash_dense(x, t, nullptr)).remove(id);
  }
  void remove(uint32_t id) {
    for (auto& b : buckets) b.remove(id);
  }
  void clear() {
    for (auto& b : buckets) b.clear(type == KL_BUCKET_RESERVOIR);
  }
  // collect_counts (index.rs:219-234), returned sorted by id.
  template <class F>
  void collect(F code_of, std::vector<std::pair<uint32_t, uint32_t>>& out) const {
    std::map<uint32_t, uint32_t> counts;
    for (int t = 0; t < L; ++t) {
      const Bucket& b = buckets[(size_t)t * nb + (code_of(t) & (uint64_t)(nb - 1))];
      int n = std::min(b.len, b.cap);
      for (int i = 0; i < n; ++i) counts[b.data[i]] += 1;
    }
    out.assign(counts.begin(), counts.end());
  }
  void query_dense(const float* x, std::vector<std::pair<uint32_t, uint32_t>>& out) const {
    collect([&](int t) { return hash->hash_dense(x, t, nullptr); }, out);
  }
  void query_sparse(const SparseRow& r, std::vector<std::pair<uint32_t, uint32_t>>& out) const {
    collect([&](int t) { return hash->hash_sparse(r, t, nullptr); }, out);
  }
};

// ---------------------------------------------------------------------------
// Sampling (sampling/*.rs).  Candidates arrive sorted by id.
// ---------------------------------------------------------------------------
void sample_select(int type, int top_k, int threshold,
                   const std::vector<std::pair<uint32_t, uint32_t>>& cand,
                   std::vector<uint32_t>& out) {
  out.clear();
  if (type == KL_SAMPLING_VANILLA) {  // vanilla.rs:8-12
    for (auto& c : cand) out.push_back(c.first);
    return;
  }
  if (cand.empty()) return;
  if (type == KL_SAMPLING_TOPK) {  // topk.rs:19-34
    std::vector<std::pair<uint32_t, uint32_t>> s = cand;
    std::stable_sort(s.begin(), s.end(), [](auto& a, auto& b) {
      if (a.second != b.second) return a.second > b.second;
      return a.first < b.first;
    });
    for (size_t i = 0; i < s.size() && (int)i < top_k; ++i) out.push_back(s[i].first);
    return;
  }
  // threshold.rs:20-43
  for (auto& c : cand)
    if (c.second >= (uint32_t)threshold) out.push_back(c.first);
  if (!out.empty()) return;
  auto best = cand[0];
  for (auto& c : cand)
    if (c.second > best.second || (c.second == best.second && c.first < best.first)) best = c;
  out.push_back(best.first);
}

// ---------------------------------------------------------------------------
// RebuildScheduler (lsh/maintenance.rs:28-98)
// ---------------------------------------------------------------------------
struct Scheduler {
  uint64_t base;
  double decay;
  uint64_t count = 0, next, cur = 0;
  Scheduler(uint64_t b, double d) : base(b), decay(d), next(b) {}
  bool should_rebuild(uint64_t step) {
    cur = step;
    if (cur >= next) {
      count += 1;
      uint64_t interval = (uint64_t)((double)base * std::exp(decay * (double)count));
      next = cur + std::max<uint64_t>(interval, 1);
      return true;
    }
    return false;
  }
};

// ---------------------------------------------------------------------------
// AdaptiveScheduler (crates/klearu-mongoose/src/scheduler.rs:44-213).  The
// reference samples ceil(n * sample_fraction) neurons with rand 0.8.5's
// StdRng shuffle; that stream is not available here, so the sampled indices
// (sorted) are an input.  Everything else -- counters, the drift fraction in
// f32, the EMA with alpha 0.3 -- follows the reference line by line.
// ---------------------------------------------------------------------------
struct Adaptive {
  size_t min_interval, max_interval;
  float sample_fraction, drift_threshold;
  float drift_ema = 0.0f, ema_alpha = 0.3f;
  size_t steps_since_rebuild = 0, steps_since_check = 0;
  std::vector<uint32_t> sampled;               // indices into the neuron rows
  std::vector<std::vector<uint64_t>> baseline;  // [sampled][L]

  // record_baseline (scheduler.rs:96-129) with explicit sampled indices.
  void record_baseline(const Hash& h, const float* rows, int n, int ld, const uint32_t* idx, int ns) {
    sampled.assign(idx, idx + ns);
    baseline.assign(ns, std::vector<uint64_t>(h.L));
    for (int i = 0; i < ns; ++i)
      for (int t = 0; t < h.L; ++t) baseline[i][t] = h.hash_dense(rows + (size_t)idx[i] * ld, t, nullptr);
    (void)n;
    steps_since_rebuild = 0;
    steps_since_check = 0;
    drift_ema = 0.0f;
  }
  // estimate_drift (scheduler.rs:163-195)
  float estimate_drift(const Hash& h, const float* rows, int n, int ld) const {
    if (baseline.empty() || sampled.empty()) return 0.0f;
    size_t changed = 0;
    for (size_t b = 0; b < sampled.size(); ++b) {
      if ((int)sampled[b] >= n) continue;
      bool any = false;
      for (int t = 0; t < h.L && !any; ++t)
        any = (size_t)t < baseline[b].size() && h.hash_dense(rows + (size_t)sampled[b] * ld, t, nullptr) != baseline[b][t];
      if (any) ++changed;
    }
    return (float)changed / (float)sampled.size();
  }
  // should_rebuild (scheduler.rs:133-159)
  bool should_rebuild(const Hash& h, const float* rows, int n, int ld) {
    steps_since_rebuild += 1;
    steps_since_check += 1;
    if (steps_since_rebuild >= max_interval) {
      steps_since_rebuild = 0;
      steps_since_check = 0;
      return true;
    }
    if (steps_since_check < min_interval) return false;
    const float drift = estimate_drift(h, rows, n, ld);
    drift_ema = ema_alpha * drift + (1.0f - ema_alpha) * drift_ema;
    steps_since_check = 0;
    if (drift_ema >= drift_threshold) {
      steps_since_rebuild = 0;
      return true;
    }
    return false;
  }
  void notify_rebuild() {  // scheduler.rs:198-201
    steps_since_rebuild = 0;
    steps_since_check = 0;
  }
};

// ---------------------------------------------------------------------------
// Activations (layer.rs:250-308)
// ---------------------------------------------------------------------------
float activate(float x, int act) {
  switch (act) {
    case KL_ACT_RELU: return std::fmax(x, 0.0f);
    case KL_ACT_SIGMOID: return 1.0f / (1.0f + std::exp(-x));
    case KL_ACT_TANH: return std::tanh(x);
    default: return x;
  }
}
float activation_derivative(float pre, float post, int act) {
  switch (act) {
    case KL_ACT_RELU: return pre > 0.0f ? 1.0f : 0.0f;
    case KL_ACT_SIGMOID: return post * (1.0f - post);
    case KL_ACT_TANH: return 1.0f - post * post;
    default: return 1.0f;
  }
}
std::vector<float> softmax(const std::vector<float>& v) {
  if (v.empty()) return {};
  float mx = -std::numeric_limits<float>::infinity();
  for (float x : v) mx = std::fmax(mx, x);
  std::vector<float> e(v.size());
  for (size_t i = 0; i < v.size(); ++i) e[i] = std::exp(v[i] - mx);
  float sum = 0.0f;
  for (float x : e) sum += x;
  if (sum > 0.0f) {
    for (float& x : e) x = x / sum;
  } else {
    for (float& x : e) x = 1.0f / (float)v.size();
  }
  return e;
}

// ---------------------------------------------------------------------------
// Layer (network/layer.rs) with f32 or bf16 row storage.
// ---------------------------------------------------------------------------
struct LayerOut {
  std::vector<float> activations;  // dense [N] (layer.rs:110-113)
  std::vector<uint32_t> active;
  std::vector<float> pre;
  std::vector<float> post;         // post-activation in active order
};

struct Layer {
  kl_layer_config cfg;
  int d, N;
  bool bf16;
  std::vector<float> wf;        // [N][d] f32 storage
  std::vector<uint16_t> wb;     // [N][d] bf16 storage
  std::vector<float> bias;
  std::vector<float> m, v, mb, vb;  // optimizer state (SGD momentum in m/mb)
  std::vector<Index> shards;    // one index, or P indices over neuron slices
  std::vector<uint32_t> shard_lo;  // first neuron id of each shard (+ end)
  float sgd_momentum = 0.9f;       // net.rs:233-238 creates Sgd::new(0.9)

  float w(size_t n, size_t i) const { return bf16 ? bf16_to_f32(wb[n * d + i]) : wf[n * d + i]; }
  void row(size_t n, std::vector<float>& out) const {
    out.resize(d);
    for (int i = 0; i < d; ++i) out[i] = w(n, i);
  }

  void build_index() {  // layer.rs:40-44 / 228-233: insert every neuron in id order
    std::vector<float> r;
    for (size_t s = 0; s < shards.size(); ++s) {
      shards[s].clear();
      for (uint32_t n = shard_lo[s]; n < shard_lo[s + 1]; ++n) {
        row(n, r);
        shards[s].insert(n, r.data());
      }
    }
  }

  // Neuron::forward (neuron.rs:47-62): sequential sum of w*x, then + bias.
  float dot_dense(uint32_t n, const float* x) const {
    float s = 0.0f;
    if (bf16) {
      const uint16_t* p = &wb[(size_t)n * d];
      for (int i = 0; i < d; ++i) s += bf16_to_f32(p[i]) * x[i];
    } else {
      const float* p = &wf[(size_t)n * d];
      for (int i = 0; i < d; ++i) s += p[i] * x[i];
    }
    return s + bias[n];
  }
  // Same value from the nonzeros only: the skipped terms are w*0 = +-0, which
  // leave a sequential f32 sum unchanged (up to the sign of a zero result).
  float dot_sparse(uint32_t n, const SparseRow& r) const {
    float s = 0.0f;
    for (int j = 0; j < r.nnz; ++j) s += w(n, r.idx[j]) * r.val[j];
    return s + bias[n];
  }

  void query(const float* x, const SparseRow* sr, std::vector<std::pair<uint32_t, uint32_t>>& cand) const {
    cand.clear();
    std::vector<std::pair<uint32_t, uint32_t>> part;
    for (auto& ix : shards) {
      if (sr) ix.query_sparse(*sr, part);
      else ix.query_dense(x, part);
      cand.insert(cand.end(), part.begin(), part.end());
    }
  }

  // Layer::forward (layer.rs:65-120).  `sr` non-null => use the sparse form of
  // the same input (bit-identical results; the dense form is the reference's).
  void forward(const float* x, const SparseRow* sr, LayerOut& o) const {
    std::vector<std::pair<uint32_t, uint32_t>> cand;
    query(x, sr, cand);
    sample_select(cfg.sampling, cfg.top_k, cfg.sampling_threshold, cand, o.active);
    if (o.active.empty()) {
      o.active.resize(N);
      for (int i = 0; i < N; ++i) o.active[i] = (uint32_t)i;
    }
    o.active.erase(std::remove_if(o.active.begin(), o.active.end(),
                                  [&](uint32_t id) { return (int)id >= N; }),
                   o.active.end());
    o.pre.resize(o.active.size());
    for (size_t i = 0; i < o.active.size(); ++i)
      o.pre[i] = sr ? dot_sparse(o.active[i], *sr) : dot_dense(o.active[i], x);
    if (cfg.activation == KL_ACT_SOFTMAX) {
      o.post = softmax(o.pre);
    } else {
      o.post.resize(o.pre.size());
      for (size_t i = 0; i < o.pre.size(); ++i) o.post[i] = activate(o.pre[i], cfg.activation);
    }
    o.activations.assign(N, 0.0f);
    for (size_t i = 0; i < o.active.size(); ++i) o.activations[o.active[i]] = o.post[i];
  }

  // Local gradients (layer.rs:139-194).
  std::vector<float> local_grads(const LayerOut& o, const float* grad_out, int grad_len) const {
    size_t n = o.active.size();
    std::vector<float> res(n, 0.0f);
    auto go_of = [&](uint32_t id) { return (int)id < grad_len ? grad_out[id] : 0.0f; };
    if (cfg.activation == KL_ACT_SOFTMAX) {
      std::vector<float> s = softmax(o.pre);
      for (size_t i = 0; i < n; ++i) {
        for (size_t j = 0; j < n; ++j) {
          float go_j = go_of(o.active[j]);
          if (i == j) res[i] += go_j * s[j] * (1.0f - s[j]);
          else res[i] += go_j * (-s[i] * s[j]);
        }
      }
    } else {
      for (size_t i = 0; i < n; ++i) {
        uint32_t id = o.active[i];
        res[i] = go_of(id) * activation_derivative(o.pre[i], o.activations[id], cfg.activation);
      }
    }
    return res;
  }

  // Optimizer::update on one row (adam.rs:27-76 / sgd.rs:17-58).  `g` is the
  // dense row gradient, `gb` the bias gradient.  bf16 rows are updated as
  // Bf16Weights::update_from_f32 (bf16/mod.rs:85-88): bf16(w + delta).
  void update_row(uint32_t n, const float* g, float gb, int opt, float lr, uint64_t step) {
    const size_t o = (size_t)n * d;
    if (opt == KL_OPT_ADAM) {
      const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
      uint64_t t = std::max<uint64_t>(step, 1);
      float c1 = 1.0f - powi_f32(b1, (int)t);
      float c2 = 1.0f - powi_f32(b2, (int)t);
      for (int i = 0; i < d; ++i) {
        float gi = g[i];
        m[o + i] = b1 * m[o + i] + (1.0f - b1) * gi;
        v[o + i] = b2 * v[o + i] + (1.0f - b2) * gi * gi;
        float mh = m[o + i] / c1;
        float vh = v[o + i] / c2;
        float q = lr * mh / (std::sqrt(vh) + eps);
        if (bf16) wb[o + i] = f32_to_bf16(bf16_to_f32(wb[o + i]) + (-q));
        else wf[o + i] -= q;
      }
      mb[n] = b1 * mb[n] + (1.0f - b1) * gb;
      vb[n] = b2 * vb[n] + (1.0f - b2) * gb * gb;
      float mh = mb[n] / c1, vh = vb[n] / c2;
      bias[n] -= lr * mh / (std::sqrt(vh) + eps);
    } else {
      const float mom = sgd_momentum;
      for (int i = 0; i < d; ++i) {
        float vv = mom * m[o + i] - lr * g[i];
        m[o + i] = vv;
        if (bf16) wb[o + i] = f32_to_bf16(bf16_to_f32(wb[o + i]) + vv);
        else wf[o + i] += vv;
      }
      float vv = mom * mb[n] - lr * gb;
      mb[n] = vv;
      bias[n] += vv;
    }
  }
};

// compute_loss (net.rs:180-199)
float compute_loss(const LayerOut& o, const uint32_t* labels, int nl) {
  if (nl == 0) return 0.0f;
  const float eps = 1e-7f;
  float loss = 0.0f;
  for (int i = 0; i < nl; ++i) {
    uint32_t lab = labels[i];
    bool active = std::find(o.active.begin(), o.active.end(), lab) != o.active.end();
    float prob = active ? std::fmax(o.activations[lab], eps) : eps;
    loss -= std::log(prob);
  }
  return loss / (float)nl;
}
// compute_loss_gradient (net.rs:205-230)
std::vector<float> compute_loss_gradient(const LayerOut& o, const uint32_t* labels, int nl, int N) {
  std::vector<float> g(N, 0.0f);
  if (nl == 0) return g;
  for (uint32_t id : o.active)
    if ((int)id < N) g[id] = o.activations[id];
  float lw = 1.0f / (float)nl;
  for (int i = 0; i < nl; ++i)
    if ((int)labels[i] < N) g[labels[i]] -= lw;
  return g;
}

// ---------------------------------------------------------------------------
// Network (network/net.rs)
// ---------------------------------------------------------------------------
struct Net {
  std::vector<Layer> layers;
  int opt;
  uint64_t step = 0;
  Scheduler sched{100, 0.1};
  bool sparse_input = false;  // use the sparse form of layer-0 inputs

  void forward(const float* x, const SparseRow* sr, std::vector<LayerOut>& outs) const {
    outs.resize(layers.size());
    const float* cur = x;
    for (size_t l = 0; l < layers.size(); ++l) {
      layers[l].forward(cur, l == 0 ? sr : nullptr, outs[l]);
      cur = outs[l].activations.data();
    }
  }

  // Network::backward (net.rs:122-146) + Layer::backward (layer.rs:124-225).
  void backward_exact(const std::vector<LayerOut>& outs, const float* x, const SparseRow* sr,
                      std::vector<float> grad, float lr) {
    for (int l = (int)layers.size() - 1; l >= 0; --l) {
      Layer& L = layers[l];
      const LayerOut& o = outs[l];
      std::vector<float> grad_in(L.d, 0.0f);
      if (o.active.empty()) {
        grad = grad_in;
        continue;
      }
      std::vector<float> lg = L.local_grads(o, grad.data(), (int)grad.size());
      std::vector<float> dense_in;
      const float* in = l == 0 ? x : outs[l - 1].activations.data();
      if (l == 0 && sr) {
        dense_in.assign(L.d, 0.0f);
        for (int j = 0; j < sr->nnz; ++j) dense_in[sr->idx[j]] = sr->val[j];
        in = dense_in.data();
      }
      std::vector<float> gw(L.d);
      for (size_t i = 0; i < o.active.size(); ++i) {
        uint32_t id = o.active[i];
        for (int j = 0; j < L.d; ++j) gw[j] = lg[i] * in[j];
        if (l > 0)  // layer 0's input gradient is discarded by the reference
          for (int j = 0; j < L.d; ++j) grad_in[j] += lg[i] * L.w(id, j);
        L.update_row(id, gw.data(), lg[i], opt, lr, step);
      }
      grad = grad_in;
    }
  }

  float train_exact(const int32_t* rowptr, const uint32_t* idx, const float* val,
                    const int32_t* lptr, const uint32_t* labels, int B, float lr) {
    if (B == 0) return 0.0f;
    float total = 0.0f;
    const int d0 = layers[0].d;
    std::vector<float> dense(d0);
    std::vector<LayerOut> outs;
    for (int s = 0; s < B; ++s) {
      SparseRow r{idx + rowptr[s], val + rowptr[s], rowptr[s + 1] - rowptr[s]};
      const float* x = nullptr;
      if (!sparse_input) {  // SparseVector::to_dense (sparse.rs:77-83)
        std::fill(dense.begin(), dense.end(), 0.0f);
        for (int j = 0; j < r.nnz; ++j) dense[r.idx[j]] = r.val[j];
        x = dense.data();
      }
      forward(x, sparse_input ? &r : nullptr, outs);
      const LayerOut& last = outs.back();
      const uint32_t* lab = labels + lptr[s];
      int nl = lptr[s + 1] - lptr[s];
      total += compute_loss(last, lab, nl);
      std::vector<float> g = compute_loss_gradient(last, lab, nl, layers.back().N);
      backward_exact(outs, x, sparse_input ? &r : nullptr, std::move(g), lr);
    }
    after_step();
    return total / (float)B;
  }

  void after_step() {  // net.rs:109-116
    step += 1;
    if (sched.should_rebuild(step))
      for (auto& L : layers) L.build_index();
  }

  // Batched mode: forward every example against the step-start weights, sum
  // per-row gradients over the batch in example order, then one optimizer
  // update per touched row with t = max(step, 1).
  float train_batched(const int32_t* rowptr, const uint32_t* idx, const float* val,
                      const int32_t* lptr, const uint32_t* labels, int B, float lr) {
    if (B == 0) return 0.0f;
    const int nL = (int)layers.size();
    std::vector<std::vector<LayerOut>> outs(B);
    std::vector<std::vector<float>> grads(B);
    float total = 0.0f;
    std::vector<SparseRow> rows(B);
    std::vector<std::vector<float>> dense(B);
    for (int s = 0; s < B; ++s) {
      rows[s] = SparseRow{idx + rowptr[s], val + rowptr[s], rowptr[s + 1] - rowptr[s]};
      dense[s].assign(layers[0].d, 0.0f);
      for (int j = 0; j < rows[s].nnz; ++j) dense[s][rows[s].idx[j]] = rows[s].val[j];
      forward(sparse_input ? nullptr : dense[s].data(), sparse_input ? &rows[s] : nullptr, outs[s]);
      const uint32_t* lab = labels + lptr[s];
      int nl = lptr[s + 1] - lptr[s];
      total += compute_loss(outs[s].back(), lab, nl);
      grads[s] = compute_loss_gradient(outs[s].back(), lab, nl, layers.back().N);
    }
    for (int l = nL - 1; l >= 0; --l) {
      Layer& L = layers[l];
      std::vector<std::vector<float>> lgs(B);
      for (int s = 0; s < B; ++s) lgs[s] = L.local_grads(outs[s][l], grads[s].data(), (int)grads[s].size());
      // input gradients with the old weights
      if (l > 0) {
        for (int s = 0; s < B; ++s) {
          std::vector<float> gi(L.d, 0.0f);
          const LayerOut& o = outs[s][l];
          for (size_t i = 0; i < o.active.size(); ++i)
            for (int j = 0; j < L.d; ++j) gi[j] += lgs[s][i] * L.w(o.active[i], j);
          grads[s] = std::move(gi);
        }
      }
      // per-row gradient sums in example order
      std::map<uint32_t, std::pair<std::vector<float>, float>> G;
      for (int s = 0; s < B; ++s) {
        const LayerOut& o = outs[s][l];
        const float* in = l == 0 ? dense[s].data() : outs[s][l - 1].activations.data();
        for (size_t i = 0; i < o.active.size(); ++i) {
          auto& e = G[o.active[i]];
          if (e.first.empty()) {
            e.first.assign(L.d, 0.0f);
            e.second = 0.0f;
          }
          for (int j = 0; j < L.d; ++j) e.first[j] += lgs[s][i] * in[j];
          e.second += lgs[s][i];
        }
      }
      for (auto& kv : G) L.update_row(kv.first, kv.second.first.data(), kv.second.second, opt, lr, step);
    }
    after_step();
    return total / (float)B;
  }
};

}  // namespace

// ===========================================================================
// C API for the Python test harness (ctypes) and the CPU baseline.
// ===========================================================================
extern "C" {

uint64_t orc_siphash13_usize2(uint64_t a, uint64_t b) { return siphash13_two_words(a, b); }
float orc_powi_f32(float a, int b) { return powi_f32(a, b); }
uint16_t orc_f32_to_bf16(float f) { return f32_to_bf16(f); }
uint64_t orc_splitmix_mod(uint64_t seed, uint64_t bound) { return splitmix_mod(seed, bound); }

// ---- hash ----
void* orc_hash_create(int kind, int d, int k, int L, int w, const kl_hash_params* p) {
  return new std::shared_ptr<Hash>(make_hash(kind, d, k, L, w, p));
}
void orc_hash_destroy(void* h) { delete static_cast<std::shared_ptr<Hash>*>(h); }
void orc_hash_dense(void* hp, const float* X, int n, int ldx, uint64_t* codes, float* min_abs) {
  auto& h = **static_cast<std::shared_ptr<Hash>*>(hp);
  for (int i = 0; i < n; ++i)
    for (int t = 0; t < h.L; ++t)
      codes[(size_t)i * h.L + t] = h.hash_dense(X + (size_t)i * ldx, t, min_abs ? &min_abs[(size_t)i * h.L + t] : nullptr);
}
void orc_hash_sparse(void* hp, const int32_t* rowptr, const uint32_t* idx, const float* val, int n,
                     uint64_t* codes, float* min_abs) {
  auto& h = **static_cast<std::shared_ptr<Hash>*>(hp);
  for (int i = 0; i < n; ++i) {
    SparseRow r{idx + rowptr[i], val + rowptr[i], rowptr[i + 1] - rowptr[i]};
    for (int t = 0; t < h.L; ++t)
      codes[(size_t)i * h.L + t] = h.hash_sparse(r, t, min_abs ? &min_abs[(size_t)i * h.L + t] : nullptr);
  }
}

// ---- standalone bucket (KATs of bucket/*.rs) ----
struct OrcBucket {
  std::vector<uint32_t> store;
  Bucket b;
  int type;
};
void* orc_bucket_create(int type, int cap) {
  auto* ob = new OrcBucket();
  ob->store.assign(cap, 0);
  ob->b.data = ob->store.data();
  ob->b.cap = cap;
  ob->type = type;
  return ob;
}
void orc_bucket_destroy(void* p) { delete static_cast<OrcBucket*>(p); }
void orc_bucket_insert(void* p, uint32_t id) {
  auto* ob = static_cast<OrcBucket*>(p);
  if (ob->type == KL_BUCKET_FIFO) ob->b.insert_fifo(id);
  else ob->b.insert_reservoir(id);
}
int orc_bucket_remove(void* p, uint32_t id) { return static_cast<OrcBucket*>(p)->b.remove(id) ? 1 : 0; }
void orc_bucket_clear(void* p) {
  auto* ob = static_cast<OrcBucket*>(p);
  ob->b.clear(ob->type == KL_BUCKET_RESERVOIR);
}
int orc_bucket_contents(void* p, uint32_t* out) {
  auto* ob = static_cast<OrcBucket*>(p);
  for (int i = 0; i < ob->b.len; ++i) out[i] = ob->b.data[i];
  return ob->b.len;
}
uint64_t orc_bucket_total(void* p) { return static_cast<OrcBucket*>(p)->b.count; }

// ---- index ----
void* orc_index_create(void* hp, int bucket_type, int cap) {
  return new Index(*static_cast<std::shared_ptr<Hash>*>(hp), bucket_type, cap);
}
void orc_index_destroy(void* p) { delete static_cast<Index*>(p); }
void orc_index_insert(void* p, const uint32_t* ids, const float* rows, int n, int ld) {
  auto* ix = static_cast<Index*>(p);
  for (int i = 0; i < n; ++i) ix->insert(ids[i], rows + (size_t)i * ld);
}
void orc_index_insert_sparse(void* p, const uint32_t* ids, const int32_t* rowptr, const uint32_t* idx,
                             const float* val, int n) {
  auto* ix = static_cast<Index*>(p);
  for (int i = 0; i < n; ++i) {
    SparseRow r{idx + rowptr[i], val + rowptr[i], rowptr[i + 1] - rowptr[i]};
    ix->insert_sparse(ids[i], r);
  }
}
void orc_index_remove(void* p, const uint32_t* ids, int n) {
  auto* ix = static_cast<Index*>(p);
  for (int i = 0; i < n; ++i) ix->remove(ids[i]);
}
void orc_index_remove_with_weights(void* p, const uint32_t* ids, const float* rows, int n, int ld) {
  auto* ix = static_cast<Index*>(p);
  for (int i = 0; i < n; ++i) ix->remove_with_weights(ids[i], rows + (size_t)i * ld);
}
void orc_index_clear(void* p) { static_cast<Index*>(p)->clear(); }
// Queries: writes up to `cap_out` (id, count) pairs sorted by id; returns the size.
int orc_index_query(void* p, const float* x, uint32_t* ids, uint32_t* counts, int cap_out) {
  std::vector<std::pair<uint32_t, uint32_t>> c;
  static_cast<Index*>(p)->query_dense(x, c);
  int n = std::min((int)c.size(), cap_out);
  for (int i = 0; i < n; ++i) {
    ids[i] = c[i].first;
    if (counts) counts[i] = c[i].second;
  }
  return (int)c.size();
}
int orc_index_query_sparse(void* p, const uint32_t* idx, const float* val, int nnz, uint32_t* ids,
                           uint32_t* counts, int cap_out) {
  std::vector<std::pair<uint32_t, uint32_t>> c;
  SparseRow r{idx, val, nnz};
  static_cast<Index*>(p)->query_sparse(r, c);
  int n = std::min((int)c.size(), cap_out);
  for (int i = 0; i < n; ++i) {
    ids[i] = c[i].first;
    if (counts) counts[i] = c[i].second;
  }
  return (int)c.size();
}
void orc_index_export(void* p, uint32_t* ids, uint32_t* lens, uint64_t* counts) {
  auto* ix = static_cast<Index*>(p);
  std::memcpy(ids, ix->store.data(), ix->store.size() * 4);
  for (size_t i = 0; i < ix->buckets.size(); ++i) {
    lens[i] = (uint32_t)ix->buckets[i].len;
    if (counts) counts[i] = ix->buckets[i].count;
  }
}

// ---- sampling ----
int orc_sample(int type, int top_k, int threshold, const uint32_t* ids, const uint32_t* counts, int n,
               uint32_t* out) {
  std::vector<std::pair<uint32_t, uint32_t>> c(n);
  for (int i = 0; i < n; ++i) c[i] = {ids[i], counts[i]};
  std::vector<uint32_t> o;
  sample_select(type, top_k, threshold, c, o);
  std::copy(o.begin(), o.end(), out);
  return (int)o.size();
}

// ---- scheduler ----
void* orc_adaptive_create(uint64_t min_interval, uint64_t max_interval, float sample_fraction, float drift_threshold) {
  auto* a = new Adaptive();
  a->min_interval = min_interval;
  a->max_interval = max_interval;
  a->sample_fraction = sample_fraction;
  a->drift_threshold = drift_threshold;
  return a;
}
void orc_adaptive_destroy(void* p) { delete static_cast<Adaptive*>(p); }
void orc_adaptive_record_baseline(void* p, void* hp, const float* rows, int n, int ld, const uint32_t* idx, int ns) {
  static_cast<Adaptive*>(p)->record_baseline(**static_cast<std::shared_ptr<Hash>*>(hp), rows, n, ld, idx, ns);
}
int orc_adaptive_should_rebuild(void* p, void* hp, const float* rows, int n, int ld) {
  return static_cast<Adaptive*>(p)->should_rebuild(**static_cast<std::shared_ptr<Hash>*>(hp), rows, n, ld) ? 1 : 0;
}
void orc_adaptive_notify_rebuild(void* p) { static_cast<Adaptive*>(p)->notify_rebuild(); }
float orc_adaptive_drift(void* p) { return static_cast<Adaptive*>(p)->drift_ema; }
uint64_t orc_adaptive_steps(void* p) { return static_cast<Adaptive*>(p)->steps_since_rebuild; }
void* orc_sched_create(uint64_t base, double decay) { return new Scheduler(base, decay); }
void orc_sched_destroy(void* p) { delete static_cast<Scheduler*>(p); }
int orc_sched_should_rebuild(void* p, uint64_t step) { return static_cast<Scheduler*>(p)->should_rebuild(step) ? 1 : 0; }
uint64_t orc_sched_next(void* p) { return static_cast<Scheduler*>(p)->next; }
uint64_t orc_sched_count(void* p) { return static_cast<Scheduler*>(p)->count; }

// ---- loss / gradient (net.rs:180-230) on an explicit LayerOutput ----
float orc_compute_loss(const float* activations, int N, const uint32_t* active, int na,
                       const uint32_t* labels, int nl) {
  LayerOut o;
  o.activations.assign(activations, activations + N);
  o.active.assign(active, active + na);
  return compute_loss(o, labels, nl);
}
void orc_compute_loss_gradient(const float* activations, int N, const uint32_t* active, int na,
                               const uint32_t* labels, int nl, float* grad) {
  LayerOut o;
  o.activations.assign(activations, activations + N);
  o.active.assign(active, active + na);
  auto g = compute_loss_gradient(o, labels, nl, N);
  std::copy(g.begin(), g.end(), grad);
}
// Optimizer::update on one row, standalone (adam.rs / sgd.rs KATs).
void orc_optimizer_update(int opt, float* w, const float* g, int d, float* bias, float gb, double lr,
                          uint64_t step, float* m, float* v, float* mb, float* vb, float momentum) {
  Layer L;
  L.sgd_momentum = momentum;
  L.d = d;
  L.N = 1;
  L.bf16 = false;
  L.wf.assign(w, w + d);
  L.bias = {*bias};
  L.m.assign(m, m + d);
  L.v.assign(v, v + d);
  L.mb = {*mb};
  L.vb = {*vb};
  L.update_row(0, g, gb, opt, (float)lr, step);
  std::copy(L.wf.begin(), L.wf.end(), w);
  std::copy(L.m.begin(), L.m.end(), m);
  std::copy(L.v.begin(), L.v.end(), v);
  *bias = L.bias[0];
  *mb = L.mb[0];
  *vb = L.vb[0];
}

// ---- network ----
// nshards > 1: the LAST layer's index is split into nshards indices over
// contiguous neuron slices [r*N/P, (r+1)*N/P) sharing one hash family, each
// with bucket capacity cap / P.
void* orc_net_create(const kl_net_config* cfg, const kl_layer_init* init, int nshards, int sparse_input) {
  auto* net = new Net();
  net->opt = cfg->optimizer;
  net->sparse_input = sparse_input != 0;
  const bool bf = cfg->weight_dtype == KL_DTYPE_BF16;
  net->layers.resize(cfg->num_layers);
  for (int l = 0; l < cfg->num_layers; ++l) {
    Layer& L = net->layers[l];
    L.cfg = cfg->layers[l];
    L.d = L.cfg.input_dim;
    L.N = L.cfg.num_neurons;
    L.bf16 = bf;
    size_t nd = (size_t)L.N * L.d;
    if (bf) {
      L.wb.resize(nd);
      for (size_t i = 0; i < nd; ++i) L.wb[i] = f32_to_bf16(init[l].weights[i]);
    } else {
      L.wf.assign(init[l].weights, init[l].weights + nd);
    }
    L.bias.assign(L.N, 0.0f);
    if (init[l].bias) L.bias.assign(init[l].bias, init[l].bias + L.N);
    L.m.assign(nd, 0.0f);
    L.v.assign(cfg->optimizer == KL_OPT_ADAM ? nd : 0, 0.0f);
    L.mb.assign(L.N, 0.0f);
    L.vb.assign(L.N, 0.0f);
    const kl_lsh_config& lc = L.cfg.lsh;
    int w = std::min(8, L.d);  // index.rs:325-330 DEFAULT_WINDOW_SIZE.min(input_dim)
    std::shared_ptr<Hash> h(make_hash(lc.hash_function, L.d, lc.num_hashes, lc.num_tables, w, &init[l].hash));
    int P = (l == cfg->num_layers - 1) ? std::max(1, nshards) : 1;
    for (int r = 0; r <= P; ++r) L.shard_lo.push_back((uint32_t)(((uint64_t)r * L.N) / P));
    L.shards.reserve(P);
    // Sharded: each shard's buckets hold cap / P ids (at least 1), so a
    // sample's candidate budget over all shards stays L * cap, as unsharded.
    const int shard_cap = P > 1 ? std::max(1, lc.bucket_capacity / P) : lc.bucket_capacity;
    for (int r = 0; r < P; ++r) L.shards.emplace_back(h, lc.bucket_type, shard_cap);
    L.build_index();
  }
  const kl_lsh_config& l0 = cfg->layers[0].lsh;
  net->sched = Scheduler((uint64_t)l0.rebuild_interval_base, l0.rebuild_decay);
  return net;
}
void orc_net_destroy(void* p) { delete static_cast<Net*>(p); }

float orc_net_train_step(void* p, const int32_t* rowptr, const uint32_t* idx, const float* val,
                         const int32_t* lptr, const uint32_t* labels, int B, double lr, int mode) {
  auto* net = static_cast<Net*>(p);
  if (mode == KL_MODE_BATCHED) return net->train_batched(rowptr, idx, val, lptr, labels, B, (float)lr);
  return net->train_exact(rowptr, idx, val, lptr, labels, B, (float)lr);
}

// HogwildNetwork::train_parallel (hogwild.rs:65-95): ceil(B/threads)-sized
// chunks, each a train_step on the shared, unsynchronised network.
float orc_net_train_hogwild(void* p, const int32_t* rowptr, const uint32_t* idx, const float* val,
                            const int32_t* lptr, const uint32_t* labels, int B, double lr, int threads) {
  auto* net = static_cast<Net*>(p);
  if (B == 0 || threads <= 0) return 0.0f;
  int chunk = (B + threads - 1) / threads;
  int nchunks = (B + chunk - 1) / chunk;
  std::vector<float> losses(nchunks, 0.0f);
#pragma omp parallel for num_threads(threads) schedule(static, 1)
  for (int c = 0; c < nchunks; ++c) {
    int s0 = c * chunk, s1 = std::min(B, s0 + chunk);
    losses[c] = net->train_exact(rowptr + s0, idx, val, lptr + s0, labels, s1 - s0, (float)lr);
  }
  float sum = 0.0f;
  for (float l : losses) sum += l;
  return sum / (float)nchunks;
}

// Forward one example (no update).  Results of every layer are kept and read
// with orc_net_output.
struct ForwardCache {
  std::vector<LayerOut> outs;
};
static thread_local ForwardCache g_fwd;
void orc_net_forward(void* p, const uint32_t* idx, const float* val, int nnz) {
  auto* net = static_cast<Net*>(p);
  SparseRow r{idx, val, nnz};
  if (net->sparse_input) {
    net->forward(nullptr, &r, g_fwd.outs);
  } else {
    std::vector<float> dense(net->layers[0].d, 0.0f);
    for (int j = 0; j < nnz; ++j) dense[idx[j]] = val[j];
    net->forward(dense.data(), nullptr, g_fwd.outs);
  }
}
// Active ids (sorted by id), pre-activations and activations of `layer` from
// the last orc_net_forward; returns the active count.
int orc_net_output(int layer, uint32_t* ids, float* pre, float* act, int cap_out) {
  const LayerOut& o = g_fwd.outs[layer];
  std::vector<size_t> ord(o.active.size());
  for (size_t i = 0; i < ord.size(); ++i) ord[i] = i;
  std::sort(ord.begin(), ord.end(), [&](size_t a, size_t b) { return o.active[a] < o.active[b]; });
  int n = std::min((int)ord.size(), cap_out);
  for (int i = 0; i < n; ++i) {
    if (ids) ids[i] = o.active[ord[i]];
    if (pre) pre[i] = o.pre[ord[i]];
    if (act) act[i] = o.post[ord[i]];
  }
  return (int)ord.size();
}
void orc_net_get_layer(void* p, int l, float* w, float* b, float* m, float* v, float* mb, float* vb) {
  auto* net = static_cast<Net*>(p);
  Layer& L = net->layers[l];
  size_t nd = (size_t)L.N * L.d;
  if (w)
    for (size_t i = 0; i < nd; ++i) w[i] = L.bf16 ? bf16_to_f32(L.wb[i]) : L.wf[i];
  if (b) std::copy(L.bias.begin(), L.bias.end(), b);
  if (m) std::copy(L.m.begin(), L.m.end(), m);
  if (v && !L.v.empty()) std::copy(L.v.begin(), L.v.end(), v);
  if (mb) std::copy(L.mb.begin(), L.mb.end(), mb);
  if (vb) std::copy(L.vb.begin(), L.vb.end(), vb);
}
uint64_t orc_net_step(void* p) { return static_cast<Net*>(p)->step; }
uint64_t orc_net_next_rebuild(void* p) { return static_cast<Net*>(p)->sched.next; }
void orc_net_rebuild(void* p) {
  for (auto& L : static_cast<Net*>(p)->layers) L.build_index();
}
// Export the index of `layer` (shard `shard`).
void orc_net_export_index(void* p, int l, int shard, uint32_t* ids, uint32_t* lens, uint64_t* counts) {
  Index& ix = static_cast<Net*>(p)->layers[l].shards[shard];
  orc_index_export(&ix, ids, lens, counts);
}

}  // extern "C"
