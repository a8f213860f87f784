// api.cu -- the C ABI (include/klearu_gpu.h): handles, validation, device
// memory, and the host-side orchestration of the SLIDE train step.
//
// Host orchestration mirrors crates/klearu-core/src/network/net.rs:
//   Network::new        -> kl_net_create   (net.rs:19-57, layer.rs:30-61)
//   Network::train_step -> kl_net_train_step (net.rs:81-119)
//   Network::forward    -> kl_net_forward  (net.rs:62-78)
//   RebuildScheduler    -> Scheduler below (lsh/maintenance.rs:70-82)
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include <nccl.h>

#include <functional>

#include "engine.h"
#include "watchdog.h"

using namespace kl;

namespace kl {
static std::atomic<unsigned long long> g_launches{0};
void count_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
// Process-wide count of device and pinned-host allocations made by this library.
static std::atomic<unsigned long long> g_allocs{0};
}  // namespace kl

// ---------------------------------------------------------------------------
// Small host utilities
// ---------------------------------------------------------------------------
namespace {

struct KlError {
  kl_status st;
  std::string msg;
};
[[noreturn]] void raise(kl_status st, const std::string& m) { throw KlError{st, m}; }
void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    if (e == cudaErrorMemoryAllocation) raise(KL_ENOMEM, std::string(what) + ": " + cudaGetErrorString(e));
    raise(KL_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
}
void ck_launch(const char* what) { ck(cudaGetLastError(), what); }
void require(bool c, const std::string& m) {
  if (!c) raise(KL_EINVAL, m);
}
void support(bool c, const std::string& m) {
  if (!c) raise(KL_EUNSUPPORTED, m);
}

// Device allocation owned by one object.
struct DBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DBuf() = default;
  DBuf(const DBuf&) = delete;
  DBuf& operator=(const DBuf&) = delete;
  ~DBuf() {
    if (p) cudaFree(p);
  }
  void alloc(size_t n) {
    if (n <= bytes && p) return;
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    if (n == 0) n = 16;
    ck(cudaMalloc(&p, n), "cudaMalloc");
    g_allocs.fetch_add(1, std::memory_order_relaxed);
    bytes = n;
  }
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

// f32::powi lowered to compiler-rt's square-and-multiply (adam.rs:52-53).
float powi_f32(float a, int b) {
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

// SipHash-1-3 (zero keys) over two 8-byte words: DefaultHasher of
// (usize, usize), used by DwtaHash's sparse fallback (dwta.rs:131-134).
// Written from the published SipHash specification.
uint64_t siphash13_two_words(uint64_t a, uint64_t b) {
  auto rotl = [](uint64_t x, int r) { return (x << r) | (x >> (64 - r)); };
  uint64_t v0 = 0x736f6d6570736575ULL, v1 = 0x646f72616e646f6dULL, v2 = 0x6c7967656e657261ULL,
           v3 = 0x7465646279746573ULL;
  auto round = [&]() {
    v0 += v1; v1 = rotl(v1, 13); v1 ^= v0; v0 = rotl(v0, 32);
    v2 += v3; v3 = rotl(v3, 16); v3 ^= v2;
    v0 += v3; v3 = rotl(v3, 21); v3 ^= v0;
    v2 += v1; v1 = rotl(v1, 17); v1 ^= v2; v2 = rotl(v2, 32);
  };
  for (uint64_t m : {a, b}) {
    v3 ^= m;
    round();
    v0 ^= m;
  }
  const uint64_t last = (uint64_t)16 << 56;
  v3 ^= last;
  round();
  v0 ^= last;
  v2 ^= 0xff;
  round();
  round();
  round();
  return v0 ^ v1 ^ v2 ^ v3;
}

// This library's seeded generator (SplitMix64).  Not rand's ChaCha12.
struct SplitMix {
  uint64_t s;
  uint64_t next() {
    uint64_t z = (s += 0x9e3779b97f4a7c15ULL);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
  }
  double unit() { return (double)(next() >> 11) * (1.0 / 9007199254740992.0); }
  uint64_t below(uint64_t n) { return next() % n; }
  double normal() {  // Box-Muller
    double u1 = unit(), u2 = unit();
    if (u1 < 1e-300) u1 = 1e-300;
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
  }
  template <class T>
  void shuffle(std::vector<T>& v) {
    for (size_t i = v.size(); i > 1; --i) std::swap(v[i - 1], v[below(i)]);
  }
};

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

int bits_for(uint64_t n) {  // bits needed for values < n
  int b = 0;
  while (b < 64 && ((n - 1) >> b) != 0 && n > 1) ++b;
  return b;
}

}  // namespace

// ---------------------------------------------------------------------------
// Handles
// ---------------------------------------------------------------------------
struct kl_ctx_s {
  int device = 0;
  cudaStream_t stream = nullptr;
  DBuf err;  // int device error word
  std::string last_error;
};

struct HashImpl {
  kl_ctx_t ctx;
  DevHash dh;
  DBuf planes, planesT, windows, fallback, perms, plist, poff, tcplanes;
  std::unique_ptr<TcPlanes> tc;
};
struct kl_hash_s {
  std::shared_ptr<HashImpl> h;
};

struct IndexImpl {
  kl_ctx_t ctx;
  std::shared_ptr<HashImpl> hash;
  DevTables T;
  DBuf ids, len, cnt;
  DBuf bkt, scratch, qids, qcnt, qn, qoff;
  int nb_bits = 0;

  void hash_dense_to_bkt(const DenseIn& in) {
    bkt.alloc((size_t)T.L * std::max(in.n, 1) * 2);
    HashOut o;
    o.bkt = bkt.as<uint16_t>();
    o.bkt_ld = in.n;
    o.nb_mask = (uint32_t)(T.nb - 1);
    launch_hash_dense(hash->dh, in, o, ctx->stream);
    ck_launch("hash");
  }
  void hash_sparse_to_bkt(const SparseIn& in) {
    bkt.alloc((size_t)T.L * std::max(in.n, 1) * 2);
    HashOut o;
    o.bkt = bkt.as<uint16_t>();
    o.bkt_ld = in.n;
    o.nb_mask = (uint32_t)(T.nb - 1);
    launch_hash_sparse(hash->dh, in, o, ctx->stream);
    ck_launch("hash");
  }
  void insert_from_bkt(const uint32_t* idsin, int n) {
    if (n <= 0) return;
    scratch.alloc(insert_scratch_bytes(T, n));
    InsertScratch s;
    carve_insert_scratch(T, n, scratch.p, &s);
    launch_tables_insert(T, idsin, bkt.as<uint16_t>(), n, n, s, ctx->err.as<int>(), ctx->stream);
    ck_launch("insert");
  }
  void clear() {
    launch_tables_clear(T, ctx->stream);
    ck_launch("clear");
  }
  // Query: padded results into qids/qcnt/qn, then CSR compaction.
  // Probe into per-query padded (id, count) lists sorted by id: qids / qcnt
  // [n][L*cap], sizes in qn.  Returns the stride.
  int probe_padded(int n) {
    const int stride = T.L * T.cap;
    qids.alloc((size_t)std::max(n, 1) * stride * 4);
    qcnt.alloc((size_t)std::max(n, 1) * stride * 4);
    qn.alloc((size_t)std::max(n, 1) * 4);
    ProbeArgs a;
    a.T = T;
    a.bkt = bkt.as<uint16_t>();
    a.bkt_ld = n;
    a.nq = n;
    a.N = 0;
    a.id_bits = 32;
    a.out_ids = qids.as<uint32_t>();
    a.out_counts = qcnt.as<uint32_t>();
    a.out_stride = stride;
    a.out_n = qn.as<int32_t>();
    a.err = ctx->err.as<int>();
    launch_probe(a, ctx->stream);
    ck_launch("probe");
    return stride;
  }
  void query(int n, int mode, uint32_t* out_ids, uint32_t* out_counts, int32_t* out_offsets,
             int32_t capacity, int32_t* overflow) {
    const int stride = probe_padded(n);
    if (overflow) ck(cudaMemsetAsync(overflow, 0, 4, ctx->stream), "memset");
    launch_scan(qn.as<int32_t>(), out_offsets, n, nullptr, ctx->stream);
    ck_launch("scan");
    launch_compact(qids.as<uint32_t>(), mode == KL_QUERY_COUNTS ? qcnt.as<uint32_t>() : nullptr,
                   stride, out_offsets, n, out_ids, mode == KL_QUERY_COUNTS ? out_counts : nullptr,
                   capacity, overflow, ctx->err.as<int>(), ctx->stream);
    ck_launch("compact");
  }
};
struct kl_index_s {
  std::shared_ptr<IndexImpl> ix;
};

namespace {

std::shared_ptr<HashImpl> make_hash(kl_ctx_t ctx, int kind, int d, int k, int L, int w,
                                    const kl_hash_params* p) {
  require(d >= 1 && k >= 1 && L >= 1, "hash: input_dim, k and num_tables must be >= 1");
  auto H = std::make_shared<HashImpl>();
  H->ctx = ctx;
  DevHash& h = H->dh;
  h.kind = kind;
  h.d = d;
  h.k = k;
  h.L = L;
  cudaStream_t st = ctx->stream;
  switch (kind) {
    case KL_HASH_SIMHASH:
    case KL_HASH_SRP: {
      support(k <= 32, "SimHash/SRP: num_hashes > 32");
      support((int64_t)L * k <= 1024, "SimHash/SRP: num_tables*num_hashes > 1024");
      h.LK = L * k;
      h.dpad = (int)round_up(d, 16);
      h.lkpad = (int)round_up(h.LK, 16);
      std::vector<int8_t> dense((size_t)h.LK * h.dpad, 0), dT((size_t)d * h.lkpad, 0);
      if (kind == KL_HASH_SIMHASH) {
        require(p && p->planes, "SimHash: planes required");
        for (int tb = 0; tb < h.LK; ++tb)
          for (int i = 0; i < d; ++i) {
            int8_t v = p->planes[(size_t)tb * d + i];
            require(v >= -1 && v <= 1, "SimHash: plane entries must be -1, 0 or 1");
            dense[(size_t)tb * h.dpad + i] = v;
          }
      } else {
        require(p && p->srp_rowptr && (p->srp_rowptr[h.LK] == 0 || (p->srp_idx && p->srp_coef)),
                "SRP: rowptr/idx/coef required");
        for (int tb = 0; tb < h.LK; ++tb)
          for (uint32_t e = p->srp_rowptr[tb]; e < p->srp_rowptr[tb + 1]; ++e) {
            require(p->srp_idx[e] < (uint32_t)d, "SRP: index >= input_dim");
            require(p->srp_coef[e] == 1 || p->srp_coef[e] == -1, "SRP: coefficients must be +-1");
            dense[(size_t)tb * h.dpad + p->srp_idx[e]] = p->srp_coef[e];
          }
      }
      for (int tb = 0; tb < h.LK; ++tb)
        for (int i = 0; i < d; ++i) dT[(size_t)i * h.lkpad + tb] = dense[(size_t)tb * h.dpad + i];
      h.nt = (int)ceil_div(d, PL_T);
      std::vector<uint16_t> plist;
      std::vector<uint32_t> poff((size_t)h.LK * (h.nt + 1), 0);
      for (int tb = 0; tb < h.LK; ++tb) {
        for (int ti = 0; ti < h.nt; ++ti) {
          poff[(size_t)tb * (h.nt + 1) + ti] = (uint32_t)plist.size();
          for (int i = ti * PL_T; i < std::min(d, (ti + 1) * PL_T); ++i) {
            const int8_t v = dense[(size_t)tb * h.dpad + i];
            if (v) plist.push_back((uint16_t)((i - ti * PL_T) | (v < 0 ? 0x8000 : 0)));
          }
        }
        poff[(size_t)tb * (h.nt + 1) + h.nt] = (uint32_t)plist.size();
      }
      plist.resize(plist.size() + 128, 0);  // slack for the kernel's read-ahead (3 windows of 32)
      H->plist.alloc(plist.size() * 2);
      H->poff.alloc(poff.size() * 4);
      ck(cudaMemcpyAsync(H->plist.p, plist.data(), plist.size() * 2, cudaMemcpyHostToDevice, st), "upload");
      ck(cudaMemcpyAsync(H->poff.p, poff.data(), poff.size() * 4, cudaMemcpyHostToDevice, st), "upload");
      h.plist = H->plist.as<uint16_t>();
      h.poff = H->poff.as<uint32_t>();
      H->planes.alloc(dense.size());
      H->planesT.alloc(dT.size());
      ck(cudaMemcpyAsync(H->planes.p, dense.data(), dense.size(), cudaMemcpyHostToDevice, st), "upload");
      ck(cudaMemcpyAsync(H->planesT.p, dT.data(), dT.size(), cudaMemcpyHostToDevice, st), "upload");
      // exact bf16 copy of the planes for the tensor-core projection, grouped by table
      auto tc = std::make_unique<TcPlanes>();
      if (tc_plane_layout(d, k, L, tc.get())) {
        std::vector<uint16_t> pb((size_t)tc->H * tc->Nh * tc->dpad, 0);
        for (int t = 0; t < L; ++t) {
          const int grp = t / tc->tph, lt = t % tc->tph;
          for (int b = 0; b < k; ++b) {
            const size_t row = (size_t)grp * tc->Nh + (size_t)lt * k + b;
            for (int i = 0; i < d; ++i) {
              const int8_t v = dense[(size_t)(t * k + b) * h.dpad + i];
              pb[row * tc->dpad + i] = v == 0 ? 0 : (v > 0 ? 0x3F80 : 0xBF80);  // bf16 +1 / -1
            }
          }
        }
        H->tcplanes.alloc(pb.size() * 2);
        ck(cudaMemcpyAsync(H->tcplanes.p, pb.data(), pb.size() * 2, cudaMemcpyHostToDevice, st), "upload");
        tc->planes = H->tcplanes.p;
        tc->err = ctx->err.as<int>();
        tc->ready = tc_plane_map(tc.get());
        H->tc = std::move(tc);
        h.tc = H->tc.get();
      }
      ck(cudaStreamSynchronize(st), "sync");
      h.planes = H->planes.as<int8_t>();
      h.planesT = H->planesT.as<int8_t>();
      break;
    }
    case KL_HASH_WTA:
    case KL_HASH_DWTA: {
      require(w >= 1 && w <= d, "WTA/DWTA: window_size must be in [1, input_dim] (dwta.rs:46-49)");
      h.w = w;
      h.bpw = 1;
      if (w > 1) {
        h.bpw = 0;
        while ((1 << h.bpw) < w) ++h.bpw;
      }
      require((int64_t)k * h.bpw <= 64, "WTA/DWTA: k * bits_per_window exceeds 64 (dwta.rs:51-54)");
      require(p && p->windows, "WTA/DWTA: windows required");
      const size_t nw = (size_t)L * k * w;
      for (size_t i = 0; i < nw; ++i) require(p->windows[i] < (uint32_t)d, "WTA/DWTA: window dim >= input_dim");
      std::vector<uint8_t> fb((size_t)L * k);
      for (int t = 0; t < L; ++t)
        for (int kk = 0; kk < k; ++kk) fb[(size_t)t * k + kk] = (uint8_t)(siphash13_two_words(t, kk) % (uint64_t)w);
      H->windows.alloc(nw * 4);
      H->fallback.alloc(fb.size());
      ck(cudaMemcpyAsync(H->windows.p, p->windows, nw * 4, cudaMemcpyHostToDevice, st), "upload");
      ck(cudaMemcpyAsync(H->fallback.p, fb.data(), fb.size(), cudaMemcpyHostToDevice, st), "upload");
      ck(cudaStreamSynchronize(st), "sync");
      h.windows = H->windows.as<uint32_t>();
      h.fallback = H->fallback.as<uint8_t>();
      break;
    }
    case KL_HASH_MINHASH: {
      support(k <= 64, "MinHash: num_hashes > 64");
      require(p && p->perms, "MinHash: perms required");
      h.bin_size = (d + k - 1) / k;
      const size_t n = (size_t)L * d;
      H->perms.alloc(n * 4);
      ck(cudaMemcpyAsync(H->perms.p, p->perms, n * 4, cudaMemcpyHostToDevice, st), "upload");
      ck(cudaStreamSynchronize(st), "sync");
      h.perms = H->perms.as<uint32_t>();
      break;
    }
    default:
      raise(KL_EINVAL, "unknown hash kind");
  }
  return H;
}

// Seeded parameters following the reference distributions.
struct SeededParams {
  std::vector<int8_t> planes;
  std::vector<uint32_t> windows, perms, rowptr, idx;
  std::vector<int8_t> coef;
  kl_hash_params p{};
};
void seeded_params(int kind, int d, int k, int L, int w, float sparsity, uint64_t seed, SeededParams& sp) {
  SplitMix rng{seed};
  switch (kind) {
    case KL_HASH_SIMHASH:  // simhash.rs:37-71: order table, bit, dim; 1/6, 2/3, 1/6
      sp.planes.resize((size_t)L * k * d);
      for (auto& v : sp.planes) {
        double r = rng.unit();
        v = r < 1.0 / 6.0 ? -1 : (r < 1.0 / 6.0 + 2.0 / 3.0 ? 0 : 1);
      }
      sp.p.planes = sp.planes.data();
      break;
    case KL_HASH_WTA:
    case KL_HASH_DWTA: {  // first w of a full shuffle per (table, fn)
      std::vector<uint32_t> all(d);
      for (int t = 0; t < L; ++t)
        for (int kk = 0; kk < k; ++kk) {
          for (int i = 0; i < d; ++i) all[i] = (uint32_t)i;
          rng.shuffle(all);
          sp.windows.insert(sp.windows.end(), all.begin(), all.begin() + w);
        }
      sp.p.windows = sp.windows.data();
      break;
    }
    case KL_HASH_MINHASH: {
      std::vector<uint32_t> all(d);
      for (int t = 0; t < L; ++t) {
        for (int i = 0; i < d; ++i) all[i] = (uint32_t)i;
        rng.shuffle(all);
        sp.perms.insert(sp.perms.end(), all.begin(), all.end());
      }
      sp.p.perms = sp.perms.data();
      break;
    }
    case KL_HASH_SRP: {  // srp.rs:60-78
      const double pneg = sparsity / 2.0, pzero_end = pneg + (1.0 - sparsity);
      sp.rowptr.push_back(0);
      for (int tb = 0; tb < L * k; ++tb) {
        for (int i = 0; i < d; ++i) {
          double r = rng.unit();
          if (r < pneg) {
            sp.idx.push_back((uint32_t)i);
            sp.coef.push_back(-1);
          } else if (r >= pzero_end) {
            sp.idx.push_back((uint32_t)i);
            sp.coef.push_back(1);
          }
        }
        sp.rowptr.push_back((uint32_t)sp.idx.size());
      }
      sp.p.srp_rowptr = sp.rowptr.data();
      sp.p.srp_idx = sp.idx.data();
      sp.p.srp_coef = sp.coef.data();
      break;
    }
  }
}

std::shared_ptr<IndexImpl> make_index(kl_ctx_t ctx, std::shared_ptr<HashImpl> h, int bucket_type,
                                      int cap) {
  require(cap > 0, "bucket capacity must be positive (fifo.rs:18, reservoir.rs:25)");
  require(bucket_type == KL_BUCKET_FIFO || bucket_type == KL_BUCKET_RESERVOIR, "unknown bucket type");
  support(h->dh.k <= 12, "index: num_hashes > 12 (more than 4096 buckets per table)");
  support(h->dh.L <= 1024, "index: num_tables > 1024");
  support((int64_t)h->dh.L * cap <= probe_max_items(),
          "index: num_tables * bucket_capacity exceeds the probe kernel's shared-memory capacity");
  auto I = std::make_shared<IndexImpl>();
  I->ctx = ctx;
  I->hash = std::move(h);
  DevTables& T = I->T;
  T.L = I->hash->dh.L;
  T.nb = 1 << I->hash->dh.k;
  T.cap = cap;
  T.type = bucket_type;
  const size_t LB = (size_t)T.L * T.nb;
  I->ids.alloc(LB * cap * 4);
  I->len.alloc(LB * 4);
  I->cnt.alloc(LB * 8);
  T.ids = I->ids.as<uint32_t>();
  T.len = I->len.as<uint32_t>();
  T.cnt = I->cnt.as<uint64_t>();
  ck(cudaMemsetAsync(T.ids, 0, LB * cap * 4, ctx->stream), "memset");
  ck(cudaMemsetAsync(T.len, 0, LB * 4, ctx->stream), "memset");
  ck(cudaMemsetAsync(T.cnt, 0, LB * 8, ctx->stream), "memset");
  return I;
}

DenseIn dense_rows(const void* rows, int dtype, int n, int ld) {
  require(dtype == KL_DTYPE_F32 || dtype == KL_DTYPE_BF16, "dtype must be KL_DTYPE_F32 or KL_DTYPE_BF16");
  DenseIn in;
  in.X = rows;
  in.dtype = dtype;
  in.ld_row = ld;
  in.ld_elem = 1;
  in.n = n;
  return in;
}

thread_local std::string g_thread_error;

kl_status finish(kl_ctx_t ctx, const KlError& e) {
  if (ctx) ctx->last_error = e.msg;
  g_thread_error = e.msg;
  return e.st;
}

}  // namespace

#define KL_API_BEGIN(ctxexpr)                 \
  kl_ctx_t ctx__ = (ctxexpr);                 \
  try {                                       \
    if (ctx__) ctx__->last_error.clear();     \
    DeviceGuard guard__(ctx__ ? ctx__->device : 0);
#define KL_API_END                                                     \
  }                                                                    \
  catch (const KlError& e) {                                           \
    return finish(ctx__, e);                                           \
  }                                                                    \
  catch (const std::bad_alloc&) {                                      \
    return finish(ctx__, KlError{KL_ENOMEM, "host allocation failed"}); \
  }                                                                    \
  return KL_OK;

namespace {
// Read and clear the device error word (synchronises).
void check_device_errors(kl_ctx_t ctx) {
  ck(cudaStreamSynchronize(ctx->stream), "stream synchronize");
  int e = 0;
  ck(cudaMemcpy(&e, ctx->err.p, 4, cudaMemcpyDeviceToHost), "read error word");
  if (e) {
    ck(cudaMemset(ctx->err.p, 0, 4), "clear error word");
    if (e & DERR_BOUNDS) raise(KL_EBOUNDS, "device kernel saw an out-of-range id or index");
    if (e & DERR_CAPACITY) raise(KL_ECAPACITY, "an output exceeded its capacity and was truncated");
    if (e & DERR_TIMEOUT) raise(KL_ETIMEOUT, "a bounded device wait gave up");
    if (e & DERR_TMA) raise(KL_ECUDA, "a TMA tensor map could not be encoded (misaligned buffer or pitch)");
  }
}
}  // namespace

// ===========================================================================
// Context
// ===========================================================================
extern "C" int kl_abi_version(void) { return KLEARU_GPU_ABI_VERSION; }

extern "C" kl_status kl_ctx_create(int device, void* stream, kl_ctx_t* out) {
  if (!out) return KL_EINVAL;
  *out = nullptr;
  try {
    int n = 0;
    ck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
    require(device >= 0 && device < n, "device index out of range");
    DeviceGuard g(device);
    auto* c = new kl_ctx_s();
    c->device = device;
    c->stream = static_cast<cudaStream_t>(stream);
    try {
      c->err.alloc(4);
      ck(cudaMemset(c->err.p, 0, 4), "memset");
    } catch (...) {
      delete c;
      throw;
    }
    *out = c;
  } catch (const KlError& e) {
    return e.st;
  }
  return KL_OK;
}
extern "C" kl_status kl_ctx_destroy(kl_ctx_t ctx) {
  if (!ctx) return KL_EINVAL;
  {
    DeviceGuard g(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    ctx->err.~DBuf();
    new (&ctx->err) DBuf();
  }
  delete ctx;
  return KL_OK;
}
extern "C" kl_status kl_ctx_set_stream(kl_ctx_t ctx, void* stream) {
  if (!ctx) return KL_EINVAL;
  ctx->stream = static_cast<cudaStream_t>(stream);
  return KL_OK;
}
extern "C" kl_status kl_ctx_sync(kl_ctx_t ctx) {
  if (!ctx) return KL_EINVAL;
  KL_API_BEGIN(ctx)
  check_device_errors(ctx);
  KL_API_END
}
extern "C" kl_status kl_ctx_check(kl_ctx_t ctx) { return kl_ctx_sync(ctx); }
extern "C" const char* kl_last_error(kl_ctx_t ctx) {
  return ctx ? ctx->last_error.c_str() : g_thread_error.c_str();
}
namespace kl {
void set_thread_error(const std::string& m) { g_thread_error = m; }
}  // namespace kl

// ===========================================================================
// Hash
// ===========================================================================
extern "C" kl_status kl_hash_create(kl_ctx_t ctx, int kind, int input_dim, int k, int num_tables,
                                    int window_size, const kl_hash_params* params_host, kl_hash_t* out) {
  if (!ctx || !out) return KL_EINVAL;
  KL_API_BEGIN(ctx)
  *out = nullptr;
  auto H = make_hash(ctx, kind, input_dim, k, num_tables, window_size, params_host);
  *out = new kl_hash_s{H};
  KL_API_END
}
extern "C" kl_status kl_hash_create_seeded(kl_ctx_t ctx, int kind, int input_dim, int k, int num_tables,
                                           int window_size, float srp_sparsity, uint64_t seed,
                                           kl_hash_t* out) {
  if (!ctx || !out) return KL_EINVAL;
  KL_API_BEGIN(ctx)
  *out = nullptr;
  require(input_dim >= 1 && k >= 1 && num_tables >= 1, "hash: input_dim, k and num_tables must be >= 1");
  require(srp_sparsity >= 0.0f && srp_sparsity <= 1.0f, "SRP: sparsity must be in [0, 1] (srp.rs:50-53)");
  if (kind == KL_HASH_WTA || kind == KL_HASH_DWTA)
    require(window_size >= 1 && window_size <= input_dim, "WTA/DWTA: window_size must be in [1, input_dim]");
  SeededParams sp;
  seeded_params(kind, input_dim, k, num_tables, window_size, srp_sparsity, seed, sp);
  auto H = make_hash(ctx, kind, input_dim, k, num_tables, window_size, &sp.p);
  *out = new kl_hash_s{H};
  KL_API_END
}
extern "C" kl_status kl_hash_destroy(kl_hash_t h) {
  if (!h) return KL_EINVAL;
  delete h;
  return KL_OK;
}
extern "C" kl_status kl_hash_info(kl_hash_t h, int* kind, int* d, int* k, int* L) {
  if (!h) return KL_EINVAL;
  if (kind) *kind = h->h->dh.kind;
  if (d) *d = h->h->dh.d;
  if (k) *k = h->h->dh.k;
  if (L) *L = h->h->dh.L;
  return KL_OK;
}
static kl_status set_projection(HashImpl* H, int mode) {
  if (mode < KL_PROJ_AUTO || mode > KL_PROJ_TENSOR) return KL_EINVAL;
  if (H->tc) H->tc->mode = mode;
  else if (mode == KL_PROJ_TENSOR && (H->dh.kind == KL_HASH_SIMHASH || H->dh.kind == KL_HASH_SRP))
    return KL_EUNSUPPORTED;  // the planes do not fit the tensor-core kernel's shared memory
  return KL_OK;
}
extern "C" kl_status kl_hash_set_projection(kl_hash_t h, int mode) {
  if (!h) return KL_EINVAL;
  return set_projection(h->h.get(), mode);
}
extern "C" kl_status kl_hash_dense_batch(kl_hash_t h, const float* X, int n, int ldx, uint64_t* codes,
                                         float* min_abs_proj) {
  if (!h) return KL_EINVAL;
  KL_API_BEGIN(h->h->ctx)
  require(n >= 0 && (n == 0 || (X && codes && ldx >= h->h->dh.d)), "hash_dense_batch: bad arguments");
  HashOut o;
  o.codes = codes;
  o.min_abs = min_abs_proj;
  launch_hash_dense(h->h->dh, dense_rows(X, KL_DTYPE_F32, n, ldx), o, ctx__->stream);
  ck_launch("hash_dense_batch");
  KL_API_END
}
extern "C" kl_status kl_hash_dense_batch_rows(kl_hash_t h, const void* rows, int n, int ld, int dtype,
                                              uint64_t* codes, float* min_abs_proj) {
  if (!h) return KL_EINVAL;
  KL_API_BEGIN(h->h->ctx)
  require(n >= 0 && (n == 0 || (rows && codes && ld >= h->h->dh.d)), "hash_dense_batch_rows: bad arguments");
  HashOut o;
  o.codes = codes;
  o.min_abs = min_abs_proj;
  launch_hash_dense(h->h->dh, dense_rows(rows, dtype, n, ld), o, ctx__->stream);
  ck_launch("hash_dense_batch_rows");
  KL_API_END
}
extern "C" kl_status kl_hash_sparse_batch(kl_hash_t h, const int32_t* rowptr, const uint32_t* idx,
                                          const float* val, int n, uint64_t* codes, float* min_abs_proj) {
  if (!h) return KL_EINVAL;
  KL_API_BEGIN(h->h->ctx)
  require(n >= 0 && (n == 0 || (rowptr && codes)), "hash_sparse_batch: bad arguments");
  HashOut o;
  o.codes = codes;
  o.min_abs = min_abs_proj;
  launch_hash_sparse(h->h->dh, SparseIn{rowptr, idx, val, n}, o, ctx__->stream);
  ck_launch("hash_sparse_batch");
  KL_API_END
}

// ===========================================================================
// Index
// ===========================================================================
extern "C" kl_status kl_index_create(kl_ctx_t ctx, kl_hash_t h, int bucket_type, int capacity,
                                     kl_index_t* out) {
  if (!ctx || !h || !out) return KL_EINVAL;
  KL_API_BEGIN(ctx)
  *out = nullptr;
  auto I = make_index(ctx, h->h, bucket_type, capacity);
  *out = new kl_index_s{I};
  KL_API_END
}
extern "C" kl_status kl_index_destroy(kl_index_t ix) {
  if (!ix) return KL_EINVAL;
  delete ix;
  return KL_OK;
}
extern "C" kl_status kl_index_set_projection(kl_index_t ix, int mode) {
  if (!ix) return KL_EINVAL;
  return set_projection(ix->ix->hash.get(), mode);
}
extern "C" kl_status kl_index_info(kl_index_t ix, int* L, int* nb, int* cap, int* type) {
  if (!ix) return KL_EINVAL;
  if (L) *L = ix->ix->T.L;
  if (nb) *nb = ix->ix->T.nb;
  if (cap) *cap = ix->ix->T.cap;
  if (type) *type = ix->ix->T.type;
  return KL_OK;
}
extern "C" kl_status kl_index_insert_batch(kl_index_t ix, const uint32_t* ids, const void* rows, int n,
                                           int ld, int dtype) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  require(n >= 0 && (n == 0 || (ids && rows && ld >= I.hash->dh.d)), "insert_batch: bad arguments");
  if (n == 0) return KL_OK;
  I.hash_dense_to_bkt(dense_rows(rows, dtype, n, ld));
  I.insert_from_bkt(ids, n);
  KL_API_END
}
extern "C" kl_status kl_index_insert_sparse_batch(kl_index_t ix, const uint32_t* ids, const int32_t* rowptr,
                                                  const uint32_t* idx, const float* val, int n) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  require(n >= 0 && (n == 0 || (ids && rowptr)), "insert_sparse_batch: bad arguments");
  if (n == 0) return KL_OK;
  I.hash_sparse_to_bkt(SparseIn{rowptr, idx, val, n});
  I.insert_from_bkt(ids, n);
  KL_API_END
}
extern "C" kl_status kl_index_remove(kl_index_t ix, const uint32_t* ids, int n) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  require(n >= 0 && (n == 0 || ids), "remove: bad arguments");
  launch_tables_remove(I.T, ids, n, ctx__->stream);
  ck_launch("remove");
  KL_API_END
}
extern "C" kl_status kl_index_remove_with_weights(kl_index_t ix, const uint32_t* ids, const void* rows,
                                                  int n, int ld, int dtype) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  require(n >= 0 && (n == 0 || (ids && rows && ld >= I.hash->dh.d)), "remove_with_weights: bad arguments");
  if (n == 0) return KL_OK;
  I.hash_dense_to_bkt(dense_rows(rows, dtype, n, ld));
  launch_tables_remove_hashed(I.T, ids, I.bkt.as<uint16_t>(), n, n, ctx__->stream);
  ck_launch("remove_with_weights");
  KL_API_END
}
extern "C" kl_status kl_index_rebuild(kl_index_t ix, const uint32_t* ids, const void* rows, int n, int ld,
                                      int dtype) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  require(n >= 0 && (n == 0 || (rows && ld >= I.hash->dh.d)), "rebuild: bad arguments");
  I.clear();
  if (n == 0) return KL_OK;
  I.hash_dense_to_bkt(dense_rows(rows, dtype, n, ld));
  I.insert_from_bkt(ids, n);
  KL_API_END
}
extern "C" kl_status kl_index_clear(kl_index_t ix) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  I.clear();
  KL_API_END
}
extern "C" kl_status kl_index_query_batch(kl_index_t ix, const float* X, int n, int ldx, int mode,
                                          uint32_t* out_ids, uint32_t* out_counts, int32_t* out_offsets,
                                          int32_t capacity, int32_t* overflow) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  require(mode == KL_QUERY_COUNTS || mode == KL_QUERY_UNION, "query: unknown mode");
  require(n >= 0 && out_offsets && (n == 0 || (X && ldx >= I.hash->dh.d)), "query: bad arguments");
  require(capacity >= 0 && (capacity == 0 || out_ids), "query: bad capacity");
  if (n == 0) {
    ck(cudaMemsetAsync(out_offsets, 0, 4, ctx__->stream), "memset");
    return KL_OK;
  }
  I.hash_dense_to_bkt(dense_rows(X, KL_DTYPE_F32, n, ldx));
  I.query(n, mode, out_ids, out_counts, out_offsets, capacity, overflow);
  KL_API_END
}
// SparseInferenceEngine::infer / infer_linear for a batch of inputs.
static void bolt_body(IndexImpl& I, const void* W, int dtype, int64_t ldw, const float* bias, int N, const float* X,
                      int n, int ldx, float mult, int base_top_k, int relu, uint32_t* out_ids, float* out_act,
                      int32_t* out_n, int stride) {
  require(dtype == KL_DTYPE_F32 || dtype == KL_DTYPE_BF16, "bolt: dtype must be KL_DTYPE_F32 or KL_DTYPE_BF16");
  require(n >= 0 && N >= 0 && base_top_k >= 0 && stride >= 0, "bolt: negative size");
  require(n == 0 || (X && W && out_ids && out_act && out_n && ldx >= I.hash->dh.d && ldw >= I.hash->dh.d),
          "bolt: bad arguments");
  support(I.T.L * I.T.cap <= probe_max_items(), "bolt: num_tables * bucket_capacity exceeds the probe's limit");
  support(bolt_smem_bytes(I.hash->dh.d, I.T.L * I.T.cap) <= 200 * 1024, "bolt: input_dim too large");
  if (n == 0) return;
  // effective_k = (base_top_k as f32 * sparsity_multiplier) as usize (sparse_inference.rs:40)
  const float ek = (float)base_top_k * mult;
  const int k = !(ek > 0.0f) ? 0 : (ek >= 2147483647.0f ? 2147483647 : (int)ek);
  I.hash_dense_to_bkt(dense_rows(X, KL_DTYPE_F32, n, ldx));
  BoltArgs a;
  a.cand_stride = I.probe_padded(n);
  a.cand_ids = I.qids.as<uint32_t>();
  a.cand_cnt = I.qcnt.as<uint32_t>();
  a.cand_n = I.qn.as<int32_t>();
  a.nq = n;
  a.L = I.T.L;
  a.k = k;
  a.N = N;
  a.d = I.hash->dh.d;
  a.X = X;
  a.ldx = ldx;
  a.W = W;
  a.wdtype = dtype;
  a.ldw = ldw;
  a.bias = bias;
  a.relu = relu;
  a.out_ids = out_ids;
  a.out_act = out_act;
  a.out_n = out_n;
  a.out_stride = stride;
  a.err = I.ctx->err.as<int>();
  launch_bolt(a, I.ctx->stream);
  ck_launch("bolt");
}
extern "C" kl_status kl_bolt_infer_batch(kl_index_t ix, const void* weights, int dtype, int ld, const float* bias,
                                         int num_neurons, const float* X, int n, int ldx, float sparsity_multiplier,
                                         int base_top_k, int relu, uint32_t* out_ids, float* out_act,
                                         int32_t* out_n, int stride) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  bolt_body(I, weights, dtype, ld, bias, num_neurons, X, n, ldx, sparsity_multiplier, base_top_k, relu, out_ids,
            out_act, out_n, stride);
  KL_API_END
}
extern "C" kl_status kl_index_query_sparse_batch(kl_index_t ix, const int32_t* rowptr, const uint32_t* idx,
                                                 const float* val, int n, int mode, uint32_t* out_ids,
                                                 uint32_t* out_counts, int32_t* out_offsets, int32_t capacity,
                                                 int32_t* overflow) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  require(mode == KL_QUERY_COUNTS || mode == KL_QUERY_UNION, "query: unknown mode");
  require(n >= 0 && out_offsets && (n == 0 || rowptr), "query_sparse: bad arguments");
  require(capacity >= 0 && (capacity == 0 || out_ids), "query: bad capacity");
  if (n == 0) {
    ck(cudaMemsetAsync(out_offsets, 0, 4, ctx__->stream), "memset");
    return KL_OK;
  }
  I.hash_sparse_to_bkt(SparseIn{rowptr, idx, val, n});
  I.query(n, mode, out_ids, out_counts, out_offsets, capacity, overflow);
  KL_API_END
}
extern "C" kl_status kl_index_export(kl_index_t ix, uint32_t* ids, uint32_t* lens, uint64_t* counts) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  const size_t LB = (size_t)I.T.L * I.T.nb;
  cudaStream_t st = ctx__->stream;
  if (ids) ck(cudaMemcpyAsync(ids, I.T.ids, LB * I.T.cap * 4, cudaMemcpyDeviceToDevice, st), "export");
  if (lens) ck(cudaMemcpyAsync(lens, I.T.len, LB * 4, cudaMemcpyDeviceToDevice, st), "export");
  if (counts) ck(cudaMemcpyAsync(counts, I.T.cnt, LB * 8, cudaMemcpyDeviceToDevice, st), "export");
  KL_API_END
}
extern "C" kl_status kl_index_import(kl_index_t ix, const uint32_t* ids, const uint32_t* lens,
                                     const uint64_t* counts) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  require(ids && lens, "import: ids and lens required");
  const size_t LB = (size_t)I.T.L * I.T.nb;
  cudaStream_t st = ctx__->stream;
  ck(cudaMemcpyAsync(I.T.ids, ids, LB * I.T.cap * 4, cudaMemcpyDeviceToDevice, st), "import");
  ck(cudaMemcpyAsync(I.T.len, lens, LB * 4, cudaMemcpyDeviceToDevice, st), "import");
  if (counts) ck(cudaMemcpyAsync(I.T.cnt, counts, LB * 8, cudaMemcpyDeviceToDevice, st), "import");
  else ck(cudaMemsetAsync(I.T.cnt, 0, LB * 8, st), "import");
  KL_API_END
}

// ===========================================================================
// AdaptiveScheduler (crates/klearu-mongoose/src/scheduler.rs:44-213): the
// drift check hashes the sampled rows on the GPU and counts, on the GPU, the
// rows whose code changed in any table; counters, drift and EMA are the
// reference's host arithmetic (f32).
// ===========================================================================
struct kl_adaptive_s {
  kl_ctx_t ctx;
  std::shared_ptr<HashImpl> hash;
  size_t min_interval = 0, max_interval = 0;
  float sample_fraction = 0.f, drift_threshold = 0.f;
  float drift_ema = 0.f, ema_alpha = 0.3f;
  size_t steps_since_rebuild = 0, steps_since_check = 0;
  int S = 0;  // sampled rows
  DBuf idx, base, cur, rows, changed;
};

namespace {
// rows[i] = f32 copy of row idx[i] (zeros for indices >= n); element (r, c)
// of the source at r * ld_row + c * ld_elem (row- or feature-major weights)
__global__ void adaptive_gather_kernel(const void* X, int dtype, int64_t ld_row, int64_t ld_elem, int n,
                                       const uint32_t* idx, int S, int d, float* out) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)S * d) return;
  const int i = (int)(g / d), c = (int)(g % d);
  const uint32_t r = idx[i];
  float v = 0.f;
  if (r < (uint32_t)n) {
    const int64_t o = (int64_t)r * ld_row + (int64_t)c * ld_elem;
    v = dtype == KL_DTYPE_BF16 ? to_f(static_cast<const __nv_bfloat16*>(X)[o])
                               : static_cast<const float*>(X)[o];
  }
  out[g] = v;
}
// changed += number of sampled rows (< n) whose code differs in any table
__global__ void adaptive_compare_kernel(const uint64_t* cur, const uint64_t* base, const uint32_t* idx, int S,
                                        int L, int n, int* changed) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= S || idx[i] >= (uint32_t)n) return;
  bool any = false;
  for (int t = 0; t < L && !any; ++t) any = cur[(int64_t)i * L + t] != base[(int64_t)i * L + t];
  if (any) atomicAdd(changed, 1);
}

// The rows a scheduler watches: n rows of d elements, element (r, c) at
// X[r * ld_row + c * ld_elem].
struct RowsView {
  const void* X;
  int dtype;
  int64_t ld_row, ld_elem;
  int n;
};

void adaptive_hash(kl_adaptive_s* a, const RowsView& rv, DBuf& codes) {
  cudaStream_t st = a->ctx->stream;
  const DevHash& h = a->hash->dh;
  adaptive_gather_kernel<<<(unsigned)ceil_div((int64_t)a->S * h.d, 256), 256, 0, st>>>(
      rv.X, rv.dtype, rv.ld_row, rv.ld_elem, rv.n, a->idx.as<uint32_t>(), a->S, h.d, a->rows.as<float>());
  count_launch();
  ck_launch("adaptive gather");
  DenseIn in;
  in.X = a->rows.p;
  in.dtype = KL_DTYPE_F32;
  in.ld_row = h.d;
  in.ld_elem = 1;
  in.n = a->S;
  HashOut o;
  o.codes = codes.as<uint64_t>();
  launch_hash_dense(h, in, o, st);
  ck_launch("adaptive hash");
}

// AdaptiveScheduler::record_baseline (scheduler.rs:89-125).
void adaptive_record(kl_adaptive_s* a, const std::shared_ptr<HashImpl>& hash, const RowsView& rv,
                     const uint32_t* sampled_host, int n_sampled, uint64_t seed) {
  const int n = rv.n;
  std::vector<uint32_t> idx;
  if (sampled_host) {
    require(n_sampled >= 0, "adaptive: n_sampled must be >= 0");
    idx.assign(sampled_host, sampled_host + n_sampled);
  } else {
    // scheduler.rs:104-110: ceil(n * fraction) clamped to [1, n] indices of a
    // seeded shuffle, sorted (this library's SplitMix64 stream, not StdRng)
    const size_t S = std::min<size_t>((size_t)n, std::max<size_t>(1, (size_t)std::ceil((float)n * a->sample_fraction)));
    std::vector<uint32_t> perm((size_t)n);
    for (int i = 0; i < n; ++i) perm[(size_t)i] = (uint32_t)i;
    SplitMix rng{seed};
    for (size_t i = (size_t)n - 1; n > 0 && i > 0; --i) std::swap(perm[i], perm[(size_t)(rng.next() % (uint64_t)(i + 1))]);
    idx.assign(perm.begin(), perm.begin() + S);
  }
  std::sort(idx.begin(), idx.end());
  a->hash = hash;
  a->S = (int)idx.size();
  const int L = a->hash->dh.L;
  a->steps_since_rebuild = 0;
  a->steps_since_check = 0;
  a->drift_ema = 0.f;
  if (idx.empty()) return;  // no neurons: nothing to watch (scheduler.rs tests: empty_neurons)
  a->idx.alloc(idx.size() * 4);
  a->base.alloc(idx.size() * L * 8);
  a->cur.alloc(idx.size() * L * 8);
  a->rows.alloc(idx.size() * (size_t)a->hash->dh.d * 4);
  cudaStream_t st = a->ctx->stream;
  ck(cudaMemcpyAsync(a->idx.p, idx.data(), idx.size() * 4, cudaMemcpyHostToDevice, st), "upload");
  adaptive_hash(a, rv, a->base);
  ck(cudaStreamSynchronize(st), "sync");
}

// AdaptiveScheduler::should_rebuild (scheduler.rs:130-160) with
// estimate_drift (scheduler.rs:163-195) on the GPU.  A drift check reads the
// changed count back, so it waits for the work queued before it.
bool adaptive_check(kl_adaptive_s* a, const RowsView& rv) {
  a->steps_since_rebuild += 1;
  a->steps_since_check += 1;
  if (a->steps_since_rebuild >= a->max_interval) {  // forced (scheduler.rs:141-145)
    a->steps_since_rebuild = 0;
    a->steps_since_check = 0;
    return true;
  }
  if (a->steps_since_check < a->min_interval) return false;
  float drift = 0.f;
  if (a->hash && a->S > 0) {
    cudaStream_t st = a->ctx->stream;
    adaptive_hash(a, rv, a->cur);
    ck(cudaMemsetAsync(a->changed.p, 0, 4, st), "memset");
    adaptive_compare_kernel<<<(unsigned)ceil_div(a->S, 256), 256, 0, st>>>(
        a->cur.as<uint64_t>(), a->base.as<uint64_t>(), a->idx.as<uint32_t>(), a->S, a->hash->dh.L, rv.n,
        a->changed.as<int>());
    count_launch();
    ck_launch("adaptive compare");
    int changed = 0;
    ck(cudaMemcpyAsync(&changed, a->changed.p, 4, cudaMemcpyDeviceToHost, st), "copy");
    ck(cudaStreamSynchronize(st), "sync");
    drift = (float)changed / (float)a->S;
  }
  a->drift_ema = a->ema_alpha * drift + (1.0f - a->ema_alpha) * a->drift_ema;
  a->steps_since_check = 0;
  if (a->drift_ema >= a->drift_threshold) {
    a->steps_since_rebuild = 0;
    return true;
  }
  return false;
}
}  // namespace

extern "C" kl_status kl_adaptive_create(kl_ctx_t ctx, uint64_t min_interval, uint64_t max_interval,
                                        float sample_fraction, float drift_threshold, kl_adaptive_t* out) {
  if (!ctx || !out) return KL_EINVAL;
  KL_API_BEGIN(ctx)
  *out = nullptr;
  require(min_interval <= max_interval, "adaptive: min_interval must be <= max_interval (scheduler.rs:61-64)");
  require(sample_fraction >= 0.f && sample_fraction <= 1.f, "adaptive: sample_fraction must be in [0, 1]");
  require(drift_threshold >= 0.f && drift_threshold <= 1.f, "adaptive: drift_threshold must be in [0, 1]");
  auto* a = new kl_adaptive_s();
  a->ctx = ctx;
  a->min_interval = (size_t)min_interval;
  a->max_interval = (size_t)max_interval;
  a->sample_fraction = sample_fraction;
  a->drift_threshold = drift_threshold;
  a->changed.alloc(4);
  *out = a;
  KL_API_END
}
extern "C" kl_status kl_adaptive_destroy(kl_adaptive_t a) {
  if (!a) return KL_EINVAL;
  {
    DeviceGuard g(a->ctx->device);
    cudaStreamSynchronize(a->ctx->stream);
    delete a;
  }
  return KL_OK;
}
extern "C" kl_status kl_adaptive_record_baseline(kl_adaptive_t a, kl_hash_t h, const void* rows, int n, int ld,
                                                 int dtype, const uint32_t* sampled_host, int n_sampled,
                                                 uint64_t seed) {
  if (!a || !h) return KL_EINVAL;
  KL_API_BEGIN(a->ctx)
  require(n >= 0 && (n == 0 || (rows && ld >= h->h->dh.d)), "adaptive: bad rows");
  require(dtype == KL_DTYPE_F32 || dtype == KL_DTYPE_BF16, "adaptive: dtype must be F32 or BF16");
  adaptive_record(a, h->h, RowsView{rows, dtype, ld, 1, n}, sampled_host, n_sampled, seed);
  KL_API_END
}
extern "C" kl_status kl_adaptive_should_rebuild(kl_adaptive_t a, const void* rows, int n, int ld, int dtype,
                                                int* rebuild_host) {
  if (!a || !rebuild_host) return KL_EINVAL;
  KL_API_BEGIN(a->ctx)
  *rebuild_host = 0;
  if (a->hash && a->S > 0 && a->steps_since_rebuild + 1 < a->max_interval &&
      a->steps_since_check + 1 >= a->min_interval) {
    require(rows && ld >= a->hash->dh.d, "adaptive: bad rows");
    require(dtype == KL_DTYPE_F32 || dtype == KL_DTYPE_BF16, "adaptive: dtype must be F32 or BF16");
  }
  *rebuild_host = adaptive_check(a, RowsView{rows, dtype, ld, 1, n}) ? 1 : 0;
  KL_API_END
}
extern "C" kl_status kl_adaptive_notify_rebuild(kl_adaptive_t a) {
  if (!a) return KL_EINVAL;
  a->steps_since_rebuild = 0;
  a->steps_since_check = 0;
  return KL_OK;
}
extern "C" kl_status kl_adaptive_state(kl_adaptive_t a, float* drift_ema_host, uint64_t* steps_since_rebuild_host,
                                       int* n_sampled_host) {
  if (!a) return KL_EINVAL;
  if (n_sampled_host) *n_sampled_host = a->S;
  if (drift_ema_host) *drift_ema_host = a->drift_ema;
  if (steps_since_rebuild_host) *steps_since_rebuild_host = (uint64_t)a->steps_since_rebuild;
  return KL_OK;
}

// ===========================================================================
// Network
// ===========================================================================
namespace {

// RebuildScheduler (lsh/maintenance.rs:28-98).
struct Scheduler {
  uint64_t base = 100;
  double decay = 0.1;
  uint64_t count = 0, next = 100, cur = 0;
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

struct Layer {
  kl_layer_config cfg{};
  int d = 0, N = 0;
  bool fm = false;   // feature-major weights (layer 0)
  int ldw = 0;       // weight row pitch (elements)
  int ldN = 0;       // pitch of dense rows over this layer's neurons
  int ldd = 0;       // pitch of dense rows over this layer's inputs
  int stride = 0;    // max active per example
  int nchunk = 0;
  int id_bits = 0;
  uint32_t id_base = 0;  // global id of row 0 (the rank's slice of a sharded output layer)
  int f0 = 0, nf = 0;    // feature rows whose optimizer state this rank updates (layer 0; all rows unsharded)
  DBuf W, b, m, v, mb, vb;
  std::shared_ptr<IndexImpl> index;
  // per-step buffers
  DBuf bkt, ids, cnt, pre, post, lg, h, dx_in, dxpart, lgd, tmask, gfeat;
  DBuf dmark, dtouched, dslot, dlg;  // dense-collision update scratch (row-major layers)
  int64_t dldb = 0;  // sample pitch of the dense update's gradient matrix (0: segmented path)
  bool premarked = false;  // this step's rows were marked before the forward, which filled the matrix
  DBuf hist, cur, touched, ctr, ent_s, ent_v, fslot, flong;
  size_t ent_cap = 0;
  DBuf stats;  // u64 [3]: active_sum, touched_rows, input_nnz
  uint64_t examples = 0, steps = 0, rebuilds = 0, input_nnz = 0;
  // sharded output layer with a selection over all shards (TopK below the
  // candidate count, Threshold): every local candidate with its table count
  bool shard_select = false;
  int cstride = 0;
  DBuf cids, ccnt, ccn;

  ActiveSet act() const {
    return ActiveSet{ids.as<uint32_t>(), cnt.as<int32_t>(), stride, pre.as<float>(), post.as<float>(),
                     lg.as<float>()};
  }
};

}  // namespace

// Per-example capacities of the sharded batch exchange (input nnz, labels).
#define KL_SHARD_NNZ_PER_EXAMPLE_H 512
// Per-example capacities of the graph-captured step's batch buffers.
#define KL_GRAPH_NNZ_PER_EXAMPLE 512
#define KL_GRAPH_LABELS_PER_EXAMPLE 32
#define KL_SHARD_LABELS_PER_EXAMPLE_H 32
void nccl_ck(ncclResult_t r, const char* what);

namespace {
__global__ void loss_final_kernel(const float* acc, int B, float* out1, float* out2) {
  const float v = B > 0 ? __fdiv_rn(*acc, (float)B) : 0.0f;
  if (out1) *out1 = v;
  if (out2) *out2 = v;
}
void launch_loss_final(const float* acc, int B, float* out1, float* out2, cudaStream_t st) {
  loss_final_kernel<<<1, 1, 0, st>>>(acc, B, out1, out2);
  count_launch();
}
}  // namespace

struct kl_net_s {
  kl_ctx_t ctx;
  kl_net_config cfg{};
  std::vector<kl_layer_config> layer_cfgs;
  std::vector<std::unique_ptr<Layer>> layers;
  int wdtype = KL_DTYPE_F32;
  int max_batch = 0;
  uint64_t step = 0;
  Scheduler sched;
  DBuf labprob, loss_acc, rb_bkt, rb_scratch;
  size_t labprob_cap = 0;
  // host-batch ingestion (kl_net_train_step_host): two slots, each a pinned
  // host buffer and a device buffer holding one packed CSR batch.  h2d marks
  // the slot's upload done, used the end of the step that read it.
  struct HostSlot {
    void* pinned = nullptr;
    DBuf dev;
    size_t cap = 0;
    cudaEvent_t h2d = nullptr, used = nullptr;
  };
  HostSlot hslots[2];
  int hnext = 0;
  cudaStream_t copy_stream = nullptr;
  // sharded step: the hidden-weight all-gather's stream and its ordering events
  cudaStream_t comm_stream = nullptr;
  cudaEvent_t ev_hidden = nullptr, ev_gather = nullptr, ev_cnt = nullptr, ev_cnt_done = nullptr;
  DBuf sel_hist, sel_cut, sel_eq_all;  // global selection over the output shards
  // neuron sharding of the output layer (kl_net_create_sharded)
  int rank = 0, nranks = 1;
  ncclComm_t comm = nullptr;
  // Failure detection of a sharded net (kl_net_set_comm_timeout).  With a
  // timeout set, the net's synchronising waits poll the streams and the
  // communicator's asynchronous error instead of blocking; a failed or timed-out
  // wait aborts the communicator, and every later call that needs it returns
  // KL_ENCCL.  stuck: the streams had not drained after the abort, so the
  // destructor must not wait on them.
  int comm_timeout_ms = 0;
  bool comm_aborted = false, stuck = false;
  std::string comm_abort_why;
  void require_comm() {
    if (comm_aborted) raise(KL_ENCCL, "the communicator was aborted (" + comm_abort_why + "); recreate the network");
  }
  void abort_comm(const std::string& why) {
    if (comm) ncclCommAbort(comm);
    comm = nullptr;
    comm_aborted = true;
    comm_abort_why = why;
  }
  bool streams_ready() {
    const cudaStream_t ss[4] = {ctx->stream, comm_stream, side_stream, copy_stream};
    for (int i = 0; i < 4; ++i) {
      if (i > 0 && !ss[i]) continue;  // streams the net has not created yet
      const cudaError_t e = cudaStreamQuery(ss[i]);
      if (e == cudaErrorNotReady) return false;
      ck(e, "stream query");
    }
    return true;
  }
  // Before a host read that would block inside CUDA (a copy into pageable
  // memory, an event wait): the bounded wait, when one is set.
  void guard_blocking_read(const void* host_dst) {
    if (nranks <= 1 || comm_timeout_ms <= 0 || comm_aborted) return;
    if (host_dst) {
      cudaPointerAttributes a{};
      if (cudaPointerGetAttributes(&a, host_dst) == cudaSuccess && a.type == cudaMemoryTypeHost) return;
      cudaGetLastError();
    }
    wait_streams();
  }
  // Wait for the net's streams; on a sharded net with a timeout, a bounded
  // wait that aborts the communicator on its error or at the deadline.
  void wait_streams() {
    if (nranks <= 1 || comm_timeout_ms <= 0 || comm_aborted) {
      ck(cudaStreamSynchronize(ctx->stream), "sync");
      return;
    }
    const WaitReport r = bounded_wait(
        [&] { return streams_ready(); },
        [&] {
          ncclResult_t a = ncclSuccess;
          const ncclResult_t q = ncclCommGetAsyncError(comm, &a);
          if (q != ncclSuccess) return (int)q;
          return (a == ncclSuccess || a == ncclInProgress) ? 0 : (int)a;
        },
        [&] { abort_comm(""); }, wall_ms, sleep_ms, (double)comm_timeout_ms, (double)comm_timeout_ms);
    if (r.result == WaitResult::kDone) return;
    stuck = !r.drained;
    const std::string tail = r.drained ? "" : "; device work was still pending after the abort";
    if (r.result == WaitResult::kCommError) {
      comm_abort_why = std::string("NCCL error: ") + ncclGetErrorString((ncclResult_t)r.comm_error);
      raise(KL_ENCCL, "a peer rank failed (" + comm_abort_why + "); communicator aborted" + tail);
    }
    comm_abort_why = "no progress within " + std::to_string(comm_timeout_ms) + " ms";
    raise(KL_ETIMEOUT, "sharded step made " + comm_abort_why + " (a peer rank is missing?); communicator aborted" + tail);
  }
  int rank_batch = 0;             // examples per rank per step (cfg max_batch)
  int nnz_cap = 0, lab_cap = 0;   // per-rank capacities of the batch exchange
  ShardLayout shl{};
  DBuf dsend, drecv, g_rowptr, g_idx, g_val, g_lptr, g_labels, gcnt, tmask_all;
  std::vector<std::unique_ptr<kl_index_s>> index_handles;

  // Phase profiler: CUDA events on the context stream around each phase of
  // each layer; read (and synchronised) by kl_net_profile_read.
  bool prof = false;
  struct Ev {
    cudaEvent_t a, b;
    int layer, phase;
  };
  std::vector<Ev> pending;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pool;
  std::vector<double> prof_ms;
  std::vector<uint64_t> prof_calls;
  // events around layer 0's streaming Adam launch (KL_PHASE_STREAM)
  int stream_ev = -1;
  static void stream_hook(void* self, int after) {
    auto* n = static_cast<kl_net_s*>(self);
    if (!after) n->stream_ev = n->prof_begin(0, KL_PHASE_STREAM);
    else n->prof_end(n->stream_ev);
  }
  int prof_begin(int layer, int phase) {
    if (!prof) return -1;
    std::pair<cudaEvent_t, cudaEvent_t> e;
    if (!pool.empty()) {
      e = pool.back();
      pool.pop_back();
    } else {
      ck(cudaEventCreate(&e.first), "event");
      ck(cudaEventCreate(&e.second), "event");
    }
    ck(cudaEventRecord(e.first, ctx->stream), "event");
    pending.push_back(Ev{e.first, e.second, layer, phase});
    return (int)pending.size() - 1;
  }
  void prof_end(int i) {
    if (i >= 0) ck(cudaEventRecord(pending[i].b, ctx->stream), "event");
  }
  void prof_collect() {
    ck(cudaStreamSynchronize(ctx->stream), "sync");
    prof_ms.resize(layers.size() * KL_NPHASES, 0.0);
    prof_calls.resize(layers.size() * KL_NPHASES, 0);
    for (auto& e : pending) {
      float ms = 0.0f;
      ck(cudaEventElapsedTime(&ms, e.a, e.b), "elapsed");
      prof_ms[(size_t)e.layer * KL_NPHASES + e.phase] += ms;
      prof_calls[(size_t)e.layer * KL_NPHASES + e.phase] += 1;
      pool.emplace_back(e.a, e.b);
    }
    pending.clear();
  }
  struct Phase {
    kl_net_s* n;
    int i;
    Phase(kl_net_s* net, int layer, int phase) : n(net), i(net->prof_begin(layer, phase)) {}
    ~Phase() { n->prof_end(i); }
  };
  ~kl_net_s() {
    for (auto& h : hslots) {
      if (h.h2d) cudaEventSynchronize(h.h2d);
      if (h.pinned) cudaFreeHost(h.pinned);
      if (h.h2d) cudaEventDestroy(h.h2d);
      if (h.used) cudaEventDestroy(h.used);
    }
    if (copy_stream) cudaStreamDestroy(copy_stream);
    if (comm_stream) cudaStreamSynchronize(comm_stream), cudaStreamDestroy(comm_stream);
    if (side_stream) cudaStreamSynchronize(side_stream), cudaStreamDestroy(side_stream);
    if (ev_fork) cudaEventDestroy(ev_fork);
    if (ev_join) cudaEventDestroy(ev_join);
    if (ev_hidden) cudaEventDestroy(ev_hidden);
    if (ev_gather) cudaEventDestroy(ev_gather);
    if (ev_cnt) cudaEventDestroy(ev_cnt);
    if (ev_cnt_done) cudaEventDestroy(ev_cnt_done);
    if (gexec) cudaGraphExecDestroy(gexec);
    if (sh_gexec) cudaGraphExecDestroy(sh_gexec);
    if (cap_stream) cudaStreamDestroy(cap_stream);
    if (comm) ncclCommDestroy(comm);
    for (auto& e : pending) pool.emplace_back(e.a, e.b);
    for (auto& e : pool) {
      cudaEventDestroy(e.first);
      cudaEventDestroy(e.second);
    }
  }

  void rebuild_layer(Layer& L) {
    Phase ph(this, layer_index_of(L), KL_PHASE_REBUILD);
    cudaStream_t st = ctx->stream;
    IndexImpl& I = *L.index;
    DenseIn in;
    in.X = L.W.p;
    in.dtype = wdtype;
    in.n = L.N;
    if (L.fm) {
      in.ld_row = 1;
      in.ld_elem = L.ldw;
    } else {
      in.ld_row = L.ldw;
      in.ld_elem = 1;
    }
    rb_bkt.alloc((size_t)I.T.L * L.N * 2);
    HashOut o;
    o.bkt = rb_bkt.as<uint16_t>();
    o.bkt_ld = L.N;
    o.nb_mask = (uint32_t)(I.T.nb - 1);
    launch_hash_dense(I.hash->dh, in, o, st);
    ck_launch("rebuild hash");
    I.clear();
    rb_scratch.alloc(insert_scratch_bytes(I.T, L.N));
    InsertScratch s;
    carve_insert_scratch(I.T, L.N, rb_scratch.p, &s);
    launch_tables_insert(I.T, nullptr, rb_bkt.as<uint16_t>(), L.N, L.N, s, ctx->err.as<int>(), st);
    ck_launch("rebuild insert");
    L.rebuilds++;
  }
  int layer_index_of(const Layer& L) const {
    for (size_t i = 0; i < layers.size(); ++i)
      if (layers[i].get() == &L) return (int)i;
    return 0;
  }
  void rebuild_all() {
    for (auto& L : layers) rebuild_layer(*L);
  }

  // Rebuild policy.  KL_REBUILD_SCHEDULE: the reference's RebuildScheduler
  // (net.rs:109-116), all layers together.  KL_REBUILD_ADAPTIVE: one mongoose
  // AdaptiveScheduler per layer (scheduler.rs:44-213), each layer rebuilt when
  // its own sampled hash codes drift, then a new baseline is recorded.
  kl_rebuild_policy policy{};
  std::vector<std::unique_ptr<kl_adaptive_s>> adapt;
  RowsView rows_of(const Layer& L) const {
    return L.fm ? RowsView{L.W.p, wdtype, 1, L.ldw, L.N} : RowsView{L.W.p, wdtype, L.ldw, 1, L.N};
  }
  uint64_t adaptive_seed(int l) const {
    return policy.seed + (uint64_t)l * 1000003ULL + layers[(size_t)l]->rebuilds * 7919ULL;
  }
  void after_step() {
    if (policy.kind != KL_REBUILD_ADAPTIVE) {
      if (sched.should_rebuild(step)) rebuild_all();
      return;
    }
    for (size_t l = 0; l < layers.size(); ++l) {
      Layer& L = *layers[l];
      if (adaptive_check(adapt[l].get(), rows_of(L))) {
        rebuild_layer(L);
        adaptive_record(adapt[l].get(), L.index->hash, rows_of(L), nullptr, 0, adaptive_seed((int)l));
      }
    }
  }

  // Optimizer constants of the current step, copied to the device before
  // the step's kernels (they read them from dopt).
  DBuf dopt;
  OptStep opt_host{};
  void upload_opt(double lr) {
    opt_host = opt_step(lr);
    launch_set_opt(dopt.as<OptStep>(), opt_host, ctx->stream);
    ck_launch("optimizer step");
  }
  OptStep opt_step(double lr) const {
    OptStep o;
    o.opt = cfg.optimizer;
    o.lr = (float)lr;
    o.b1 = 0.9f;
    o.b2 = 0.999f;
    o.eps = 1e-8f;
    o.omb1 = 1.0f - o.b1;
    o.omb2 = 1.0f - o.b2;
    const uint64_t t = std::max<uint64_t>(step, 1);
    o.c1 = 1.0f - powi_f32(o.b1, (int)t);
    o.c2 = 1.0f - powi_f32(o.b2, (int)t);
    o.mom = 0.9f;
    return o;
  }

  // Forward of nq examples starting at example s0 of the batch (views by
  // pointer offset: CSR offsets stay absolute).  train=true also computes
  // the loss gradient in the output layer.
  void forward(const kl_batch& b, int s0, int nq, bool train) {
    for (int l = 0; l < (int)layers.size(); ++l) forward_layer(l, b, s0, nq, train);
  }

  // One layer of the forward.  Layer 0 reads examples [s0, s0+nq) of the batch
  // and writes its activations to rows [hrow0, hrow0+nq) of its h; later
  // layers read rows [0, nq) of the previous layer's h.  `after_probe` runs
  // between the probe and the active-row kernels (the sharded step's global
  // empty-selection fallback).
  // Arguments of the row-major active-row kernel of layer l (l >= 1) for the
  // examples from s0 of batch b.
  RmArgs rm_args(int l, const kl_batch& b, int s0, float* hout) {
    Layer& L = *layers[l];
    const Layer& P = *layers[l - 1];
    RmArgs ra{};
    ra.W = L.W.p;
    ra.wdtype = wdtype;
    ra.ldw = L.ldw;
    ra.d = L.d;
    ra.bias = L.b.as<float>();
    ra.act = L.cfg.activation;
    ra.X = P.h.as<float>();
    ra.ldx = P.ldN;
    ra.A = L.act();
    ra.h = hout;
    ra.ldh = L.ldN;
    ra.dxpart = L.dxpart.as<float>();
    ra.nchunk = L.nchunk;
    ra.lab_ptr = b.label_ptr + s0;
    ra.labels = b.labels;
    ra.labprob = labprob.as<float>();
    ra.err = ctx->err.as<int>();
    ra.id_base = L.id_base;
    ra.only_empty = nullptr;
    ra.lgd_dense = nullptr;
    ra.slot_of = nullptr;
    ra.ldb = 0;
    return ra;
  }
  DenseScratch dense_scratch(Layer& L) {
    return DenseScratch{L.dmark.as<uint32_t>(), L.dtouched.as<uint32_t>(), L.dslot.as<uint32_t>(),
                        L.ctr.as<uint32_t>(), L.dlg.as<float>(), L.dldb};
  }
  void forward_layer(int l, const kl_batch& b, int s0, int nq, bool train, int hrow0 = 0,
                     const std::function<void(Layer&)>& after_probe = nullptr) {
    cudaStream_t st = ctx->stream;
    const int nL = (int)layers.size();
    SparseIn in{b.rowptr + s0, b.idx, b.val, nq};
    {
      Layer& L = *layers[l];
      const bool last = l == nL - 1;
      IndexImpl& I = *L.index;
      HashOut ho;
      ho.bkt = L.bkt.as<uint16_t>();
      ho.bkt_ld = max_batch;
      ho.nb_mask = (uint32_t)(I.T.nb - 1);
      Phase ph_hash(this, l, KL_PHASE_HASH);
      if (l == 0) {
        launch_hash_sparse(I.hash->dh, in, ho, st);
      } else {
        const Layer& P = *layers[l - 1];
        DenseIn di;
        di.X = P.h.p;
        di.dtype = KL_DTYPE_F32;
        di.ld_row = P.ldN;
        di.ld_elem = 1;
        di.n = nq;
        launch_hash_dense(I.hash->dh, di, ho, st);
      }
      ck_launch("layer hash");
      ph_hash.~Phase();
      new (&ph_hash) Phase(this, l, KL_PHASE_PROBE);
      ProbeArgs pa;
      pa.T = I.T;
      pa.bkt = L.bkt.as<uint16_t>();
      pa.bkt_ld = max_batch;
      pa.nq = nq;
      pa.N = L.N;
      pa.sampling = L.cfg.sampling;
      pa.top_k = L.cfg.top_k;
      pa.threshold = L.cfg.sampling_threshold;
      pa.id_bits = L.id_bits;
      pa.out_ids = L.ids.as<uint32_t>();
      pa.out_stride = L.stride;
      pa.out_n = L.cnt.as<int32_t>();
      pa.err = ctx->err.as<int>();
      pa.stat_active = L.stats.as<unsigned long long>();
      pa.fallback = !(last && nranks > 1);
      if (last && L.shard_select) {  // every local candidate; shard_select_exchange selects
        pa.sampling = KL_SAMPLING_VANILLA;
        pa.out_ids = L.cids.as<uint32_t>();
        pa.out_counts = L.ccnt.as<uint32_t>();
        pa.out_stride = L.cstride;
        pa.out_n = L.ccn.as<int32_t>();
        pa.stat_active = nullptr;
      }
      launch_probe(pa, st);
      ck_launch("probe");
      if (after_probe) after_probe(L);
      // fused train step with the dense update: mark the touched rows now (part
      // of building the active sets) so that the forward stores its gradients
      // straight into the update's matrix; a sharded step marks its fallback
      // examples' rows before their pass
      L.premarked = false;
      if (!L.fm && last && train && L.cfg.activation != KL_ACT_SOFTMAX && L.dldb > 0) {
        ck(cudaMemsetAsync(L.ctr.p, 0, 16, st), "memset");
        launch_rm_mark(L.act(), nq, dense_scratch(L), st);
        ck_launch("rm mark");
        L.premarked = true;
      }
      ph_hash.~Phase();
      new (&ph_hash) Phase(this, l, KL_PHASE_FORWARD);
      float* hout = nullptr;
      if (!last) {
        hout = L.h.as<float>() + (size_t)hrow0 * L.ldN;
        ck(cudaMemsetAsync(hout, 0, (size_t)nq * L.ldN * 4, st), "memset");
      }
      const ActiveSet A = L.act();
      if (L.fm) {
        launch_fm_forward(L.W.p, wdtype, L.ldw, L.d, L.b.as<float>(), L.cfg.activation, in, A, hout, L.ldN,
                          ctx->err.as<int>(), st);
        ck_launch("fm forward");
        if (L.cfg.activation == KL_ACT_SOFTMAX) {
          launch_softmax(A, hout, L.ldN, nullptr, nullptr, nullptr, nq, st);
          ck_launch("softmax");
        }
      } else {
        RmArgs ra = rm_args(l, b, s0, hout);
        const bool softmax = L.cfg.activation == KL_ACT_SOFTMAX;
        const bool fused = last && train && !softmax;
        if (fused && L.premarked) {
          const DenseScratch D = dense_scratch(L);
          ra.lgd_dense = D.LGd;
          ra.slot_of = D.slot_of;
          ra.ldb = D.ldb;
        }
        launch_rm_forward(ra, nq, fused ? RM_FUSED : RM_FWD, st);
        ck_launch("rm forward");
        if (softmax) {
          launch_softmax(A, hout, L.ldN, last && train ? b.label_ptr + s0 : nullptr, b.labels, labprob.as<float>(),
                         nq, st);
          ck_launch("softmax");
          if (last && train) {
            launch_rm_forward(ra, nq, RM_DX, st);
            ck_launch("rm dx");
          }
        }
      }
    }
  }

  // Backward + updates for the examples of the last forward (net.rs:122-146).
  void backward(const kl_batch& b, int s0, int nq, double lr) {
    cudaStream_t st = ctx->stream;
    const int nL = (int)layers.size();
    // input gradient of the output layer
    {
      Phase ph(this, nL - 1, KL_PHASE_BACKWARD);
      Layer& L = *layers[nL - 1];
      launch_reduce_dx(L.dxpart.as<float>(), L.nchunk, L.ldd, L.d, L.cnt.as<int32_t>(), L.dx_in.as<float>(), nq,
                       st);
      ck_launch("reduce dx");
    }
    for (int l = nL - 2; l >= 0; --l) {
      Phase ph(this, l, KL_PHASE_BACKWARD);
      Layer& L = *layers[l];
      const Layer& U = *layers[l + 1];
      float* lgd = nullptr;
      uint32_t* tmask = nullptr;
      if (L.fm) {
        ck(cudaMemsetAsync(L.lgd.p, 0, (size_t)nq * L.ldN * 4, st), "memset");
        ck(cudaMemsetAsync(L.tmask.p, 0, (size_t)ceil_div(L.N, 32) * 4, st), "memset");
        lgd = L.lgd.as<float>();
        tmask = L.tmask.as<uint32_t>();
      }
      launch_local_grads(L.act(), L.cfg.activation, U.dx_in.as<float>(), U.ldd, lgd, L.ldN, tmask, nq, st);
      ck_launch("local grads");
      if (!L.fm) {
        const Layer& P = *layers[l - 1];
        RmArgs ra{};
        ra.W = L.W.p;
        ra.wdtype = wdtype;
        ra.ldw = L.ldw;
        ra.d = L.d;
        ra.bias = L.b.as<float>();
        ra.act = L.cfg.activation;
        ra.X = P.h.as<float>();
        ra.ldx = P.ldN;
        ra.A = L.act();
        ra.dxpart = L.dxpart.as<float>();
        ra.nchunk = L.nchunk;
        ra.err = ctx->err.as<int>();
        launch_rm_forward(ra, nq, RM_DX, st);
        ck_launch("rm dx");
        launch_reduce_dx(L.dxpart.as<float>(), L.nchunk, L.ldd, L.d, L.cnt.as<int32_t>(), L.dx_in.as<float>(), nq,
                         st);
        ck_launch("reduce dx");
      }
    }
    // optimizer updates (every gradient above used the pre-update weights)
    update_layers(b, s0, nq, lr);
  }

  // Optimizer updates of every layer for examples [s0, s0+nq) of the batch.
  // The sparse-input layer's update (an HBM stream over all its feature rows)
  // and the other layers' updates (latency-bound gathers of L2-resident rows)
  // touch disjoint state, so without the phase profiler the first runs on a
  // side stream, forked from and joined back into the context stream (in a
  // captured step graph: two parallel branches).
  cudaStream_t side_stream = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  void ensure_side_stream() {
    if (side_stream) return;
    ck(cudaStreamCreateWithFlags(&side_stream, cudaStreamNonBlocking), "side stream");
    ck(cudaEventCreateWithFlags(&ev_fork, cudaEventDisableTiming), "event");
    ck(cudaEventCreateWithFlags(&ev_join, cudaEventDisableTiming), "event");
  }
  void update_layers(const kl_batch& b, int s0, int nq, double lr) {
    (void)lr;  // the step's optimizer constants are in dopt (upload_opt)
    const int nL = (int)layers.size();
    if (prof || nL < 2) {
      for (int l = nL - 1; l >= 0; --l) update_layer(l, b, s0, nq);
      return;
    }
    ensure_side_stream();
    cudaStream_t st = ctx->stream;
    ck(cudaEventRecord(ev_fork, st), "event");
    ck(cudaStreamWaitEvent(side_stream, ev_fork, 0), "stream wait");
    update_layer(0, b, s0, nq, side_stream);
    ck(cudaEventRecord(ev_join, side_stream), "event");
    for (int l = nL - 1; l >= 1; --l) update_layer(l, b, s0, nq);
    ck(cudaStreamWaitEvent(st, ev_join, 0), "stream wait");
  }
  void update_layer(int l, const kl_batch& b, int s0, int nq, cudaStream_t on = nullptr) {
    cudaStream_t st = on ? on : ctx->stream;
    const OptStep* o = dopt.as<OptStep>();
    SparseIn in{b.rowptr + s0, b.idx, b.val, nq};
    {
      Phase ph(this, l, KL_PHASE_UPDATE);
      Layer& L = *layers[l];
      unsigned long long* stat = L.stats.as<unsigned long long>() + 1;
      if (!L.premarked) ck(cudaMemsetAsync(L.ctr.p, 0, 16, st), "memset");
      SegScratch S{L.hist.as<uint32_t>(), L.cur.as<uint32_t>(), L.touched.as<uint32_t>(), L.ctr.as<uint32_t>(),
                   L.ent_s.as<uint32_t>(), L.ent_v.as<float>(), L.fslot.as<uint32_t>(), L.flong.as<uint32_t>()};
      if (L.fm) {
        launch_fm_update(L.W.p, wdtype, L.ldw, L.d, L.f0, L.nf, L.N, L.b.as<float>(), L.m.as<float>(), L.v.as<float>(),
                         L.mb.as<float>(), L.vb.as<float>(), in, L.lgd.as<float>(), L.ldN, L.tmask.as<uint32_t>(),
                         S, L.gfeat.as<float>(), o, stat, ctx->err.as<int>(), st, &kl_net_s::stream_hook, this);
        ck_launch("fm update");
      } else {
        const Layer& P = *layers[l - 1];
        if (L.dldb > 0) {
          const DenseScratch D = dense_scratch(L);
          launch_rm_update_dense(L.W.p, wdtype, L.ldw, L.d, L.b.as<float>(), L.m.as<float>(), L.v.as<float>(),
                                 L.mb.as<float>(), L.vb.as<float>(), P.h.as<float>(), P.ldN, L.act(), nq, L.N, D,
                                 o, stat, st, L.premarked);
          L.premarked = false;
          launch_count_touched(L.ctr.as<uint32_t>(), stat, st);
        } else {
          launch_rm_update(L.W.p, wdtype, L.ldw, L.d, L.b.as<float>(), L.m.as<float>(), L.v.as<float>(),
                           L.mb.as<float>(), L.vb.as<float>(), P.h.as<float>(), P.ldN, L.act(), nq, L.N, S, o,
                           stat, st);
        }
        ck_launch("rm update");
      }
    }
  }

  // The output layer's selection over all shards for the nq examples of the
  // last probe (Layer::shard_select): count histograms summed over the ranks,
  // the per-example cut, the ranks' numbers of candidates at the cut, and the
  // compaction of this rank's selected candidates into the active set.
  void shard_select_exchange(Layer& L, int nq) {
    cudaStream_t st = ctx->stream;
    const int Lt = L.cfg.lsh.num_tables;
    int32_t* hist = sel_hist.as<int32_t>();
    launch_sel_hist(L.ccnt.as<uint32_t>(), L.ccn.as<int32_t>(), L.cstride, Lt, hist, nq, st);
    ck_launch("selection histogram");
    nccl_ck(ncclAllReduce(hist, hist, (size_t)nq * (Lt + 1), ncclInt32, ncclSum, comm, st),
            "all-reduce selection histograms");
    int32_t* sc = sel_cut.as<int32_t>();  // cut, need, global size, local count at the cut: [4][nq]
    launch_sel_cut(hist, Lt, L.cfg.sampling, L.cfg.top_k, L.cfg.sampling_threshold, L.ccnt.as<uint32_t>(),
                   L.ccn.as<int32_t>(), L.cstride, sc, sc + nq, sc + 2 * nq, sc + 3 * nq, nq, st);
    ck_launch("selection cut");
    int32_t* eq_all = sel_eq_all.as<int32_t>();
    nccl_ck(ncclAllGather(sc + 3 * nq, eq_all, (size_t)nq, ncclInt32, comm, st), "all-gather cut counts");
    launch_sel_apply(L.cids.as<uint32_t>(), L.ccnt.as<uint32_t>(), L.ccn.as<int32_t>(), L.cstride, sc, sc + nq,
                     sc + 2 * nq, eq_all, rank, nq, L.N, L.act(), ctx->err.as<int>(),
                     L.stats.as<unsigned long long>(), st);
    ck_launch("selection apply");
  }

  // One batched train step of a neuron-sharded network (nranks > 1).  `lb`
  // holds this rank's B examples; the global batch is the P*B examples of all
  // ranks in rank order.  Collectives, all on the context stream:
  //  (1) all-gather of the packed batches (inputs and labels);
  //  (2) all-gather of the hidden activations (data-parallel hidden forward);
  //  (3) all-reduce of each example's number of selected candidates (global
  //      empty-selection fallback);
  //  (4) one group: all-reduce of the label probabilities (the loss) and
  //      reduce-scatter of the output layer's input gradient;
  //  (5) one group: all-gather of the hidden local gradients and touched masks.
  // The replicated hidden layer then applies the same update on every rank.
  // Steps (1)-(3) of a sharded step for `lb` (this rank's examples): the
  // global batch, the hidden layer's forward and the output layer's forward
  // over the global batch on this rank's slice (with the input-gradient
  // partials when `train`).  Returns the global batch.
  kl_batch sharded_forward(const kl_batch& lb, bool train) {
    shard_pack(lb);
    return sharded_forward_body(train);
  }
  // Every collective of a sharded step is sized by the configured per-rank
  // batch, never by this rank's data, so that no rank can leave the collective
  // sequence on its own.  A batch that cannot be exchanged (another example
  // count, or more nnz / labels than the fixed exchange capacity) is sent as an
  // empty batch with a fault word: every rank then raises the fault at its next
  // synchronising call and applies the step with a zero learning rate.
  // shard_pack copies this rank's batch into the exchange buffer (its only
  // step that depends on the caller's arrays and sizes); everything after it
  // reads fixed buffers, so it can be captured in a CUDA graph.
  static bool shard_batch_ok(const kl_batch& lb, int B, int nnz_cap_, int lab_cap_) {
    return lb.batch == B && lb.nnz <= nnz_cap_ && !(lb.label_ptr && lb.nlabels > lab_cap_);
  }
  void shard_pack(const kl_batch& lb) {
    const int B = rank_batch;
    uint32_t fault = 0;
    if (lb.batch != B) fault = DERR_BOUNDS;
    else if (!shard_batch_ok(lb, B, nnz_cap, lab_cap)) fault = DERR_CAPACITY;
    launch_shard_pack(dsend.as<uint32_t>(), shl, lb, B, fault, ctx->stream);
    ck_launch("shard pack");
  }
  kl_batch sharded_forward_body(bool train) {
    cudaStream_t st = ctx->stream;
    const int P = nranks, B = rank_batch, PB = P * B;
    Layer& H = *layers[0];
    Layer& O = *layers[1];
    // (1) the global batch
    nccl_ck(ncclAllGather(dsend.p, drecv.p, (size_t)shl.words, ncclUint32, comm, st), "all-gather batches");
    launch_shard_unpack(drecv.as<uint32_t>(), shl, P, B, g_rowptr.as<int32_t>(), g_idx.as<uint32_t>(),
                        g_val.as<float>(), g_lptr.as<int32_t>(), g_labels.as<uint32_t>(), ctx->err.as<int>(),
                        dopt.as<OptStep>(), st);
    ck_launch("shard unpack");
    kl_batch gb{};
    gb.batch = PB;
    gb.rowptr = g_rowptr.as<int32_t>();
    gb.idx = g_idx.as<uint32_t>();
    gb.val = g_val.as<float>();
    gb.label_ptr = g_lptr.as<int32_t>();
    gb.labels = g_labels.as<uint32_t>();
    gb.nnz = P * nnz_cap;
    gb.nlabels = P * lab_cap;
    ck(cudaMemsetAsync(loss_acc.p, 0, 4, st), "memset");
    ck(cudaMemsetAsync(labprob.p, 0, (size_t)P * lab_cap * 4, st), "memset");
    // (2) hidden forward of this rank's examples, then every rank's activations
    forward_layer(0, gb, rank * B, B, train, rank * B);
    {
      float* h = H.h.as<float>();
      nccl_ck(ncclAllGather(h + (size_t)rank * B * H.ldN, h, (size_t)B * H.ldN, ncclFloat32, comm, st),
              "all-gather hidden activations");
    }
    // output forward over the global batch.  (3) runs on the comm stream from
    // the probe on, beside the forward; an example that no rank selected a
    // candidate for then takes every local neuron (the fallback) and a second
    // forward pass computes only those examples.
    forward_layer(1, gb, 0, PB, train, 0, [&](Layer& L) {
      if (L.shard_select) {  // the selection itself is global (and decides the fallback)
        shard_select_exchange(L, PB);
        return;
      }
      ck(cudaEventRecord(ev_cnt, st), "event");
      ck(cudaStreamWaitEvent(comm_stream, ev_cnt, 0), "stream wait");
      nccl_ck(ncclAllReduce(L.cnt.p, gcnt.p, (size_t)PB, ncclInt32, ncclSum, comm, comm_stream),
              "all-reduce selections");
      ck(cudaEventRecord(ev_cnt_done, comm_stream), "event");
    });
    if (!O.shard_select) {
      Phase ph(this, 1, KL_PHASE_FORWARD);
      ck(cudaStreamWaitEvent(st, ev_cnt_done, 0), "stream wait");
      launch_shard_fallback(O.act(), gcnt.as<int32_t>(), O.N, PB, ctx->err.as<int>(), st);
      ck_launch("shard fallback");
      RmArgs ra = rm_args(1, gb, 0, nullptr);
      ra.only_empty = gcnt.as<int32_t>();
      if (train && O.premarked) {
        const DenseScratch D = dense_scratch(O);
        launch_rm_mark(O.act(), PB, D, st, gcnt.as<int32_t>());
        ck_launch("rm mark (fallback examples)");
        ra.lgd_dense = D.LGd;
        ra.slot_of = D.slot_of;
        ra.ldb = D.ldb;
      }
      launch_rm_forward(ra, PB, train ? RM_FUSED : RM_FWD, st);
      ck_launch("rm forward (fallback examples)");
    }
    return gb;
  }

  void train_sharded(const kl_batch& lb, double lr) {
    (void)lr;  // the step's optimizer constants are in dopt (upload_opt)
    shard_pack(lb);
    if (!graph_disabled && !prof && shard_batch_ok(lb, rank_batch, nnz_cap, lab_cap)) {
      sharded_graph_step();
      return;
    }
    train_sharded_body();
  }
  // The sharded step after the pack as one CUDA graph (NCCL collectives
  // included), replayed per step: the step issues ~70 launches and collectives,
  // which cost more host time than the GPU spends on them.  First use runs
  // eagerly, the second captures.  A batch that the exchange must flag takes
  // the eager body: its collectives are the same, so the ranks stay matched.
  cudaGraphExec_t sh_gexec = nullptr;
  bool sh_warm = false;
  unsigned long long sh_graph_kernels = 0;
  void sharded_graph_step() {
    cudaStream_t st = ctx->stream;
    if (!sh_warm) {
      sh_warm = true;
      train_sharded_body();
      return;
    }
    if (!sh_gexec) {
      if (!cap_stream) ck(cudaStreamCreateWithFlags(&cap_stream, cudaStreamNonBlocking), "capture stream");
      ensure_side_stream();
      // the capture stream starts after this call's pack
      ck(cudaEventRecord(ev_fork, st), "event");
      ck(cudaStreamWaitEvent(cap_stream, ev_fork, 0), "stream wait");
      cudaGraph_t g = nullptr;
      ctx->stream = cap_stream;
      bool ok = cudaStreamBeginCapture(cap_stream, cudaStreamCaptureModeRelaxed) == cudaSuccess;
      const unsigned long long n0 = g_launches.load();
      if (ok) {
        try {
          train_sharded_body();
        } catch (...) {
          ok = false;
        }
        ok = cudaStreamEndCapture(cap_stream, &g) == cudaSuccess && ok && g;
      }
      ctx->stream = st;
      if (ok) ok = cudaGraphInstantiate(&sh_gexec, g, 0) == cudaSuccess;
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
      if (!ok) {
        sh_gexec = nullptr;
        graph_disabled = true;  // eager from now on (same collectives)
        train_sharded_body();
        return;
      }
      sh_graph_kernels = g_launches.load() - n0;
      g_launches.fetch_sub(sh_graph_kernels);  // counted again per replay below
    }
    ck(cudaGraphLaunch(sh_gexec, st), "graph launch");
    count_launch((unsigned)sh_graph_kernels);
  }
  void train_sharded_body() {
    cudaStream_t st = ctx->stream;
    const int P = nranks, B = rank_batch, PB = P * B;
    Layer& H = *layers[0];
    Layer& O = *layers[1];
    const kl_batch gb = sharded_forward_body(true);
    // The output layer's update needs only its forward (active sets, local
    // gradients) and the hidden activations: without the phase profiler it
    // runs on the side stream from here, beside the collectives and the hidden
    // layer's backward and update below.
    const bool fork = !prof;
    if (fork) {
      ensure_side_stream();
      ck(cudaEventRecord(ev_fork, st), "event");
      ck(cudaStreamWaitEvent(side_stream, ev_fork, 0), "stream wait");
      update_layer(1, gb, 0, PB, side_stream);
      ck(cudaEventRecord(ev_join, side_stream), "event");
    }
    // (4) loss probabilities and the output layer's input gradient
    {
      Phase ph(this, 1, KL_PHASE_BACKWARD);
      launch_reduce_dx(O.dxpart.as<float>(), O.nchunk, O.ldd, O.d, O.cnt.as<int32_t>(), O.dx_in.as<float>(), PB, st);
      ck_launch("reduce dx");
      float* dx = O.dx_in.as<float>();
      nccl_ck(ncclGroupStart(), "group");
      nccl_ck(ncclAllReduce(labprob.p, labprob.p, (size_t)P * lab_cap, ncclFloat32, ncclSum, comm, st),
              "all-reduce label probabilities");
      nccl_ck(ncclReduceScatter(dx, dx + (size_t)rank * B * O.ldd, (size_t)B * O.ldd, ncclFloat32, ncclSum, comm, st),
              "reduce-scatter input gradient");
      nccl_ck(ncclGroupEnd(), "group");
    }
    launch_loss(gb.label_ptr, labprob.as<float>(), PB, loss_acc.as<float>(), st);
    ck_launch("loss");
    // hidden local gradients of this rank's examples; (5) everyone's
    {
      Phase ph(this, 0, KL_PHASE_BACKWARD);
      const int nw = (int)ceil_div(H.N, 32);
      ck(cudaMemsetAsync(H.lgd.p, 0, (size_t)PB * H.ldN * 4, st), "memset");
      ck(cudaMemsetAsync(H.tmask.p, 0, (size_t)nw * 4, st), "memset");
      float* lgd = H.lgd.as<float>();
      launch_local_grads(H.act(), H.cfg.activation, O.dx_in.as<float>() + (size_t)rank * B * O.ldd, O.ldd,
                         lgd + (size_t)rank * B * H.ldN, H.ldN, H.tmask.as<uint32_t>(), B, st);
      ck_launch("local grads");
      nccl_ck(ncclGroupStart(), "group");
      nccl_ck(ncclAllGather(lgd + (size_t)rank * B * H.ldN, lgd, (size_t)B * H.ldN, ncclFloat32, comm, st),
              "all-gather hidden gradients");
      nccl_ck(ncclAllGather(H.tmask.p, tmask_all.p, (size_t)nw, ncclUint32, comm, st), "all-gather touched masks");
      nccl_ck(ncclGroupEnd(), "group");
      launch_shard_or_masks(H.tmask.as<uint32_t>(), tmask_all.as<uint32_t>(), P, nw, st);
      ck_launch("or masks");
    }
    // (6) The hidden layer's update, over this rank's feature rows only; then
    // an in-place all-gather of the updated rows on the comm stream.  The next
    // step's kernels wait for it and for the output layer's update.
    update_layer(0, gb, 0, PB);
    {
      const int R = (int)ceil_div(H.d, P);
      ck(cudaEventRecord(ev_hidden, st), "event");
      ck(cudaStreamWaitEvent(comm_stream, ev_hidden, 0), "stream wait");
      const size_t esz = wdtype == KL_DTYPE_BF16 ? 2 : 4;
      char* w = static_cast<char*>(H.W.p);
      nccl_ck(ncclAllGather(w + (size_t)rank * R * H.ldw * esz, w, (size_t)R * H.ldw,
                            wdtype == KL_DTYPE_BF16 ? ncclBfloat16 : ncclFloat32, comm, comm_stream),
              "all-gather hidden weights");
      ck(cudaEventRecord(ev_gather, comm_stream), "event");
    }
    if (fork) ck(cudaStreamWaitEvent(st, ev_join, 0), "stream wait");
    else update_layer(1, gb, 0, PB);
    ck(cudaStreamWaitEvent(st, ev_gather, 0), "stream wait");
  }

  // ---- CUDA graph of the batched single-GPU train step ------------------
  // The step's ~30 kernel launches and memsets are captured once per batch
  // size and replayed with one cudaGraphLaunch.  The graph reads the batch
  // from fixed buffers (the caller's arrays are copied in first) and the
  // optimizer constants from dopt; the rebuild check stays on the host.
  bool graph_disabled = false;
  bool graph_warm = false;
  int graph_B = -1;
  cudaGraphExec_t gexec = nullptr;
  cudaStream_t cap_stream = nullptr;
  int g_nnz_cap = 0, g_lab_cap = 0;
  unsigned long long graph_kernels = 0;  // kernels in the captured graph (launch accounting)
  DBuf gi_rowptr, gi_idx, gi_val, gi_lptr, gi_labels, loss_out;

  bool graph_usable(const kl_batch& b) const {
    return !graph_disabled && !prof && nranks == 1 && b.batch > 0 && b.nnz <= max_batch * KL_GRAPH_NNZ_PER_EXAMPLE &&
           b.nlabels <= max_batch * KL_GRAPH_LABELS_PER_EXAMPLE;
  }
  void batched_body(const kl_batch& ib) {
    cudaStream_t st = ctx->stream;
    ck(cudaMemsetAsync(loss_acc.p, 0, 4, st), "memset");
    ck(cudaMemsetAsync(labprob.p, 0, (size_t)g_lab_cap * 4, st), "memset");
    forward(ib, 0, ib.batch, true);
    launch_loss(ib.label_ptr, labprob.as<float>(), ib.batch, loss_acc.as<float>(), st);
    ck_launch("loss");
    backward(ib, 0, ib.batch, 0.0);
    launch_loss_final(loss_acc.as<float>(), ib.batch, loss_out.as<float>(), loss_acc.as<float>(), st);
    ck_launch("loss final");
  }
  void graph_step(const kl_batch& b, float* loss) {
    cudaStream_t st = ctx->stream;
    const int B = b.batch;
    if (g_nnz_cap == 0) {
      g_nnz_cap = max_batch * KL_GRAPH_NNZ_PER_EXAMPLE;
      g_lab_cap = max_batch * KL_GRAPH_LABELS_PER_EXAMPLE;
      gi_rowptr.alloc((size_t)(max_batch + 1) * 4);
      gi_lptr.alloc((size_t)(max_batch + 1) * 4);
      gi_idx.alloc((size_t)g_nnz_cap * 4);
      gi_val.alloc((size_t)g_nnz_cap * 4);
      gi_labels.alloc((size_t)g_lab_cap * 4);
      loss_out.alloc(4);
      kl_batch cap_b{};
      cap_b.batch = max_batch;
      cap_b.nnz = g_nnz_cap;
      cap_b.nlabels = g_lab_cap;
      ensure_batch_buffers(cap_b);
      ck(cudaStreamCreateWithFlags(&cap_stream, cudaStreamNonBlocking), "capture stream");
    }
    ck(cudaMemcpyAsync(gi_rowptr.p, b.rowptr, (size_t)(B + 1) * 4, cudaMemcpyDeviceToDevice, st), "batch copy");
    ck(cudaMemcpyAsync(gi_lptr.p, b.label_ptr, (size_t)(B + 1) * 4, cudaMemcpyDeviceToDevice, st), "batch copy");
    if (b.nnz > 0) {
      ck(cudaMemcpyAsync(gi_idx.p, b.idx, (size_t)b.nnz * 4, cudaMemcpyDeviceToDevice, st), "batch copy");
      ck(cudaMemcpyAsync(gi_val.p, b.val, (size_t)b.nnz * 4, cudaMemcpyDeviceToDevice, st), "batch copy");
    }
    if (b.nlabels > 0)
      ck(cudaMemcpyAsync(gi_labels.p, b.labels, (size_t)b.nlabels * 4, cudaMemcpyDeviceToDevice, st), "batch copy");
    kl_batch ib{};
    ib.batch = B;
    ib.rowptr = gi_rowptr.as<int32_t>();
    ib.idx = gi_idx.as<uint32_t>();
    ib.val = gi_val.as<float>();
    ib.label_ptr = gi_lptr.as<int32_t>();
    ib.labels = gi_labels.as<uint32_t>();
    ib.nnz = g_nnz_cap;
    ib.nlabels = g_lab_cap;
    if (!graph_warm || (gexec && graph_B != B)) {
      // first use (or a new batch size): run eagerly; capture on the next call
      if (gexec) {
        cudaGraphExecDestroy(gexec);
        gexec = nullptr;
      }
      graph_warm = true;
      batched_body(ib);
    } else {
      if (!gexec) {
        cudaGraph_t g = nullptr;
        ctx->stream = cap_stream;
        bool ok = cudaStreamBeginCapture(cap_stream, cudaStreamCaptureModeRelaxed) == cudaSuccess;
        const unsigned long long n0 = g_launches.load();
        if (ok) {
          try {
            batched_body(ib);
          } catch (...) {
            ok = false;
          }
          ok = cudaStreamEndCapture(cap_stream, &g) == cudaSuccess && ok && g;
        }
        ctx->stream = st;
        if (ok) ok = cudaGraphInstantiate(&gexec, g, 0) == cudaSuccess;
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        if (!ok) {
          gexec = nullptr;
          graph_disabled = true;  // stay eager from now on
          batched_body(ib);
          if (loss) ck(cudaMemcpyAsync(loss, loss_out.p, 4, cudaMemcpyDeviceToDevice, st), "loss copy");
          return;
        }
        graph_B = B;
        graph_kernels = g_launches.load() - n0;
        g_launches.fetch_sub(graph_kernels);  // counted again per replay below
      }
      ck(cudaGraphLaunch(gexec, st), "graph launch");
      count_launch((unsigned)graph_kernels);
    }
    if (loss) ck(cudaMemcpyAsync(loss, loss_out.p, 4, cudaMemcpyDeviceToDevice, st), "loss copy");
  }

  // Per-batch buffers grow geometrically (x1.5) so that a stream of batches
  // with varying nnz / label counts reallocates O(log) times, not per batch.
  void ensure_batch_buffers(const kl_batch& b) {
    if ((size_t)b.nlabels > labprob_cap) {
      const size_t cap = std::max<size_t>((size_t)b.nlabels, labprob_cap * 3 / 2);
      labprob.alloc(std::max<size_t>(cap, 1) * 4);
      labprob_cap = cap;
    }
    Layer& L0 = *layers[0];
    if ((size_t)b.nnz > L0.ent_cap) {
      const size_t cap = std::max<size_t>((size_t)b.nnz, L0.ent_cap * 3 / 2);
      L0.ent_s.alloc(std::max<size_t>(cap, 1) * 4);
      L0.ent_v.alloc(std::max<size_t>(cap, 1) * 4);
      L0.gfeat.alloc((size_t)std::min<int64_t>(std::max<int64_t>((int64_t)cap, 1), L0.d) * L0.ldN * 4);
      L0.ent_cap = cap;
    }
  }
};

namespace {

void validate_batch(const kl_net_s* net, const kl_batch* b) {
  require(b != nullptr, "batch is NULL");
  require(b->batch >= 0, "batch size must be >= 0");
  require(b->batch <= net->max_batch, "batch larger than the network's max_batch");
  require(b->nnz >= 0 && b->nlabels >= 0, "batch nnz / nlabels must be >= 0");
  if (b->batch > 0) require(b->rowptr && b->label_ptr, "batch rowptr / label_ptr required");
  if (b->nnz > 0) require(b->idx && b->val, "batch idx / val required");
  if (b->nlabels > 0) require(b->labels != nullptr, "batch labels required");
}

// `id_base`: global id of this layer's first neuron (the rank's slice of a
// sharded output layer; 0 otherwise).  Explicit init rows are the slice's own.
void build_layer(kl_net_s* net, int l, const kl_layer_config& c, const kl_layer_init* init,
                 uint32_t id_base = 0) {
  kl_ctx_t ctx = net->ctx;
  cudaStream_t st = ctx->stream;
  auto Lp = std::make_unique<Layer>();
  Layer& L = *Lp;
  L.cfg = c;
  L.d = c.input_dim;
  L.N = c.num_neurons;
  require(L.d >= 1 && L.N >= 1, "layer: input_dim and num_neurons must be >= 1");
  require(c.activation >= KL_ACT_RELU && c.activation <= KL_ACT_IDENTITY, "layer: unknown activation");
  require(c.sampling >= KL_SAMPLING_VANILLA && c.sampling <= KL_SAMPLING_THRESHOLD, "layer: unknown sampling");
  L.fm = (l == 0);
  if (L.fm) support(L.N <= 1024, "layer 0 (sparse input) supports at most 1024 neurons");
  else support(L.d <= 8192, "hidden/output layers support input_dim <= 8192");
  L.ldw = L.fm ? pitch_of(L.N) : pitch_of(L.d);
  L.ldN = pitch_of(L.N);
  L.ldd = pitch_of(L.d);
  L.id_bits = bits_for((uint64_t)L.N);
  const kl_lsh_config& lc = c.lsh;
  const int window = std::min(8, L.d);  // index.rs:325-330
  // hash family: explicit parameters or seeded (seed + 1_000_000, layer.rs:40)
  std::shared_ptr<HashImpl> H;
  const uint64_t lseed = net->cfg.seed + (uint64_t)l * 100000ULL;
  bool explicit_hash = init && (init->hash.planes || init->hash.windows || init->hash.perms || init->hash.srp_rowptr);
  if (explicit_hash) {
    H = make_hash(ctx, lc.hash_function, L.d, lc.num_hashes, lc.num_tables, window, &init->hash);
  } else {
    SeededParams sp;
    seeded_params(lc.hash_function, L.d, lc.num_hashes, lc.num_tables, window, 1.0f / 3.0f, lseed + 1000000ULL, sp);
    H = make_hash(ctx, lc.hash_function, L.d, lc.num_hashes, lc.num_tables, window, &sp.p);
  }
  L.index = make_index(ctx, H, lc.bucket_type, lc.bucket_capacity);
  // active capacity per example
  int64_t cap = std::min<int64_t>((int64_t)L.N, (int64_t)lc.num_tables * lc.bucket_capacity);
  if (c.sampling == KL_SAMPLING_TOPK) cap = std::min<int64_t>(cap, std::max(c.top_k, 0));
  if (L.N <= 8192) cap = std::max<int64_t>(cap, L.N);  // room for the all-neurons fallback
  L.stride = (int)std::max<int64_t>(cap, 1);
  if (L.fm) support(L.stride <= 1024, "layer 0 active capacity exceeds 1024");
  L.nchunk = (int)ceil_div(L.stride, RM_RPB);
  // parameters
  const size_t wsz = net->wdtype == KL_DTYPE_BF16 ? 2 : 4;
  const size_t nrows_store = L.fm ? (size_t)L.d : (size_t)L.N;
  const size_t welems = nrows_store * L.ldw;
  // A sharded network's hidden layer updates feature rows in P equal slices of
  // R = ceil(d / P) rows and all-gathers them in place: W holds P * R rows.
  L.f0 = 0;
  L.nf = L.d;
  size_t wrows = nrows_store;
  if (L.fm && net->nranks > 1) {
    const int R = (int)ceil_div(L.d, net->nranks);
    L.f0 = std::min(L.d, net->rank * R);
    L.nf = std::min(L.d, L.f0 + R) - L.f0;
    wrows = (size_t)R * net->nranks;
  }
  L.W.alloc(wrows * L.ldw * wsz);
  ck(cudaMemsetAsync(L.W.p, 0, wrows * L.ldw * wsz, st), "memset");
  L.m.alloc(welems * 4);
  L.v.alloc(welems * 4);
  L.b.alloc((size_t)L.N * 4);
  L.mb.alloc((size_t)L.N * 4);
  L.vb.alloc((size_t)L.N * 4);
  ck(cudaMemsetAsync(L.m.p, 0, welems * 4, st), "memset");
  ck(cudaMemsetAsync(L.v.p, 0, welems * 4, st), "memset");
  ck(cudaMemsetAsync(L.mb.p, 0, (size_t)L.N * 4, st), "memset");
  ck(cudaMemsetAsync(L.vb.p, 0, (size_t)L.N * 4, st), "memset");
  {
    // initial rows: explicit, or N(0, sqrt(2/d)) from this library's generator (neuron.rs:23-43)
    std::vector<float> rows;
    const float* src = init ? init->weights : nullptr;
    if (!src) {
      rows.resize((size_t)L.N * L.d);
      const double sd = std::sqrt(2.0 / (double)L.d);
      for (int n = 0; n < L.N; ++n) {
        SplitMix rng{lseed + (uint64_t)id_base + (uint64_t)n};
        for (int i = 0; i < L.d; ++i) rows[(size_t)n * L.d + i] = (float)(rng.normal() * sd);
      }
      src = rows.data();
    }
    DBuf tmp;
    // upload in row slabs to bound the temporary
    const int64_t slab = std::max<int64_t>(1, (int64_t)(64u << 20) / (4 * (int64_t)L.d));
    tmp.alloc((size_t)std::min<int64_t>(slab, L.N) * L.d * 4);
    for (int64_t r0 = 0; r0 < L.N; r0 += slab) {
      const int64_t nr = std::min<int64_t>(slab, L.N - r0);
      ck(cudaMemcpyAsync(tmp.p, src + (size_t)r0 * L.d, (size_t)nr * L.d * 4, cudaMemcpyHostToDevice, st), "upload");
      void* dst = L.fm ? (void*)((char*)L.W.p + (size_t)r0 * wsz) : (void*)((char*)L.W.p + (size_t)r0 * L.ldw * wsz);
      launch_f32_to_w(tmp.as<float>(), nr, L.d, L.d, dst, net->wdtype, L.ldw, L.fm, st);
      ck_launch("weights upload");
      ck(cudaStreamSynchronize(st), "sync");
    }
    std::vector<float> bias((size_t)L.N, 0.0f);
    if (init && init->bias) std::memcpy(bias.data(), init->bias, (size_t)L.N * 4);
    ck(cudaMemcpyAsync(L.b.p, bias.data(), (size_t)L.N * 4, cudaMemcpyHostToDevice, st), "upload");
    ck(cudaStreamSynchronize(st), "sync");
  }
  // per-step buffers
  const int B = net->max_batch;
  L.bkt.alloc((size_t)lc.num_tables * B * 2);
  L.ids.alloc((size_t)B * L.stride * 4);
  L.cnt.alloc((size_t)B * 4);
  L.pre.alloc((size_t)B * L.stride * 4);
  L.post.alloc((size_t)B * L.stride * 4);
  L.lg.alloc((size_t)B * L.stride * 4);
  L.h.alloc((size_t)B * L.ldN * 4);
  if (!L.fm) {
    L.dx_in.alloc((size_t)B * L.ldd * 4);
    L.dxpart.alloc((size_t)B * L.nchunk * L.ldd * 4);
  } else {
    L.lgd.alloc((size_t)B * L.ldN * 4);
    L.tmask.alloc((size_t)ceil_div(L.N, 32) * 4);
  }
  const size_t rows = L.fm ? (size_t)L.d : (size_t)L.N;
  L.hist.alloc(rows * 4);
  L.cur.alloc(rows * 4);
  L.touched.alloc(rows * 4);
  L.ctr.alloc(16);
  ck(cudaMemsetAsync(L.hist.p, 0, rows * 4, st), "memset");
  if (L.fm) {
    L.fslot.alloc((round_up(rows, 4) + 4) * 4);  // read in 16-byte units by the streaming update
    L.flong.alloc(rows * 4);
    ck(cudaMemsetAsync(L.fslot.p, 0, (round_up(rows, 4) + 4) * 4, st), "memset");
  }
  if (!L.fm) {
    // dense-collision update scratch when its gradient matrix fits the budget
    const int64_t drows = std::min<int64_t>((int64_t)L.N, (int64_t)B * L.stride);
    // slot-major [slots][ldb] gradient matrix
    const int64_t dslots = round_up(drows, 32);
    const int64_t ldb = round_up(std::max(B, 1), 32);
    if (rm_dense_fits(dslots, (int)ldb, net->cfg.dense_update_max_bytes)) {
      L.dldb = ldb;
      L.dmark.alloc((size_t)L.N * 4);
      ck(cudaMemsetAsync(L.dmark.p, 0, (size_t)L.N * 4, st), "memset");
      L.dtouched.alloc((size_t)drows * 4);
      L.dslot.alloc((size_t)L.N * 4);
      L.dlg.alloc((size_t)dslots * ldb * 4);
      ck(cudaMemsetAsync(L.dlg.p, 0, (size_t)dslots * ldb * 4, st), "memset");
    }
    L.ent_s.alloc((size_t)B * L.stride * 4);
    L.ent_v.alloc((size_t)B * L.stride * 4);
    L.ent_cap = (size_t)B * L.stride;
  }
  L.stats.alloc(3 * 8);
  ck(cudaMemsetAsync(L.stats.p, 0, 24, st), "memset");
  L.id_base = id_base;
  net->layers.push_back(std::move(Lp));
}

}  // namespace

void nccl_ck(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) raise(KL_ENCCL, std::string(what) + ": " + ncclGetErrorString(r));
}

namespace {
constexpr int KL_SHARD_NNZ_PER_EXAMPLE = KL_SHARD_NNZ_PER_EXAMPLE_H;
constexpr int KL_SHARD_LABELS_PER_EXAMPLE = KL_SHARD_LABELS_PER_EXAMPLE_H;

// Shared body of kl_net_create (nranks == 1, no communicator) and
// kl_net_create_sharded.
kl_net_s* create_net(kl_ctx_t ctx, const kl_net_config* cfg, const kl_layer_init* init, const void* unique_id,
                     int rank, int nranks) {
  require(cfg->num_layers >= 1 && cfg->layers, "net: at least one layer required");
  support(cfg->num_layers >= 2, "net: single-layer networks are not supported (layer 0 is the sparse-input layer)");
  require(cfg->optimizer == KL_OPT_SGD || cfg->optimizer == KL_OPT_ADAM, "net: unknown optimizer");
  require(cfg->weight_dtype == KL_DTYPE_F32 || cfg->weight_dtype == KL_DTYPE_BF16, "net: unknown weight dtype");
  require(cfg->max_batch >= 1 && cfg->max_batch <= 4096, "net: max_batch must be in [1, 4096]");
  for (int l = 1; l < cfg->num_layers; ++l)
    require(cfg->layers[l].input_dim == cfg->layers[l - 1].num_neurons,
            "net: layer input_dim must equal the previous layer's num_neurons");
  require(nranks >= 1 && rank >= 0 && rank < nranks, "sharded net: rank must be in [0, nranks)");
  const int nl = cfg->num_layers;
  if (nranks > 1) {
    const kl_layer_config& o = cfg->layers[nl - 1];
    support(nl == 2, "sharded net: exactly two layers (sparse-input hidden layer + sharded output layer)");
    support(o.activation != KL_ACT_SOFTMAX, "sharded net: softmax output layers are not supported");
    support(o.num_neurons >= nranks, "sharded net: fewer output neurons than ranks");
    support(o.lsh.num_tables <= 1024, "sharded net: at most 1024 output tables");
    require(cfg->max_batch <= 4096 / nranks, "sharded net: nranks * max_batch must be <= 4096");
  }
  std::unique_ptr<kl_net_s> net(new kl_net_s());
  net->ctx = ctx;
  net->cfg = *cfg;
  net->layer_cfgs.assign(cfg->layers, cfg->layers + nl);
  net->cfg.layers = net->layer_cfgs.data();
  net->wdtype = cfg->weight_dtype;
  net->rank = rank;
  net->nranks = nranks;
  if (const char* gv = std::getenv("KL_GRAPH"))
    if (!std::strcmp(gv, "0")) net->graph_disabled = true;
  net->rank_batch = cfg->max_batch;
  net->max_batch = cfg->max_batch * nranks;  // per-step buffers hold the global batch
  for (int l = 0; l < nl; ++l) {
    const kl_layer_init* li = init ? &init[l] : nullptr;
    if (nranks > 1 && l == nl - 1) {
      // this rank's contiguous slice [lo, hi) of the output neurons, buckets of cap / P ids
      kl_layer_config c = cfg->layers[l];
      const uint32_t lo = (uint32_t)(((uint64_t)rank * c.num_neurons) / nranks);
      const uint32_t hi = (uint32_t)(((uint64_t)(rank + 1) * c.num_neurons) / nranks);
      c.num_neurons = (int32_t)(hi - lo);
      c.lsh.bucket_capacity = std::max(1, c.lsh.bucket_capacity / nranks);
      kl_layer_init sl{};
      if (li) {
        sl = *li;
        if (li->weights) sl.weights = li->weights + (size_t)lo * c.input_dim;
        if (li->bias) sl.bias = li->bias + lo;
      }
      build_layer(net.get(), l, c, li ? &sl : nullptr, lo);
    } else {
      build_layer(net.get(), l, cfg->layers[l], li);
    }
  }
  // Layer::new inserts every neuron in id order (layer.rs:42-44)
  for (auto& L : net->layers) {
    net->rebuild_layer(*L);
    L->rebuilds = 0;
  }
  const kl_lsh_config& l0 = cfg->layers[0].lsh;
  net->sched.base = (uint64_t)std::max(0, l0.rebuild_interval_base);
  net->sched.decay = l0.rebuild_decay;
  net->sched.next = net->sched.base;
  net->loss_acc.alloc(4);
  net->labprob.alloc(4);
  net->dopt.alloc(sizeof(OptStep));
  if (nranks > 1) {
    const int B = net->rank_batch, P = nranks;
    net->nnz_cap = B * KL_SHARD_NNZ_PER_EXAMPLE;
    net->lab_cap = B * KL_SHARD_LABELS_PER_EXAMPLE;
    net->shl = shard_layout(B, net->nnz_cap, net->lab_cap);
    net->dsend.alloc((size_t)net->shl.words * 4);
    net->drecv.alloc((size_t)net->shl.words * 4 * P);
    net->g_rowptr.alloc((size_t)(P * B + 1) * 4);
    net->g_lptr.alloc((size_t)(P * B + 1) * 4);
    net->g_idx.alloc((size_t)P * net->nnz_cap * 4);
    net->g_val.alloc((size_t)P * net->nnz_cap * 4);
    net->g_labels.alloc((size_t)P * net->lab_cap * 4);
    net->gcnt.alloc((size_t)P * B * 4);
    {
      Layer& O = *net->layers[nl - 1];
      const kl_layer_config& oc = cfg->layers[nl - 1];
      const int64_t Mloc = (int64_t)oc.lsh.num_tables * std::max(1, oc.lsh.bucket_capacity / P);
      O.shard_select = oc.sampling == KL_SAMPLING_THRESHOLD ||
                       (oc.sampling == KL_SAMPLING_TOPK && (int64_t)oc.top_k < Mloc * P);
      if (O.shard_select) {
        const int PBn = P * B;
        O.cstride = (int)Mloc;
        O.cids.alloc((size_t)PBn * Mloc * 4);
        O.ccnt.alloc((size_t)PBn * Mloc * 4);
        O.ccn.alloc((size_t)PBn * 4);
        net->sel_hist.alloc((size_t)PBn * (oc.lsh.num_tables + 1) * 4);
        net->sel_cut.alloc((size_t)4 * PBn * 4);
        net->sel_eq_all.alloc((size_t)P * PBn * 4);
      }
    }
    net->tmask_all.alloc((size_t)P * ceil_div(net->layers[0]->N, 32) * 4);
    kl_batch cap_b{};
    cap_b.batch = P * B;
    cap_b.nnz = P * net->nnz_cap;
    cap_b.nlabels = P * net->lab_cap;
    net->ensure_batch_buffers(cap_b);
    // the collectives that overlap compute run at the highest stream priority, so
    // their kernels take SMs ahead of the compute kernels' waiting blocks
    int prio_lo = 0, prio_hi = 0;
    ck(cudaDeviceGetStreamPriorityRange(&prio_lo, &prio_hi), "stream priorities");
    ck(cudaStreamCreateWithPriority(&net->comm_stream, cudaStreamNonBlocking, prio_hi), "comm stream");
    ck(cudaEventCreateWithFlags(&net->ev_hidden, cudaEventDisableTiming), "event");
    ck(cudaEventCreateWithFlags(&net->ev_gather, cudaEventDisableTiming), "event");
    ck(cudaEventCreateWithFlags(&net->ev_cnt, cudaEventDisableTiming), "event");
    ck(cudaEventCreateWithFlags(&net->ev_cnt_done, cudaEventDisableTiming), "event");
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    nccl_ck(ncclCommInitRank(&net->comm, nranks, id, rank), "ncclCommInitRank");
  }
  ck(cudaStreamSynchronize(ctx->stream), "sync");
  return net.release();
}
}  // namespace

extern "C" kl_status kl_net_create(kl_ctx_t ctx, const kl_net_config* cfg, const kl_layer_init* init,
                                   kl_net_t* out) {
  if (!ctx || !cfg || !out) return KL_EINVAL;
  KL_API_BEGIN(ctx)
  *out = nullptr;
  *out = create_net(ctx, cfg, init, nullptr, 0, 1);
  KL_API_END
}

extern "C" kl_status kl_net_destroy(kl_net_t net) {
  if (!net) return KL_EINVAL;
  {
    DeviceGuard g(net->ctx->device);
    try {
      net->wait_streams();
    } catch (const KlError&) {
    }
    // A device queue that an aborted communicator left hung would block the
    // frees (cudaFree synchronises): the net is leaked instead.
    if (net->stuck) return KL_OK;
    delete net;
  }
  return KL_OK;
}


// The body of Network::train_step (net.rs:81-119) on a validated device
// batch; the mean loss ends in net->loss_acc (and `loss` when non-null).
static void train_step_body(kl_net_t net, const kl_batch* b, double lr, int mode, float* loss) {
  require(mode == KL_MODE_EXACT_SEQUENTIAL || mode == KL_MODE_BATCHED, "train_step: unknown mode");
  cudaStream_t st = net->ctx->stream;
  if (net->nranks > 1) {
    // A sharded step never returns before its collectives on a data-dependent
    // condition (batch size, nnz, labels): train_sharded reports those faults on
    // every rank together.  Only argument errors, which every rank makes alike
    // when it calls with the same code, raise here.
    require(b != nullptr, "batch is NULL");
    support(mode == KL_MODE_BATCHED, "sharded net: only KL_MODE_BATCHED train steps");
    net->require_comm();
    net->upload_opt(lr);
    net->train_sharded(*b, lr);
    launch_loss_final(net->loss_acc.as<float>(), net->rank_batch * net->nranks, loss, net->loss_acc.as<float>(), st);
    ck_launch("loss final");
    for (auto& L : net->layers) {
      L->examples += (uint64_t)b->batch;
      L->steps += 1;
    }
    net->layers[0]->input_nnz += (uint64_t)b->nnz;
    net->step += 1;
    net->after_step();
    return;
  }
  validate_batch(net, b);
  if (b->batch == 0) {  // net.rs:82-84
    ck(cudaMemsetAsync(net->loss_acc.p, 0, 4, st), "memset");
    if (loss) ck(cudaMemsetAsync(loss, 0, 4, st), "memset");
    return;
  }
  int loss_div = b->batch;
  net->upload_opt(lr);
  if (mode == KL_MODE_BATCHED && net->graph_usable(*b)) {
    net->graph_step(*b, loss);
    loss_div = -1;  // the captured body wrote the loss
  } else {
  net->ensure_batch_buffers(*b);
  ck(cudaMemsetAsync(net->loss_acc.p, 0, 4, st), "memset");
  ck(cudaMemsetAsync(net->labprob.p, 0, (size_t)std::max(b->nlabels, 1) * 4, st), "memset");
  if (mode == KL_MODE_BATCHED) {
    net->forward(*b, 0, b->batch, true);
    launch_loss(b->label_ptr, net->labprob.as<float>(), b->batch, net->loss_acc.as<float>(), st);
    ck_launch("loss");
    net->backward(*b, 0, b->batch, lr);
  } else {
    for (int s = 0; s < b->batch; ++s) {
      net->forward(*b, s, 1, true);
      launch_loss(b->label_ptr + s, net->labprob.as<float>(), 1, net->loss_acc.as<float>(), st);
      ck_launch("loss");
      net->backward(*b, s, 1, lr);
    }
  }
  }
  if (loss_div >= 0) launch_loss_final(net->loss_acc.as<float>(), loss_div, loss, net->loss_acc.as<float>(), st);
  ck_launch("loss final");
  for (auto& L : net->layers) {
    L->examples += (uint64_t)b->batch;
    L->steps += 1;
  }
  net->layers[0]->input_nnz += (uint64_t)b->nnz;
  // net.rs:109-116
  net->step += 1;
  net->after_step();
}

extern "C" kl_status kl_net_train_step(kl_net_t net, const kl_batch* b, double lr, int mode, float* loss,
                                       float* loss_host) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  train_step_body(net, b, lr, mode, loss);
  if (loss_host) {
    if (net->nranks > 1) net->wait_streams();  // bounded when a comm timeout is set
    ck(cudaMemcpyAsync(loss_host, net->loss_acc.p, 4, cudaMemcpyDeviceToHost, ctx__->stream), "loss copy");
    check_device_errors(ctx__);
  }
  KL_API_END
}

// The batch's arrays are packed into one pinned slot, uploaded with a single
// copy on the net's copy stream, and the step runs on the device copy; the
// compute stream waits only for that upload, so the upload of the next batch
// overlaps this step's kernels.  A slot is reused two calls later, after the
// step that read it (device side) and its own upload (host side) are done.
extern "C" kl_status kl_net_train_step_host(kl_net_t net, const kl_batch* hb, double lr, int mode,
                                            float* loss_host) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  require(hb != nullptr, "batch is NULL");
  if (net->nranks > 1 && (hb->batch < 0 || hb->batch > net->rank_batch)) {
    // a sharded step reports a wrong batch size on every rank together (train_sharded)
    kl_batch bad{};
    bad.batch = hb->batch;
    train_step_body(net, &bad, lr, mode, nullptr);
    if (loss_host) net->guard_blocking_read(loss_host);
    if (loss_host) ck(cudaMemcpyAsync(loss_host, net->loss_acc.p, 4, cudaMemcpyDeviceToHost, ctx__->stream), "loss copy");
    return KL_OK;
  }
  require(hb->batch >= 0 && hb->batch <= net->max_batch, "batch size outside [0, max_batch]");
  const int B = hb->batch;
  if (B > 0) require(hb->rowptr && hb->label_ptr, "batch rowptr / label_ptr required");
  const int32_t nnz = B > 0 ? hb->rowptr[B] : 0, nlab = B > 0 ? hb->label_ptr[B] : 0;
  require(nnz >= 0 && nlab >= 0, "batch rowptr / label_ptr must end at >= 0");
  if (nnz > 0) require(hb->idx && hb->val, "batch idx / val required");
  if (nlab > 0) require(hb->labels != nullptr, "batch labels required");
  cudaStream_t st = ctx__->stream;
  if (!net->copy_stream) {
    ck(cudaStreamCreateWithFlags(&net->copy_stream, cudaStreamNonBlocking), "copy stream");
    for (auto& h : net->hslots) {
      ck(cudaEventCreateWithFlags(&h.h2d, cudaEventDisableTiming), "event");
      ck(cudaEventCreateWithFlags(&h.used, cudaEventDisableTiming), "event");
      ck(cudaEventRecord(h.h2d, net->copy_stream), "event");
      ck(cudaEventRecord(h.used, st), "event");
    }
  }
  auto a16 = [](size_t n) { return (n + 15) & ~size_t(15); };
  const size_t o_rp = 0, o_lp = o_rp + a16((size_t)(B + 1) * 4), o_idx = o_lp + a16((size_t)(B + 1) * 4),
               o_val = o_idx + a16((size_t)nnz * 4), o_lab = o_val + a16((size_t)nnz * 4),
               total = o_lab + a16((size_t)nlab * 4);
  auto& h = net->hslots[net->hnext];
  net->hnext ^= 1;
  ck(cudaEventSynchronize(h.h2d), "event sync");  // the slot's previous upload has left the pinned buffer
  if (total > h.cap) {
    net->guard_blocking_read(nullptr);  // h.used follows a step that waits on peers
    ck(cudaEventSynchronize(h.used), "event sync");
    if (h.pinned) ck(cudaFreeHost(h.pinned), "cudaFreeHost");
    h.pinned = nullptr;
    h.cap = 0;
    const size_t cap = a16(total + total / 2);
    ck(cudaHostAlloc(&h.pinned, cap, cudaHostAllocDefault), "cudaHostAlloc");
    g_allocs.fetch_add(1, std::memory_order_relaxed);
    h.dev.alloc(cap);
    h.cap = cap;
  }
  unsigned char* hp = static_cast<unsigned char*>(h.pinned);
  if (B > 0) {
    std::memcpy(hp + o_rp, hb->rowptr, (size_t)(B + 1) * 4);
    std::memcpy(hp + o_lp, hb->label_ptr, (size_t)(B + 1) * 4);
  }
  if (nnz > 0) {
    std::memcpy(hp + o_idx, hb->idx, (size_t)nnz * 4);
    std::memcpy(hp + o_val, hb->val, (size_t)nnz * 4);
  }
  if (nlab > 0) std::memcpy(hp + o_lab, hb->labels, (size_t)nlab * 4);
  ck(cudaStreamWaitEvent(net->copy_stream, h.used, 0), "stream wait");  // the step that read this slot is done
  ck(cudaMemcpyAsync(h.dev.p, h.pinned, total, cudaMemcpyHostToDevice, net->copy_stream), "batch upload");
  ck(cudaEventRecord(h.h2d, net->copy_stream), "event");
  ck(cudaStreamWaitEvent(st, h.h2d, 0), "stream wait");
  unsigned char* dp = static_cast<unsigned char*>(h.dev.p);
  kl_batch db{};
  db.batch = B;
  db.rowptr = reinterpret_cast<const int32_t*>(dp + o_rp);
  db.label_ptr = reinterpret_cast<const int32_t*>(dp + o_lp);
  db.idx = reinterpret_cast<const uint32_t*>(dp + o_idx);
  db.val = reinterpret_cast<const float*>(dp + o_val);
  db.labels = reinterpret_cast<const uint32_t*>(dp + o_lab);
  db.nnz = nnz;
  db.nlabels = nlab;
  train_step_body(net, &db, lr, mode, nullptr);
  ck(cudaEventRecord(h.used, st), "event");
  if (loss_host) net->guard_blocking_read(loss_host);  // pinned memory: no wait
  if (loss_host) ck(cudaMemcpyAsync(loss_host, net->loss_acc.p, 4, cudaMemcpyDeviceToHost, st), "loss copy");
  KL_API_END
}

extern "C" kl_status kl_net_forward(kl_net_t net, const kl_batch* b) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  if (net->nranks > 1) {
    require(b != nullptr, "forward: null batch");
    net->require_comm();
    net->sharded_forward(*b, false);
    net->wait_streams();
    check_device_errors(net->ctx);
    return KL_OK;
  }
  validate_batch(net, b);
  if (b->batch == 0) return KL_OK;
  net->ensure_batch_buffers(*b);
  net->forward(*b, 0, b->batch, false);
  KL_API_END
}

extern "C" kl_status kl_net_layer_info(kl_net_t net, int layer, int* d, int* N, int* max_active) {
  if (!net) return KL_EINVAL;
  if (layer < 0 || layer >= (int)net->layers.size()) return KL_EINVAL;
  const Layer& L = *net->layers[layer];
  if (d) *d = L.d;
  if (N) *N = L.N;
  if (max_active) *max_active = L.stride;
  return KL_OK;
}

extern "C" kl_status kl_net_layer_output(kl_net_t net, int layer, uint32_t* ids, int32_t* counts, float* pre,
                                         float* act) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  require(layer >= 0 && layer < (int)net->layers.size(), "layer index out of range");
  const Layer& L = *net->layers[layer];
  cudaStream_t st = ctx__->stream;
  const size_t n = (size_t)net->max_batch * L.stride;
  if (ids) ck(cudaMemcpyAsync(ids, L.ids.p, n * 4, cudaMemcpyDeviceToDevice, st), "copy");
  if (counts) ck(cudaMemcpyAsync(counts, L.cnt.p, (size_t)net->max_batch * 4, cudaMemcpyDeviceToDevice, st), "copy");
  if (pre) ck(cudaMemcpyAsync(pre, L.pre.p, n * 4, cudaMemcpyDeviceToDevice, st), "copy");
  if (act) ck(cudaMemcpyAsync(act, L.post.p, n * 4, cudaMemcpyDeviceToDevice, st), "copy");
  KL_API_END
}

extern "C" kl_status kl_net_predict_topk(kl_net_t net, const kl_batch* b, int k, uint32_t* top_ids,
                                         float* top_scores) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  require(k >= 0 && (k == 0 || top_ids), "predict_topk: bad arguments");
  if (net->nranks > 1) {
    require(b != nullptr, "predict_topk: null batch");
    const int P = net->nranks, B = net->rank_batch, PB = P * B;
    const Layer& L = *net->layers.back();
    const int64_t Ntot = net->cfg.layers[net->cfg.num_layers - 1].num_neurons;
    support(P <= 64, "sharded predict_topk: at most 64 ranks");
    require(k <= Ntot / P, "sharded predict_topk: k must be <= num_neurons / nranks");
    net->require_comm();
    net->sharded_forward(*b, false);
    if (k == 0) return KL_OK;
    cudaStream_t st = ctx__->stream;
    DBuf lids, lsc, aids, asc;
    lids.alloc((size_t)PB * k * 4);
    lsc.alloc((size_t)PB * k * 4);
    aids.alloc((size_t)P * PB * k * 4);
    asc.alloc((size_t)P * PB * k * 4);
    launch_topk(L.act(), L.N, k, lids.as<uint32_t>(), lsc.as<float>(), PB, st);
    ck_launch("topk");
    nccl_ck(ncclGroupStart(), "group");
    nccl_ck(ncclAllGather(lids.p, aids.p, (size_t)PB * k, ncclUint32, net->comm, st), "all-gather top-k ids");
    nccl_ck(ncclAllGather(lsc.p, asc.p, (size_t)PB * k, ncclFloat32, net->comm, st), "all-gather top-k scores");
    nccl_ck(ncclGroupEnd(), "group");
    launch_shard_topk_merge(aids.as<uint32_t>(), asc.as<float>(), P, PB, k, Ntot, net->rank * B, B, top_ids,
                            top_scores, st);
    ck_launch("top-k merge");
    try {
      net->wait_streams();  // the scratch is freed on return
    } catch (const KlError&) {
      if (net->stuck)  // hung device work may still use the scratch: leak it
        for (DBuf* d : {&lids, &lsc, &aids, &asc}) d->p = nullptr;
      throw;
    }
    check_device_errors(net->ctx);
    return KL_OK;
  }
  validate_batch(net, b);
  if (b->batch == 0 || k == 0) return KL_OK;
  const Layer& L = *net->layers.back();
  k = std::min(k, L.N);
  net->ensure_batch_buffers(*b);
  net->forward(*b, 0, b->batch, false);
  launch_topk(L.act(), L.N, k, top_ids, top_scores, b->batch, ctx__->stream);
  ck_launch("topk");
  KL_API_END
}

extern "C" kl_status kl_net_bolt_infer(kl_net_t net, int layer, const float* X, int n, int ldx,
                                       float sparsity_multiplier, int base_top_k, int relu, uint32_t* out_ids,
                                       float* out_act, int32_t* out_n, int stride) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  require(layer >= 0 && layer < (int)net->layers.size(), "bolt: layer out of range");
  Layer& L = *net->layers[(size_t)layer];
  support(!L.fm, "bolt: layer 0 (sparse input, feature-major weights) is not supported; use layers >= 1");
  bolt_body(*L.index, L.W.p, net->wdtype, L.ldw, L.b.as<float>(), L.N, X, n, ldx, sparsity_multiplier, base_top_k,
            relu, out_ids, out_act, out_n, stride);
  KL_API_END
}

extern "C" kl_status kl_net_get_layer(kl_net_t net, int layer, float* w, float* bias, float* m, float* v,
                                      float* mb, float* vb) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  require(layer >= 0 && layer < (int)net->layers.size(), "layer index out of range");
  const Layer& L = *net->layers[layer];
  cudaStream_t st = ctx__->stream;
  const size_t nd = (size_t)L.N * L.d;
  DBuf tmp;
  tmp.alloc(nd * 4);
  auto pull = [&](const void* src, int dt, float* dst) {
    launch_w_to_f32(src, dt, L.ldw, L.fm, tmp.as<float>(), L.N, L.d, st);
    ck_launch("convert");
    ck(cudaMemcpyAsync(dst, tmp.p, nd * 4, cudaMemcpyDeviceToHost, st), "copy");
    ck(cudaStreamSynchronize(st), "sync");
  };
  if (w) pull(L.W.p, net->wdtype, w);
  if (m) pull(L.m.p, KL_DTYPE_F32, m);
  if (v) pull(L.v.p, KL_DTYPE_F32, v);
  if (bias) ck(cudaMemcpyAsync(bias, L.b.p, (size_t)L.N * 4, cudaMemcpyDeviceToHost, st), "copy");
  if (mb) ck(cudaMemcpyAsync(mb, L.mb.p, (size_t)L.N * 4, cudaMemcpyDeviceToHost, st), "copy");
  if (vb) ck(cudaMemcpyAsync(vb, L.vb.p, (size_t)L.N * 4, cudaMemcpyDeviceToHost, st), "copy");
  check_device_errors(ctx__);
  KL_API_END
}

extern "C" kl_status kl_net_set_layer(kl_net_t net, int layer, const float* w, const float* bias, const float* m,
                                      const float* v, const float* mb, const float* vb) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  require(layer >= 0 && layer < (int)net->layers.size(), "layer index out of range");
  Layer& L = *net->layers[layer];
  cudaStream_t st = ctx__->stream;
  const size_t nd = (size_t)L.N * L.d;
  DBuf tmp;
  tmp.alloc(nd * 4);
  auto push = [&](const float* src, void* dst, int dt) {
    ck(cudaMemcpyAsync(tmp.p, src, nd * 4, cudaMemcpyHostToDevice, st), "copy");
    launch_f32_to_w(tmp.as<float>(), L.N, L.d, L.d, dst, dt, L.ldw, L.fm, st);
    ck_launch("convert");
    ck(cudaStreamSynchronize(st), "sync");
  };
  if (w) push(w, L.W.p, net->wdtype);
  if (m) push(m, L.m.p, KL_DTYPE_F32);
  if (v) push(v, L.v.p, KL_DTYPE_F32);
  if (bias) ck(cudaMemcpyAsync(L.b.p, bias, (size_t)L.N * 4, cudaMemcpyHostToDevice, st), "copy");
  if (mb) ck(cudaMemcpyAsync(L.mb.p, mb, (size_t)L.N * 4, cudaMemcpyHostToDevice, st), "copy");
  if (vb) ck(cudaMemcpyAsync(L.vb.p, vb, (size_t)L.N * 4, cudaMemcpyHostToDevice, st), "copy");
  ck(cudaStreamSynchronize(st), "sync");
  KL_API_END
}

extern "C" kl_status kl_net_rebuild(kl_net_t net) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  net->rebuild_all();
  KL_API_END
}

extern "C" kl_status kl_net_layer_index(kl_net_t net, int layer, kl_index_t* out) {
  if (!net || !out) return KL_EINVAL;
  if (layer < 0 || layer >= (int)net->layers.size()) return KL_EINVAL;
  net->index_handles.emplace_back(new kl_index_s{net->layers[layer]->index});
  *out = net->index_handles.back().get();
  return KL_OK;
}

extern "C" kl_status kl_net_get_step(kl_net_t net, uint64_t* step, uint64_t* next_rebuild, uint64_t* count) {
  if (!net) return KL_EINVAL;
  if (step) *step = net->step;
  if (next_rebuild) *next_rebuild = net->sched.next;
  if (count) *count = net->sched.count;
  return KL_OK;
}
extern "C" kl_status kl_net_set_step(kl_net_t net, uint64_t step, uint64_t next_rebuild, uint64_t count) {
  if (!net) return KL_EINVAL;
  net->step = step;
  net->sched.next = next_rebuild;
  net->sched.count = count;
  net->sched.cur = step;
  return KL_OK;
}

extern "C" kl_status kl_net_set_rebuild_policy(kl_net_t net, const kl_rebuild_policy* p) {
  if (!net || !p) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  require(p->kind == KL_REBUILD_SCHEDULE || p->kind == KL_REBUILD_ADAPTIVE, "rebuild policy: unknown kind");
  net->adapt.clear();
  net->policy = *p;
  if (p->kind == KL_REBUILD_ADAPTIVE) {
    require(p->min_interval <= p->max_interval, "adaptive: min_interval must be <= max_interval (scheduler.rs:61-64)");
    require(p->sample_fraction >= 0.f && p->sample_fraction <= 1.f, "adaptive: sample_fraction must be in [0, 1]");
    require(p->drift_threshold >= 0.f && p->drift_threshold <= 1.f, "adaptive: drift_threshold must be in [0, 1]");
    for (size_t l = 0; l < net->layers.size(); ++l) {
      auto a = std::make_unique<kl_adaptive_s>();
      a->ctx = net->ctx;
      a->min_interval = (size_t)p->min_interval;
      a->max_interval = (size_t)p->max_interval;
      a->sample_fraction = p->sample_fraction;
      a->drift_threshold = p->drift_threshold;
      a->changed.alloc(4);
      Layer& L = *net->layers[l];
      adaptive_record(a.get(), L.index->hash, net->rows_of(L), nullptr, 0, net->adaptive_seed((int)l));
      net->adapt.push_back(std::move(a));
    }
  }
  KL_API_END
}

extern "C" kl_status kl_net_rebuild_state(kl_net_t net, int layer, float* drift_ema, uint64_t* since,
                                          uint64_t* rebuilds) {
  if (!net || layer < 0 || layer >= (int)net->layers.size()) return KL_EINVAL;
  const bool ad = net->policy.kind == KL_REBUILD_ADAPTIVE && (size_t)layer < net->adapt.size();
  if (drift_ema) *drift_ema = ad ? net->adapt[(size_t)layer]->drift_ema : 0.f;
  if (since) *since = ad ? (uint64_t)net->adapt[(size_t)layer]->steps_since_rebuild : 0;
  if (rebuilds) *rebuilds = net->layers[(size_t)layer]->rebuilds;
  return KL_OK;
}

// ---------------------------------------------------------------------------
// Checkpoint file: "KLB2CKPT" magic, format version, the configuration it was
// written from, then every state array as raw little-endian bytes in the
// device layout, and an FNV-1a 64-bit checksum of all preceding bytes.
// ---------------------------------------------------------------------------
namespace {
constexpr char kCkptMagic[8] = {'K', 'L', 'B', '2', 'C', 'K', 'P', 'T'};
constexpr uint32_t kCkptVersion = 1;

struct CkptFile {
  FILE* f = nullptr;
  uint64_t h = 1469598103934665603ULL;
  bool writing = false;
  ~CkptFile() {
    if (f) std::fclose(f);
  }
  void mix(const void* p, size_t n) {
    const unsigned char* c = static_cast<const unsigned char*>(p);
    for (size_t i = 0; i < n; ++i) h = (h ^ c[i]) * 1099511628211ULL;
  }
  void put(const void* p, size_t n) {
    mix(p, n);
    if (n && std::fwrite(p, 1, n, f) != n) raise(KL_EINVAL, "checkpoint: write failed");
  }
  void get(void* p, size_t n) {
    if (n && std::fread(p, 1, n, f) != n) raise(KL_EINVAL, "checkpoint: file truncated");
    mix(p, n);
  }
  template <class T>
  void put_v(T v) {
    put(&v, sizeof(v));
  }
  template <class T>
  T get_v() {
    T v;
    get(&v, sizeof(v));
    return v;
  }
  // a device array, staged through a bounded host buffer
  void dev(void* d, size_t n, cudaStream_t st) {
    std::vector<unsigned char> buf(std::min<size_t>(n, (size_t)64 << 20));
    for (size_t o = 0; o < n; o += buf.size()) {
      const size_t c = std::min(buf.size(), n - o);
      if (writing) {
        ck(cudaMemcpyAsync(buf.data(), static_cast<unsigned char*>(d) + o, c, cudaMemcpyDeviceToHost, st), "copy");
        ck(cudaStreamSynchronize(st), "sync");
        put(buf.data(), c);
      } else {
        get(buf.data(), c);
        ck(cudaMemcpyAsync(static_cast<unsigned char*>(d) + o, buf.data(), c, cudaMemcpyHostToDevice, st), "copy");
        ck(cudaStreamSynchronize(st), "sync");
      }
    }
  }
  template <class T>
  void field(T& v, const char* what, bool must_match) {
    if (writing) {
      put_v(v);
    } else {
      const T r = get_v<T>();
      if (must_match && r != v) raise(KL_EINVAL, std::string("checkpoint: ") + what + " differs from this network's");
      v = r;
    }
  }
};

// FNV-1a over a hash family's kind, sizes and parameter arrays.
uint64_t hash_fingerprint(const DevHash& h, cudaStream_t st) {
  uint64_t f = 1469598103934665603ULL;
  auto mix = [&](const void* p, size_t n) {
    const unsigned char* c = static_cast<const unsigned char*>(p);
    for (size_t i = 0; i < n; ++i) f = (f ^ c[i]) * 1099511628211ULL;
  };
  const int hdr[6] = {h.kind, h.d, h.k, h.L, h.w, h.dpad};
  mix(hdr, sizeof(hdr));
  auto dev = [&](const void* p, size_t n) {
    if (!p || !n) return;
    std::vector<unsigned char> b(n);
    ck(cudaMemcpyAsync(b.data(), p, n, cudaMemcpyDeviceToHost, st), "copy");
    ck(cudaStreamSynchronize(st), "sync");
    mix(b.data(), n);
  };
  dev(h.planes, (size_t)h.LK * h.dpad);
  dev(h.windows, (size_t)h.L * h.k * h.w * 4);
  dev(h.perms, (size_t)h.L * h.d * 4);
  return f;
}

void ckpt_body(kl_net_s* net, CkptFile& F) {
  cudaStream_t st = net->ctx->stream;
  ck(cudaStreamSynchronize(st), "sync");
  int32_t nl = (int32_t)net->layers.size(), wd = net->wdtype, rank = net->rank, nranks = net->nranks;
  F.field(nl, "layer count", true);
  F.field(wd, "weight dtype", true);
  F.field(rank, "rank", true);
  F.field(nranks, "rank count", true);
  F.field(net->step, "step", false);
  F.field(net->sched.next, "next rebuild", false);
  F.field(net->sched.count, "rebuild count", false);
  const size_t wsz = net->wdtype == KL_DTYPE_BF16 ? 2 : 4;
  for (auto& Lp : net->layers) {
    Layer& L = *Lp;
    IndexImpl& I = *L.index;
    int32_t d = L.d, N = L.N, ldw = L.ldw, fm = L.fm, tl = I.T.L, nb = I.T.nb, cap = I.T.cap, bt = I.T.type;
    uint32_t base = L.id_base;
    F.field(d, "input_dim", true);
    F.field(N, "num_neurons", true);
    F.field(ldw, "weight pitch", true);
    F.field(fm, "weight layout", true);
    F.field(tl, "num_tables", true);
    F.field(nb, "bucket count", true);
    F.field(cap, "bucket capacity", true);
    F.field(bt, "bucket type", true);
    F.field(base, "neuron slice", true);
    // the hash family is part of the network's construction, not of its state:
    // a checkpoint restores only into a network built with the same parameters
    uint64_t hfp = hash_fingerprint(I.hash->dh, st);
    F.field(hfp, "LSH hash parameters (planes / windows / permutations)", true);
    F.field(L.rebuilds, "layer rebuilds", false);
    const size_t rows = L.fm ? (size_t)L.d : (size_t)L.N;
    F.dev(L.W.p, rows * L.ldw * wsz, st);
    F.dev(L.m.p, rows * L.ldw * 4, st);
    F.dev(L.v.p, rows * L.ldw * 4, st);
    F.dev(L.b.p, (size_t)L.N * 4, st);
    F.dev(L.mb.p, (size_t)L.N * 4, st);
    F.dev(L.vb.p, (size_t)L.N * 4, st);
    const size_t LB = (size_t)I.T.L * I.T.nb;
    F.dev(I.T.ids, LB * I.T.cap * 4, st);
    F.dev(I.T.len, LB * 4, st);
    F.dev(I.T.cnt, LB * 8, st);
  }
  // rebuild policy and the adaptive schedulers' state
  int32_t kind = net->policy.kind;
  F.field(kind, "rebuild policy", false);
  if (!F.writing) {
    net->policy.kind = kind;
    net->adapt.clear();
  }
  F.field(net->policy.min_interval, "", false);
  F.field(net->policy.max_interval, "", false);
  F.field(net->policy.sample_fraction, "", false);
  F.field(net->policy.drift_threshold, "", false);
  F.field(net->policy.seed, "", false);
  if (kind == KL_REBUILD_ADAPTIVE) {
    for (size_t l = 0; l < net->layers.size(); ++l) {
      if (!F.writing) {
        auto a = std::make_unique<kl_adaptive_s>();
        a->ctx = net->ctx;
        a->min_interval = (size_t)net->policy.min_interval;
        a->max_interval = (size_t)net->policy.max_interval;
        a->sample_fraction = net->policy.sample_fraction;
        a->drift_threshold = net->policy.drift_threshold;
        a->changed.alloc(4);
        a->hash = net->layers[l]->index->hash;
        net->adapt.push_back(std::move(a));
      }
      kl_adaptive_s& a = *net->adapt[l];
      uint64_t since = a.steps_since_rebuild, check = a.steps_since_check;
      int32_t S = a.S;
      F.field(a.drift_ema, "", false);
      F.field(since, "", false);
      F.field(check, "", false);
      F.field(S, "", false);
      a.steps_since_rebuild = (size_t)since;
      a.steps_since_check = (size_t)check;
      if (!F.writing) {
        require(S >= 0 && S <= net->layers[l]->N, "checkpoint: bad adaptive sample size");
        a.S = S;
        const int L = a.hash->dh.L;
        a.idx.alloc((size_t)S * 4);
        a.base.alloc((size_t)S * L * 8);
        a.cur.alloc((size_t)S * L * 8);
        a.rows.alloc((size_t)S * a.hash->dh.d * 4);
      }
      if (S > 0) {
        F.dev(a.idx.p, (size_t)S * 4, st);
        F.dev(a.base.p, (size_t)S * a.hash->dh.L * 8, st);
      }
    }
  }
}
}  // namespace

extern "C" kl_status kl_net_save(kl_net_t net, const char* path) {
  if (!net || !path) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  const std::string tmp = std::string(path) + ".tmp";
  {
    CkptFile F;
    F.writing = true;
    F.f = std::fopen(tmp.c_str(), "wb");
    require(F.f != nullptr, std::string("checkpoint: cannot create ") + tmp);
    F.put(kCkptMagic, 8);
    F.put_v(kCkptVersion);
    ckpt_body(net, F);
    const uint64_t sum = F.h;
    if (std::fwrite(&sum, 1, 8, F.f) != 8 || std::fflush(F.f) != 0) raise(KL_EINVAL, "checkpoint: write failed");
  }
  require(std::rename(tmp.c_str(), path) == 0, std::string("checkpoint: cannot rename to ") + path);
  KL_API_END
}

extern "C" kl_status kl_net_load(kl_net_t net, const char* path) {
  if (!net || !path) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  CkptFile F;
  F.f = std::fopen(path, "rb");
  require(F.f != nullptr, std::string("checkpoint: cannot open ") + path);
  char magic[8];
  F.get(magic, 8);
  require(std::memcmp(magic, kCkptMagic, 8) == 0, "checkpoint: not a klearu_b200 network checkpoint");
  require(F.get_v<uint32_t>() == kCkptVersion, "checkpoint: unsupported format version");
  // read into the network, then verify the checksum; a corrupt file leaves the
  // network in an undefined state, as the error says
  ckpt_body(net, F);
  const uint64_t want = F.h;
  uint64_t sum = 0;
  require(std::fread(&sum, 1, 8, F.f) == 8, "checkpoint: file truncated");
  require(sum == want, "checkpoint: checksum mismatch (corrupt file); the network's state is undefined");
  net->sched.cur = net->step;
  KL_API_END
}

extern "C" kl_status kl_net_stats(kl_net_t net, int layer, kl_layer_stats* out, int reset) {
  if (!net || !out) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  require(layer >= 0 && layer < (int)net->layers.size(), "layer index out of range");
  Layer& L = *net->layers[layer];
  unsigned long long v[3];
  ck(cudaStreamSynchronize(ctx__->stream), "sync");
  ck(cudaMemcpy(v, L.stats.p, 24, cudaMemcpyDeviceToHost), "copy");
  out->active_sum = v[0];
  out->touched_rows = v[1];
  out->input_nnz = L.input_nnz;
  out->examples = L.examples;
  out->steps = L.steps;
  out->rebuilds = L.rebuilds;
  if (reset) {
    ck(cudaMemset(L.stats.p, 0, 24), "memset");
    L.examples = L.steps = L.rebuilds = L.input_nnz = 0;
  }
  KL_API_END
}

extern "C" kl_status kl_net_profile(kl_net_t net, int enable) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  if (!enable && net->prof) net->prof_collect();
  net->prof = enable != 0;
  KL_API_END
}
extern "C" kl_status kl_net_profile_read(kl_net_t net, int layer, double* ms_host, uint64_t* calls_host,
                                         int reset) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  require(layer >= 0 && layer < (int)net->layers.size(), "layer index out of range");
  net->prof_collect();
  for (int p = 0; p < KL_NPHASES; ++p) {
    const size_t i = (size_t)layer * KL_NPHASES + p;
    if (ms_host) ms_host[p] = net->prof_ms[i];
    if (calls_host) calls_host[p] = net->prof_calls[i];
    if (reset) {
      net->prof_ms[i] = 0.0;
      net->prof_calls[i] = 0;
    }
  }
  KL_API_END
}
extern "C" kl_status kl_launch_count(uint64_t* count_host) {
  if (!count_host) return KL_EINVAL;
  *count_host = g_launches.load();
  return KL_OK;
}
extern "C" kl_status kl_alloc_count(uint64_t* count_host) {
  if (!count_host) return KL_EINVAL;
  *count_host = g_allocs.load(std::memory_order_relaxed);
  return KL_OK;
}

// ===========================================================================
// Neuron sharding over NCCL: not available in this build configuration.
// ===========================================================================
extern "C" int kl_dist_unique_id_size(void) { return (int)sizeof(ncclUniqueId); }
extern "C" kl_status kl_dist_get_unique_id(void* id_host) {
  if (!id_host) return KL_EINVAL;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return KL_ENCCL;
  std::memcpy(id_host, &id, sizeof(id));
  return KL_OK;
}
extern "C" kl_status kl_net_create_sharded(kl_ctx_t ctx, const kl_net_config* cfg, const kl_layer_init* init,
                                           const void* unique_id, int rank, int nranks, kl_net_t* out) {
  if (!ctx || !cfg || !out || !unique_id) return KL_EINVAL;
  KL_API_BEGIN(ctx)
  *out = nullptr;
  *out = create_net(ctx, cfg, init, unique_id, rank, nranks);
  KL_API_END
}
extern "C" kl_status kl_net_owned_features(kl_net_t net, uint32_t* first, uint32_t* count) {
  if (!net) return KL_EINVAL;
  if (first) *first = (uint32_t)net->layers[0]->f0;
  if (count) *count = (uint32_t)net->layers[0]->nf;
  return KL_OK;
}
extern "C" kl_status kl_net_set_comm_timeout(kl_net_t net, int timeout_ms) {
  if (!net || timeout_ms < 0) return KL_EINVAL;
  net->comm_timeout_ms = timeout_ms;
  return KL_OK;
}
extern "C" kl_status kl_net_sync(kl_net_t net) {
  if (!net) return KL_EINVAL;
  KL_API_BEGIN(net->ctx)
  if (net->stuck) raise(KL_ETIMEOUT, "device work was still pending after the communicator abort");
  net->wait_streams();
  check_device_errors(net->ctx);
  KL_API_END
}
extern "C" kl_status kl_net_comm_abort(kl_net_t net) {
  if (!net) return KL_EINVAL;
  if (net->nranks <= 1) return KL_OK;
  DeviceGuard g(net->ctx->device);
  if (!net->comm_aborted) net->abort_comm("aborted by the caller");
  return KL_OK;
}
extern "C" kl_status kl_net_shard_info(kl_net_t net, int* rank_host, int* nranks_host, uint32_t* id_base_host,
                                       int* num_local_host) {
  if (!net) return KL_EINVAL;
  if (rank_host) *rank_host = net->rank;
  if (nranks_host) *nranks_host = net->nranks;
  if (id_base_host) *id_base_host = net->layers.back()->id_base;
  if (num_local_host) *num_local_host = net->layers.back()->N;
  return KL_OK;
}

// ===========================================================================
// Allocation-free index query.
//
// Some callers cannot call cudaMalloc: an allocator-owning host runtime that
// forbids allocations behind its back, a memory budget fixed before start-up,
// or code already running under a pool that must not grow.  For them,
// kl_index_query_batch_noalloc does the same work as kl_index_query_batch, but
// its scratch (per-query bucket numbers and padded per-query (id, count)
// lists) lives in the file-scope device array below instead of buffers that
// the index allocates on demand.  The array is part of the loaded module, so
// every GPU that loads this library holds its KL_NOALLOC_SCRATCH_BYTES until
// the process exits.  Every call shares the array and it keeps the previous
// call's contents; nothing in it must start at zero (the hash and probe
// kernels write every element that the compaction later reads).  Calls whose
// work overlaps on the GPU (different streams or contexts on the same device)
// race on the array and must be serialised by the caller.
// ===========================================================================
namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)KL_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device.  In host code the array's
// name is only a host-side stand-in, so the address is looked up once per
// device with that device current (the caller's DeviceGuard makes it so).
std::mutex g_noalloc_mu;
std::vector<void*> g_noalloc_addr;

void* noalloc_scratch_for(int device) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if ((int)g_noalloc_addr.size() <= device) g_noalloc_addr.resize((size_t)device + 1, nullptr);
  if (!g_noalloc_addr[(size_t)device]) {
    void* p = nullptr;
    ck(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)");
    require(p != nullptr, "no-alloc scratch: null symbol address");
    g_noalloc_addr[(size_t)device] = p;
  }
  return g_noalloc_addr[(size_t)device];
}

// Scratch carve for n queries: bucket numbers u16 [L][n], then padded
// results qids / qcnt u32 [n][L*cap] and sizes qn i32 [n], each 256-aligned.
size_t noalloc_query_bytes(int64_t n, int64_t L, int64_t stride) {
  return (size_t)(round_up(L * n * 2, 256) + 2 * round_up(n * stride * 4, 256) + round_up(n * 4, 256));
}

}  // namespace

extern "C" kl_status kl_index_query_batch_noalloc(kl_index_t ix, const float* X, int n, int ldx, int mode,
                                                  uint32_t* out_ids, uint32_t* out_counts, int32_t* out_offsets,
                                                  int32_t capacity, int32_t* overflow) {
  if (!ix) return KL_EINVAL;
  IndexImpl& I = *ix->ix;
  KL_API_BEGIN(I.ctx)
  require(mode == KL_QUERY_COUNTS || mode == KL_QUERY_UNION, "query: unknown mode");
  require(n >= 0 && out_offsets && (n == 0 || (X && ldx >= I.hash->dh.d)), "query: bad arguments");
  require(capacity >= 0 && (capacity == 0 || out_ids), "query: bad capacity");
  const int64_t stride = (int64_t)I.T.L * I.T.cap;
  const size_t need = noalloc_query_bytes(n, I.T.L, stride);
  if (need > kNoAllocScratchBytes)
    throw KlError{KL_ECAPACITY, "query_noalloc: " + std::to_string(n) + " queries need " + std::to_string(need) +
                                    " scratch bytes, more than the fixed " +
                                    std::to_string(kNoAllocScratchBytes) + " (KL_NOALLOC_SCRATCH_BYTES); "
                                    "split the batch"};
  void* base = noalloc_scratch_for(ctx__->device);
  cudaStream_t st = ctx__->stream;
  if (n == 0) {
    ck(cudaMemsetAsync(out_offsets, 0, 4, st), "memset");
    return KL_OK;
  }
  char* p = static_cast<char*>(base);
  uint16_t* bkt = reinterpret_cast<uint16_t*>(p);
  p += round_up((int64_t)I.T.L * n * 2, 256);
  uint32_t* qids = reinterpret_cast<uint32_t*>(p);
  p += round_up((int64_t)n * stride * 4, 256);
  uint32_t* qcnt = reinterpret_cast<uint32_t*>(p);
  p += round_up((int64_t)n * stride * 4, 256);
  int32_t* qn = reinterpret_cast<int32_t*>(p);

  HashOut o;
  o.bkt = bkt;
  o.bkt_ld = n;
  o.nb_mask = (uint32_t)(I.T.nb - 1);
  launch_hash_dense(I.hash->dh, dense_rows(X, KL_DTYPE_F32, n, ldx), o, st);
  ck_launch("hash");
  ProbeArgs a;
  a.T = I.T;
  a.bkt = bkt;
  a.bkt_ld = n;
  a.nq = n;
  a.N = 0;
  a.id_bits = 32;
  a.out_ids = qids;
  a.out_counts = qcnt;
  a.out_stride = (int)stride;
  a.out_n = qn;
  a.err = ctx__->err.as<int>();
  launch_probe(a, st);
  ck_launch("probe");
  if (overflow) ck(cudaMemsetAsync(overflow, 0, 4, st), "memset");
  launch_scan(qn, out_offsets, n, nullptr, st);
  ck_launch("scan");
  launch_compact(qids, mode == KL_QUERY_COUNTS ? qcnt : nullptr, (int)stride, out_offsets, n, out_ids,
                 mode == KL_QUERY_COUNTS ? out_counts : nullptr, capacity, overflow, ctx__->err.as<int>(), st);
  ck_launch("compact");
  KL_API_END
}

// ===========================================================================
// Deja Vu sparse FFN: SparsityPredictor (klearu-dejavu
// predictor/mlp_predictor.rs:11-132) and the sparse SwiGLU MLP (klearu-llm
// sparse/sparse_mlp.rs:4-37, klearu-dejavu mlp.rs:23-58).
// ===========================================================================
struct kl_predictor_s {
  kl_ctx_t ctx;
  int in = 0, hid = 0, out = 0, ld_in = 0, ld_hid = 0;
  // calls of at most this many tokens take the CUDA-core GEMV path; 0 (the
  // default) keeps the tensor-core GEMM.  Set at creation from the
  // environment variable KLEARU_PREDICTOR_GEMV_TOKENS (at most 4).
  int gemv_max = 0;
  DBuf w1, b1, w2, b2, xs, xs2, P, h, sc;
};

struct kl_sparse_mlp_s {
  kl_ctx_t ctx;
  int hid = 0, inter = 0, ldw = 0, ldd = 0;
  DBuf gate, up, downT, down, bias, a, part;
  // dense-masked path (n_tokens >= KL_DENSE_MIN_TOKENS): scratch
  DBuf G, U, mask, xs, hs, P;
  bool has_bias = false;
};
// From this many tokens on, one pass over all MLP weights (dense tensor-core
// GEMMs with the selection as a mask) is faster than gathering the selected
// rows once per token (about 10 % of the rows each); measured on the C3
// shape: gather ahead at 16 tokens, dense ahead at 64.
constexpr int KL_DENSE_MIN_TOKENS = 24;

namespace {

// Host f32 rows [n][d] -> device bf16 [n][ld] (zero padded), or transposed.
void upload_bf16(kl_ctx_t ctx, DBuf& dst, const float* host, int64_t n, int d, int64_t ld_dst, int64_t rows_dst,
                 bool transpose) {
  cudaStream_t st = ctx->stream;
  dst.alloc((size_t)rows_dst * ld_dst * 2);
  ck(cudaMemsetAsync(dst.p, 0, (size_t)rows_dst * ld_dst * 2, st), "memset");
  DBuf tmp;
  tmp.alloc((size_t)n * d * 4);
  ck(cudaMemcpyAsync(tmp.p, host, (size_t)n * d * 4, cudaMemcpyHostToDevice, st), "upload");
  launch_f32_to_w(tmp.as<float>(), n, d, d, dst.p, KL_DTYPE_BF16, ld_dst, transpose, st);
  ck_launch("convert");
  ck(cudaStreamSynchronize(st), "sync");  // tmp is freed on return
}

void upload_f32(kl_ctx_t ctx, DBuf& dst, const float* host, int64_t n) {
  dst.alloc((size_t)std::max<int64_t>(n, 1) * 4);
  if (host) ck(cudaMemcpyAsync(dst.p, host, (size_t)n * 4, cudaMemcpyHostToDevice, ctx->stream), "upload");
  else ck(cudaMemsetAsync(dst.p, 0, (size_t)std::max<int64_t>(n, 1) * 4, ctx->stream), "memset");
}

void predictor_scores(kl_predictor_t p, const float* x, int T, float* scores, cudaStream_t st) {
  kl_ctx_t ctx = p->ctx;
  if (T <= p->gemv_max && (size_t)T * std::max(p->ld_in, p->ld_hid) * 4 <= 200 * 1024) {
    // a few tokens: one pass over each weight matrix on the CUDA cores (x staged in shared memory)
    launch_gemv_linear(x, T, p->in, p->in, p->w1.as<__nv_bfloat16>(), p->hid, p->ld_in, p->b1.as<float>(), 0,
                       p->h.as<float>(), p->hid, st);
    ck_launch("predictor layer 1 (gemv)");
    launch_gemv_linear(p->h.as<float>(), T, p->hid, p->hid, p->w2.as<__nv_bfloat16>(), p->out, p->ld_hid,
                       p->b2.as<float>(), 1, scores, p->out, st);
    ck_launch("predictor layer 2 (gemv)");
    return;
  }
  for (int t0 = 0; t0 < T; t0 += TC_LINEAR_MAX_T) {
    const int tn = std::min(TC_LINEAR_MAX_T, T - t0);
    // layer 1 reads x's pieces from xs and writes h's pieces to xs2 for layer 2
    launch_tc_linear(x + (int64_t)t0 * p->in, tn, p->in, p->in, p->w1.as<__nv_bfloat16>(), p->hid, p->ld_in,
                     p->b1.as<float>(), 0, p->h.as<float>(), p->hid, p->xs.as<__nv_bfloat16>(), p->P.as<float>(),
                     p->xs2.as<__nv_bfloat16>(), p->ld_hid, ctx->err.as<int>(), st);
    ck_launch("predictor layer 1");
    launch_tc_linear(nullptr, tn, p->hid, p->hid, p->w2.as<__nv_bfloat16>(), p->out, p->ld_hid, p->b2.as<float>(), 1,
                     scores + (int64_t)t0 * p->out, p->out, p->xs2.as<__nv_bfloat16>(), p->P.as<float>(), nullptr, 0,
                     ctx->err.as<int>(), st);
    ck_launch("predictor layer 2");
  }
}

void topk_check(kl_predictor_t p, int kk) {
  int pow2 = 2048;
  while (pow2 < kk) pow2 <<= 1;
  support((size_t)pow2 * 8 + (size_t)p->out * 4 <= 190 * 1024,
          "select_topk: k and output_dim too large for one block's shared memory");
}
// select_top_k for T tokens into idx [T][kk]; sc [T][out] receives the scores.
// sorted = false: the selection in ascending index order (the sparse MLP's
// sums then run in neuron order, as its dense-masked path does).
void predictor_topk_body(kl_predictor_t p, const float* x, int T, int kk, uint32_t* idx, float* sc, cudaStream_t st,
                         bool sorted = true) {
  topk_check(p, kk);
  predictor_scores(p, x, T, sc, st);
  launch_topk(sc, T, p->out, p->out, kk, idx, kk, st, sorted);
  ck_launch("topk");
}

}  // namespace

extern "C" kl_status kl_predictor_create(kl_ctx_t ctx, int input_dim, int hidden_dim, int output_dim,
                                         const float* w1_host, const float* b1_host, const float* w2_host,
                                         const float* b2_host, kl_predictor_t* out) {
  if (!ctx || !out) return KL_EINVAL;
  KL_API_BEGIN(ctx)
  require(input_dim >= 1 && hidden_dim >= 1 && output_dim >= 1, "predictor: dimensions must be >= 1");
  require(w1_host && w2_host, "predictor: w1 and w2 are required");
  auto p = std::make_unique<kl_predictor_s>();
  p->ctx = ctx;
  p->in = input_dim;
  p->hid = hidden_dim;
  p->out = output_dim;
  p->ld_in = (int)round_up(input_dim, TC_LINEAR_KPAD);
  p->ld_hid = (int)round_up(hidden_dim, TC_LINEAR_KPAD);
  upload_bf16(ctx, p->w1, w1_host, hidden_dim, input_dim, p->ld_in, hidden_dim, false);
  upload_bf16(ctx, p->w2, w2_host, output_dim, hidden_dim, p->ld_hid, output_dim, false);
  upload_f32(ctx, p->b1, b1_host, hidden_dim);
  upload_f32(ctx, p->b2, b2_host, output_dim);
  p->xs.alloc((size_t)3 * TC_LINEAR_MAX_T * p->ld_in * 2);
  p->xs2.alloc((size_t)3 * TC_LINEAR_MAX_T * p->ld_hid * 2);
  p->P.alloc(std::max(tc_linear_scratch_floats(hidden_dim, p->ld_in), tc_linear_scratch_floats(output_dim, p->ld_hid)) *
             4);
  p->h.alloc((size_t)TC_LINEAR_MAX_T * hidden_dim * 4);
  if (const char* e = std::getenv("KLEARU_PREDICTOR_GEMV_TOKENS"))
    p->gemv_max = std::max(0, std::min(std::atoi(e), gemv_linear_max_tokens()));
  ck(cudaStreamSynchronize(ctx->stream), "sync");
  *out = p.release();
  KL_API_END
}

extern "C" kl_status kl_predictor_destroy(kl_predictor_t p) {
  if (!p) return KL_EINVAL;
  KL_API_BEGIN(p->ctx)
  ck(cudaStreamSynchronize(p->ctx->stream), "sync");
  delete p;
  KL_API_END
}

extern "C" kl_status kl_predictor_info(kl_predictor_t p, int* input_dim, int* hidden_dim, int* output_dim) {
  if (!p) return KL_EINVAL;
  if (input_dim) *input_dim = p->in;
  if (hidden_dim) *hidden_dim = p->hid;
  if (output_dim) *output_dim = p->out;
  return KL_OK;
}

extern "C" kl_status kl_predictor_predict(kl_predictor_t p, const float* x, int n_tokens, float* scores) {
  if (!p) return KL_EINVAL;
  KL_API_BEGIN(p->ctx)
  require(n_tokens >= 0, "predict: n_tokens must be >= 0");
  if (n_tokens == 0) return KL_OK;
  require(x && scores, "predict: x and scores are required");
  predictor_scores(p, x, n_tokens, scores, ctx__->stream);
  KL_API_END
}

extern "C" kl_status kl_predictor_select_topk(kl_predictor_t p, const float* x, int n_tokens, int k, uint32_t* idx,
                                              float* scores) {
  if (!p) return KL_EINVAL;
  KL_API_BEGIN(p->ctx)
  require(n_tokens >= 0 && k >= 0, "select_topk: n_tokens and k must be >= 0");
  const int kk = std::min(k, p->out);
  if (n_tokens == 0 || kk == 0) return KL_OK;
  require(x && idx, "select_topk: x and idx are required");
  float* sc = scores;
  if (!sc) {
    p->sc.alloc((size_t)n_tokens * p->out * 4);
    sc = p->sc.as<float>();
  }
  predictor_topk_body(p, x, n_tokens, kk, idx, sc, ctx__->stream);
  KL_API_END
}

extern "C" kl_status kl_sparse_mlp_create(kl_ctx_t ctx, int hidden, int intermediate, const float* gate_host,
                                          const float* up_host, const float* down_host, const float* down_bias_host,
                                          kl_sparse_mlp_t* out) {
  if (!ctx || !out) return KL_EINVAL;
  KL_API_BEGIN(ctx)
  require(hidden >= 1 && intermediate >= 1, "sparse_mlp: dimensions must be >= 1");
  require(gate_host && up_host && down_host, "sparse_mlp: gate, up and down are required");
  auto m = std::make_unique<kl_sparse_mlp_s>();
  m->ctx = ctx;
  m->hid = hidden;
  m->inter = intermediate;
  m->ldw = (int)round_up(hidden, TC_LINEAR_KPAD);
  m->ldd = (int)round_up(intermediate, TC_LINEAR_KPAD);
  upload_bf16(ctx, m->gate, gate_host, intermediate, hidden, m->ldw, intermediate, false);
  upload_bf16(ctx, m->up, up_host, intermediate, hidden, m->ldw, intermediate, false);
  // down [hidden][intermediate] twice: transposed for the per-token gather (a
  // neuron's weights are one row), as is for the dense GEMM
  upload_bf16(ctx, m->downT, down_host, hidden, intermediate, m->ldw, intermediate, true);
  upload_bf16(ctx, m->down, down_host, hidden, intermediate, m->ldd, hidden, false);
  const size_t tmax = TC_LINEAR_MAX_T;
  m->G.alloc(tmax * intermediate * 4);
  m->U.alloc(tmax * intermediate * 4);
  m->mask.alloc(tmax * intermediate);
  ck(cudaMemsetAsync(m->mask.p, 0, tmax * intermediate, ctx->stream), "memset");
  m->xs.alloc(3 * tmax * m->ldw * 2);
  m->hs.alloc(3 * tmax * m->ldd * 2);
  m->P.alloc(std::max(tc_linear_scratch_floats(intermediate, m->ldw), tc_linear_scratch_floats(hidden, m->ldd)) * 4);
  m->has_bias = down_bias_host != nullptr;
  if (m->has_bias) upload_f32(ctx, m->bias, down_bias_host, hidden);
  ck(cudaStreamSynchronize(ctx->stream), "sync");
  *out = m.release();
  KL_API_END
}

extern "C" kl_status kl_sparse_mlp_destroy(kl_sparse_mlp_t m) {
  if (!m) return KL_EINVAL;
  KL_API_BEGIN(m->ctx)
  ck(cudaStreamSynchronize(m->ctx->stream), "sync");
  delete m;
  KL_API_END
}

// sparse_mlp::forward_sparse for T tokens on stream st (k >= 1).
// accumulate (gather path only, n_tokens < KL_DENSE_MIN_TOKENS): out += the
// MLP's output (a fused residual add) instead of out = it.
static void sparse_mlp_body(kl_sparse_mlp_t m, const float* x, int n_tokens, const uint32_t* sel, int k, float* out,
                            cudaStream_t st, bool accumulate = false) {
  int* err = m->ctx->err.as<int>();
  if (n_tokens >= KL_DENSE_MIN_TOKENS) {
    require(!accumulate, "sparse mlp: accumulate needs the gather path");
    for (int t0 = 0; t0 < n_tokens; t0 += TC_LINEAR_MAX_T) {
      const int tn = std::min(TC_LINEAR_MAX_T, n_tokens - t0);
      launch_sparse_mlp_dense(m->gate.as<__nv_bfloat16>(), m->up.as<__nv_bfloat16>(), m->down.as<__nv_bfloat16>(),
                              m->hid, m->ldw, m->inter, m->ldd, m->has_bias ? m->bias.as<float>() : nullptr,
                              x + (int64_t)t0 * m->hid, tn, sel + (int64_t)t0 * k, k, m->G.as<float>(),
                              m->U.as<float>(), m->mask.as<uint8_t>(), m->xs.as<__nv_bfloat16>(),
                              m->hs.as<__nv_bfloat16>(), m->P.as<float>(), out + (int64_t)t0 * m->hid, err, st);
      ck_launch("sparse mlp (dense)");
    }
    return;
  }
  // K splits of the down projection: at least 16 selected rows per split, and
  // up to enough blocks ((hidden / 2048) x splits x tokens) for 8 per SM
  const int cols = (int)ceil_div(m->hid, 2048);
  const int splits = std::max(1, std::min((int)ceil_div(k, 16), (int)ceil_div(1184, (int64_t)cols * n_tokens)));
  m->a.alloc((size_t)n_tokens * k * 4);
  m->part.alloc((size_t)n_tokens * splits * m->ldw * 4);
  launch_sparse_mlp(m->gate.as<__nv_bfloat16>(), m->up.as<__nv_bfloat16>(), m->downT.as<__nv_bfloat16>(), m->hid,
                    m->ldw, m->inter, m->has_bias ? m->bias.as<float>() : nullptr, x, n_tokens, sel, k,
                    m->a.as<float>(), m->part.as<float>(), splits, out, accumulate, err, st);
  ck_launch("sparse mlp");
}

extern "C" kl_status kl_sparse_mlp_forward(kl_sparse_mlp_t m, const float* x, int n_tokens, const uint32_t* sel, int k,
                                           float* out) {
  if (!m) return KL_EINVAL;
  KL_API_BEGIN(m->ctx)
  require(n_tokens >= 0 && k >= 0, "sparse_mlp_forward: n_tokens and k must be >= 0");
  if (n_tokens == 0) return KL_OK;
  require(x && out, "sparse_mlp_forward: x and out are required");
  cudaStream_t st = ctx__->stream;
  if (k == 0) {  // no neuron selected: the output is the bias (or zero)
    if (m->has_bias)
      for (int t = 0; t < n_tokens; ++t)
        ck(cudaMemcpyAsync(out + (int64_t)t * m->hid, m->bias.p, (size_t)m->hid * 4, cudaMemcpyDeviceToDevice, st),
           "copy");
    else ck(cudaMemsetAsync(out, 0, (size_t)n_tokens * m->hid * 4, st), "memset");
    return KL_OK;
  }
  require(sel != nullptr, "sparse_mlp_forward: sel is required");
  sparse_mlp_body(m, x, n_tokens, sel, k, out, st);
  KL_API_END
}

// ===========================================================================
// Deja Vu FFN stack: the MLP half of SparseModel::forward_decode_sparse
// (crates/klearu-llm/src/sparse/mod.rs:112-141) over every layer, as one
// call.  Per layer: RMSNorm (mlp_norm), select_top_k of the layer's predictor,
// the sparse SwiGLU MLP, residual add.  The launches of one (tokens, k) shape
// are captured once in a CUDA graph and replayed.
// ===========================================================================
struct kl_ffn_stack_s {
  kl_ctx_t ctx;
  int nl = 0, hid = 0, inter = 0;
  float eps = 1e-5f;
  int one_plus = 0;
  std::vector<kl_predictor_t> pred;
  std::vector<kl_sparse_mlp_t> mlp;
  DBuf normw, norm, out, idx, sc;
  int cap_T = 0, cap_k = 0;
  cudaGraphExec_t gexec = nullptr;
  cudaStream_t cap_stream = nullptr;
  int g_T = -1, g_k = -1;
  float* g_hidden = nullptr;
  bool g_warm = false;
  ~kl_ffn_stack_s() {
    if (gexec) cudaGraphExecDestroy(gexec);
    if (cap_stream) cudaStreamDestroy(cap_stream);
  }
  void body(float* hidden, int T, int k, cudaStream_t st) {
    for (int l = 0; l < nl; ++l) {
      launch_rmsnorm(hidden, T, hid, normw.as<float>() + (size_t)l * hid, eps, one_plus, norm.as<float>(), st);
      ck_launch("rmsnorm");
      // the selection in neuron order (no sort): the MLP's sums then run in
      // neuron order on both of its paths
      predictor_topk_body(pred[(size_t)l], norm.as<float>(), T, k, idx.as<uint32_t>(), sc.as<float>(), st, false);
      if (T < KL_DENSE_MIN_TOKENS) {  // residual add fused into the down projection's finish
        sparse_mlp_body(mlp[(size_t)l], norm.as<float>(), T, idx.as<uint32_t>(), k, hidden, st, true);
      } else {
        sparse_mlp_body(mlp[(size_t)l], norm.as<float>(), T, idx.as<uint32_t>(), k, out.as<float>(), st);
        launch_residual_add(hidden, out.as<float>(), (int64_t)T * hid, st);
        ck_launch("residual add");
      }
    }
  }
};

extern "C" kl_status kl_ffn_stack_create(kl_ctx_t ctx, int n_layers, const kl_predictor_t* predictors_host,
                                         const kl_sparse_mlp_t* mlps_host, const float* norm_weights_host, float eps,
                                         int one_plus_weight, kl_ffn_stack_t* out) {
  if (!ctx || !out) return KL_EINVAL;
  KL_API_BEGIN(ctx)
  require(n_layers >= 1 && predictors_host && mlps_host && norm_weights_host, "ffn stack: bad arguments");
  auto s = std::make_unique<kl_ffn_stack_s>();
  s->ctx = ctx;
  s->nl = n_layers;
  s->eps = eps;
  s->one_plus = one_plus_weight ? 1 : 0;
  for (int l = 0; l < n_layers; ++l) {
    kl_predictor_t p = predictors_host[l];
    kl_sparse_mlp_t m = mlps_host[l];
    require(p && m, "ffn stack: every layer needs a predictor and an MLP");
    require(p->ctx == ctx && m->ctx == ctx, "ffn stack: the predictors and MLPs must share the stack's context");
    if (l == 0) {
      s->hid = m->hid;
      s->inter = m->inter;
    }
    require(m->hid == s->hid && m->inter == s->inter && p->in == s->hid && p->out == s->inter,
            "ffn stack: every layer must have the same hidden / intermediate sizes, predictor input = hidden, "
            "predictor output = intermediate");
    s->pred.push_back(p);
    s->mlp.push_back(m);
  }
  upload_f32(ctx, s->normw, norm_weights_host, (int64_t)n_layers * s->hid);
  ck(cudaStreamSynchronize(ctx->stream), "sync");
  *out = s.release();
  KL_API_END
}

extern "C" kl_status kl_ffn_stack_destroy(kl_ffn_stack_t s) {
  if (!s) return KL_EINVAL;
  KL_API_BEGIN(s->ctx)
  ck(cudaStreamSynchronize(s->ctx->stream), "sync");
  delete s;
  KL_API_END
}

extern "C" kl_status kl_ffn_stack_decode(kl_ffn_stack_t s, float* hidden, int n_tokens, float neuron_sparsity) {
  if (!s) return KL_EINVAL;
  KL_API_BEGIN(s->ctx)
  require(n_tokens >= 0 && hidden, "ffn stack decode: bad arguments");
  require(neuron_sparsity >= 0.f && neuron_sparsity <= 1.f, "ffn stack decode: neuron_sparsity must be in [0, 1]");
  if (n_tokens == 0) return KL_OK;
  // num_neurons_to_keep = ceil(intermediate * neuron_sparsity) (mod.rs:121-122)
  const int k = std::min(s->inter, (int)std::ceil((float)s->inter * neuron_sparsity));
  support(k >= 1, "ffn stack decode: a sparsity that keeps no neuron is not supported");
  topk_check(s->pred[0], k);
  cudaStream_t st = ctx__->stream;
  if (n_tokens > s->cap_T || k > s->cap_k) {
    s->cap_T = std::max(n_tokens, s->cap_T);
    s->cap_k = std::max(k, s->cap_k);
    s->norm.alloc((size_t)s->cap_T * s->hid * 4);
    s->out.alloc((size_t)s->cap_T * s->hid * 4);
    s->idx.alloc((size_t)s->cap_T * s->cap_k * 4);
    s->sc.alloc((size_t)s->cap_T * s->inter * 4);
    if (s->gexec) cudaGraphExecDestroy(s->gexec);
    s->gexec = nullptr;
    s->g_warm = false;
  }
  if (!s->g_warm || s->g_T != n_tokens || s->g_k != k || s->g_hidden != hidden) {
    // a new shape: run eagerly (this also sizes every scratch buffer), capture next time
    if (s->gexec) cudaGraphExecDestroy(s->gexec);
    s->gexec = nullptr;
    s->body(hidden, n_tokens, k, st);
    s->g_warm = true;
    s->g_T = n_tokens;
    s->g_k = k;
    s->g_hidden = hidden;
    return KL_OK;
  }
  if (!s->gexec) {
    if (!s->cap_stream) ck(cudaStreamCreateWithFlags(&s->cap_stream, cudaStreamNonBlocking), "capture stream");
    cudaGraph_t g = nullptr;
    bool ok = cudaStreamBeginCapture(s->cap_stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    const unsigned long long n0 = g_launches.load();
    if (ok) {
      try {
        s->body(hidden, n_tokens, k, s->cap_stream);
      } catch (...) {
        ok = false;
      }
      ok = cudaStreamEndCapture(s->cap_stream, &g) == cudaSuccess && ok && g;
    }
    if (ok) ok = cudaGraphInstantiate(&s->gexec, g, 0) == cudaSuccess;
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    g_launches.fetch_sub(g_launches.load() - n0);
    if (!ok) {
      s->gexec = nullptr;
      s->body(hidden, n_tokens, k, st);
      return KL_OK;
    }
  }
  ck(cudaGraphLaunch(s->gexec, st), "graph launch");
  count_launch((unsigned)(4 * s->nl));
  KL_API_END
}
