// data.cu -- LibSVM / XML datasets and shuffled CSR batches (host code).
//
// The input side of the train step: a LibSVM-format file (one example per
// line, "l1,l2,... idx:val idx:val ...") parsed on all host threads into one
// CSR store, and a batch iterator that shuffles the example order (seeded
// Fisher-Yates) and assembles each batch's CSR arrays in pinned host memory,
// one batch ahead on a worker thread.  Its kl_batch feeds
// kl_net_train_step_host, whose two upload slots overlap the next batch's
// host-to-device copy with the current step.
//
// Reference behaviour followed here:
//  * crates/klearu-core/src/data/libsvm.rs:39-111 (load_from_reader): blank
//    lines and '#' lines skipped, 1-based indices detected over the whole file
//    (minimum index 1 and no index 0), out-of-range indices clamped to
//    feature_dim - 1;
//  * libsvm.rs:127-185 (parse_line): comma-separated labels, a '#' token ends
//    the line, the four error messages;
//  * crates/klearu-core/src/tensor/sparse.rs:36-57 (from_pairs): stable sort by
//    index, duplicate indices summed in file order;
//  * crates/klearu-core/src/data/dataset.rs:48-111 (BatchIterator): SplitMix64
//    Fisher-Yates shuffle, batches of batch_size in shuffled order, the last
//    one short.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <charconv>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <type_traits>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "engine.h"

namespace kl {
void set_thread_error(const std::string& m);
}

struct kl_dataset_s {
  int64_t feature_dim = 0, num_labels = 0;
  std::vector<int64_t> rowptr{0};  // [n+1] into idx / val
  std::vector<uint32_t> idx;
  std::vector<float> val;
  std::vector<int64_t> lptr{0};    // [n+1] into labels
  std::vector<uint32_t> labels;
  int64_t size() const { return (int64_t)rowptr.size() - 1; }
};

namespace {

struct ParseError {
  std::string msg;
};

inline bool is_space(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\v' || c == '\f'; }

// u32::from_str: an optional '+', then one or more decimal digits, no overflow.
bool parse_u32(const char* b, const char* e, uint32_t* out) {
  if (b < e && *b == '+') ++b;
  if (b == e) return false;
  for (const char* p = b; p < e; ++p)
    if (*p < '0' || *p > '9') return false;
  auto r = std::from_chars(b, e, *out);
  return r.ec == std::errc() && r.ptr == e;
}

// f32::from_str: an optional sign, then a decimal number with an optional
// exponent, or inf / infinity / nan in any case; correctly rounded.
bool parse_f32(const char* b, const char* e, float* out) {
  bool neg = false;
  if (b < e && (*b == '+' || *b == '-')) {
    neg = *b == '-';
    ++b;
  }
  if (b == e || *b == '+' || *b == '-') return false;
  for (const char* p = b; p < e; ++p)
    if (*p == '(' || *p == 'x' || *p == 'X') return false;  // no nan(...) payloads, no hex floats
  float v = 0.0f;
  auto r = std::from_chars(b, e, v, std::chars_format::general);
  if (r.ptr != e) return false;
  if (r.ec == std::errc::result_out_of_range) {
    // from_chars leaves v unset on overflow / underflow; Rust returns inf / 0
    double d = 0.0;
    auto r2 = std::from_chars(b, e, d, std::chars_format::general);
    if (r2.ptr != e) return false;
    v = (float)d;
  } else if (r.ec != std::errc()) {
    return false;
  }
  *out = neg ? -v : v;
  return true;
}

std::string tok(const char* b, const char* e) { return std::string(b, (size_t)(e - b)); }

// One chunk of whole lines, parsed into raw (unadjusted) pairs.
struct Chunk {
  const char* b = nullptr;
  const char* e = nullptr;
  std::vector<int64_t> rowptr{0}, lptr{0};
  std::vector<uint32_t> idx, labels;
  std::vector<float> val;
  bool has_zero = false;
  uint32_t min_idx = UINT32_MAX;
  bool any_idx = false;
  int64_t lines = 0;        // lines in the chunk
  int64_t err_line = -1;    // chunk-local line number of the first error
  std::string err;
  // second pass output
  std::vector<int64_t> frow;
  std::vector<uint32_t> fidx;
  std::vector<float> fval;
};

void parse_line(Chunk& c, const char* b, const char* e, int64_t line_no) {
  // trim
  while (b < e && is_space(*b)) ++b;
  while (e > b && is_space(e[-1])) --e;
  if (b == e || *b == '#') return;
  const char* p = b;
  auto next_token = [&](const char** tb, const char** te) {
    while (p < e && is_space(*p)) ++p;
    if (p == e) return false;
    *tb = p;
    while (p < e && !is_space(*p)) ++p;
    *te = p;
    return true;
  };
  const char *tb, *te;
  next_token(&tb, &te);
  for (const char* s = tb;;) {
    const char* q = s;
    while (q < te && *q != ',') ++q;
    uint32_t l;
    if (!parse_u32(s, q, &l))
      throw ParseError{"line " + std::to_string(line_no + 1) + ": invalid label '" + tok(s, q) + "'"};
    c.labels.push_back(l);
    if (q == te) break;
    s = q + 1;
  }
  while (next_token(&tb, &te)) {
    if (*tb == '#') break;
    const char* colon = tb;
    while (colon < te && *colon != ':') ++colon;
    if (colon == te)
      throw ParseError{"line " + std::to_string(line_no + 1) + ": expected 'index:value', got '" + tok(tb, te) + "'"};
    uint32_t ix;
    float v;
    if (!parse_u32(tb, colon, &ix))
      throw ParseError{"line " + std::to_string(line_no + 1) + ": invalid feature index '" + tok(tb, colon) + "'"};
    if (!parse_f32(colon + 1, te, &v))
      throw ParseError{"line " + std::to_string(line_no + 1) + ": invalid feature value '" + tok(colon + 1, te) +
                       "'"};
    if (ix == 0) c.has_zero = true;
    c.min_idx = std::min(c.min_idx, ix);
    c.any_idx = true;
    c.idx.push_back(ix);
    c.val.push_back(v);
  }
  c.rowptr.push_back((int64_t)c.idx.size());
  c.lptr.push_back((int64_t)c.labels.size());
}

void parse_chunk(Chunk& c) {
  const char* p = c.b;
  int64_t line = 0;
  try {
    while (p < c.e) {
      const char* q = static_cast<const char*>(std::memchr(p, '\n', (size_t)(c.e - p)));
      const char* le = q ? q : c.e;
      parse_line(c, p, le, line);
      ++line;
      p = q ? q + 1 : c.e;
    }
  } catch (const ParseError& e) {
    c.err_line = line;
    c.err = e.msg;
  }
  c.lines = line;
}

// Adjust, clamp and normalise the chunk's rows (from_pairs).
void finish_chunk(Chunk& c, uint32_t offset, int64_t dim) {
  const int64_t n = (int64_t)c.rowptr.size() - 1;
  c.frow.assign(1, 0);
  c.fidx.reserve(c.idx.size());
  c.fval.reserve(c.val.size());
  std::vector<std::pair<uint32_t, float>> row;
  for (int64_t r = 0; r < n; ++r) {
    row.clear();
    for (int64_t k = c.rowptr[r]; k < c.rowptr[r + 1]; ++k) {
      uint32_t a = c.idx[k] - offset;
      if ((int64_t)a >= dim) a = (uint32_t)(dim - 1);
      row.emplace_back(a, c.val[k]);
    }
    std::stable_sort(row.begin(), row.end(), [](const auto& x, const auto& y) { return x.first < y.first; });
    const size_t start = c.fidx.size();
    for (auto& pr : row) {
      if (c.fidx.size() > start && c.fidx.back() == pr.first) {
        c.fval.back() += pr.second;
        continue;
      }
      c.fidx.push_back(pr.first);
      c.fval.push_back(pr.second);
    }
    c.frow.push_back((int64_t)c.fidx.size());
  }
  std::vector<uint32_t>().swap(c.idx);
  std::vector<float>().swap(c.val);
}

kl_dataset_s* parse_text(const char* text, size_t len, int64_t dim, int64_t nlab, int threads) {
  if (dim < 1) throw ParseError{"feature_dim must be >= 1"};
  if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  // whole-line chunks of at least 1 MiB each
  const size_t want = std::max<size_t>(1, std::min<size_t>((size_t)threads, len / (1u << 20) + 1));
  std::vector<Chunk> ch(want);
  size_t pos = 0;
  for (size_t i = 0; i < want; ++i) {
    size_t end = i + 1 == want ? len : std::max(pos, len * (i + 1) / want);
    if (end < len) {
      const char* q = static_cast<const char*>(std::memchr(text + end, '\n', len - end));
      end = q ? (size_t)(q - text) + 1 : len;
    }
    ch[i].b = text + pos;
    ch[i].e = text + end;
    pos = end;
  }
  auto run = [&](auto&& f) {
    std::vector<std::thread> ts;
    for (size_t i = 1; i < ch.size(); ++i) ts.emplace_back([&, i] { f(ch[i]); });
    f(ch[0]);
    for (auto& t : ts) t.join();
  };
  run([](Chunk& c) { parse_chunk(c); });
  int64_t lines_before = 0;
  for (auto& c : ch) {
    if (c.err_line >= 0) {
      // the chunk numbered its lines from 0: renumber the message for the whole file
      std::string m = c.err;
      const std::string pre = "line " + std::to_string(c.err_line + 1) + ":";
      if (m.compare(0, pre.size(), pre) == 0)
        m = "line " + std::to_string(lines_before + c.err_line + 1) + ":" + m.substr(pre.size());
      throw ParseError{m};
    }
    lines_before += c.lines;
  }
  bool has_zero = false, any = false;
  uint32_t mn = UINT32_MAX;
  for (auto& c : ch) {
    has_zero |= c.has_zero;
    any |= c.any_idx;
    mn = std::min(mn, c.min_idx);
  }
  const uint32_t offset = (!has_zero && any && mn == 1) ? 1u : 0u;  // libsvm.rs:74-78
  run([&](Chunk& c) { finish_chunk(c, offset, dim); });
  auto* ds = new kl_dataset_s();
  ds->feature_dim = dim;
  ds->num_labels = nlab;
  size_t nnz = 0, nl = 0, n = 0;
  for (auto& c : ch) {
    nnz += c.fidx.size();
    nl += c.labels.size();
    n += c.frow.size() - 1;
  }
  ds->rowptr.reserve(n + 1);
  ds->lptr.reserve(n + 1);
  ds->idx.reserve(nnz);
  ds->val.reserve(nnz);
  ds->labels.reserve(nl);
  for (auto& c : ch) {
    const int64_t b0 = (int64_t)ds->idx.size(), l0 = (int64_t)ds->labels.size();
    for (size_t r = 1; r < c.frow.size(); ++r) {
      ds->rowptr.push_back(b0 + c.frow[r]);
      ds->lptr.push_back(l0 + c.lptr[r]);
    }
    ds->idx.insert(ds->idx.end(), c.fidx.begin(), c.fidx.end());
    ds->val.insert(ds->val.end(), c.fval.begin(), c.fval.end());
    ds->labels.insert(ds->labels.end(), c.labels.begin(), c.labels.end());
  }
  return ds;
}

uint64_t splitmix64(uint64_t state) {  // dataset.rs:82-87
  uint64_t z = state + 0x9e3779b97f4a7c15ULL;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

}  // namespace

// Host buffers of the batch slots: page-locked, or malloc'd where no CUDA
// device is present (those are remembered so that they are freed with free()).
static std::mutex& pageable_mu() {
  static std::mutex m;
  return m;
}
static std::vector<void*>& pageable() {
  static std::vector<void*> v;
  return v;
}
static void free_host(void* p) {
  if (!p) return;
  {
    std::lock_guard<std::mutex> g(pageable_mu());
    auto& v = pageable();
    auto it = std::find(v.begin(), v.end(), p);
    if (it != v.end()) {
      v.erase(it);
      std::free(p);
      return;
    }
  }
  cudaFreeHost(p);
}

// One assembled batch in host memory.
struct BatchSlot {
  int32_t* rowptr = nullptr;
  int32_t* lptr = nullptr;
  uint32_t* idx = nullptr;
  float* val = nullptr;
  uint32_t* labels = nullptr;
  size_t cap_rp = 0, cap_lp = 0, cap_idx = 0, cap_val = 0, cap_lab = 0;
  int batch = 0;
  int32_t nnz = 0, nlab = 0;
  bool ready = false;
  void release() {
    free_host(rowptr);
    free_host(lptr);
    free_host(idx);
    free_host(val);
    free_host(labels);
    rowptr = lptr = nullptr;
    idx = labels = nullptr;
    val = nullptr;
    cap_rp = cap_lp = cap_idx = cap_val = cap_lab = 0;
  }
};

struct kl_batch_iter_s {
  const kl_dataset_s* ds = nullptr;
  int batch_size = 1;
  bool prefetch = true;
  std::vector<int64_t> order;
  int64_t pos = 0;          // next example (position in `order`) to assemble
  int64_t nbatches = 0;     // batches in the epoch
  int64_t taken = 0;        // batches returned by next() this epoch
  int held = -1;            // slot returned by the previous next() (in the caller's hands)
  BatchSlot slot[2];
  int fill = 0;             // slot the worker fills next
  int take = 0;             // slot next() returns next
  std::thread worker;
  std::mutex mu;
  std::condition_variable cv;
  bool stop = false;
  std::string werr;         // a worker's failure (pinned allocation)

  void shuffle(uint64_t seed) {  // dataset.rs:60-80
    order.resize((size_t)ds->size());
    for (size_t i = 0; i < order.size(); ++i) order[i] = (int64_t)i;
    uint64_t st = seed;
    for (size_t i = order.size(); i-- > 1;) {
      st = splitmix64(st);
      const size_t j = (size_t)(st % (uint64_t)(i + 1));
      std::swap(order[i], order[j]);
    }
    pos = 0;
    taken = 0;
    held = -1;
    nbatches = ((int64_t)order.size() + batch_size - 1) / batch_size;
  }
  // Assemble the batch starting at `pos` into `s` (no lock held).
  void assemble(BatchSlot& s, int64_t p0) {
    const int64_t p1 = std::min<int64_t>(p0 + batch_size, (int64_t)order.size());
    const int B = (int)(p1 - p0);
    size_t nnz = 0, nl = 0;
    for (int64_t p = p0; p < p1; ++p) {
      const int64_t e = order[(size_t)p];
      nnz += (size_t)(ds->rowptr[e + 1] - ds->rowptr[e]);
      nl += (size_t)(ds->lptr[e + 1] - ds->lptr[e]);
    }
    if (nnz > (size_t)INT32_MAX || nl > (size_t)INT32_MAX) throw ParseError{"batch exceeds 2^31 nnz or labels"};
    // Page-locked buffers, so that the host-to-device copy of a batch runs at full
    // PCIe / C2C speed; pageable memory where no CUDA device is present (a host
    // without a GPU can still iterate a dataset).
    auto grow = [](auto*& ptr, size_t& cap, size_t need) {
      if (need <= cap && ptr) return;
      free_host(ptr);
      ptr = nullptr;
      const size_t c = std::max<size_t>(need + need / 2, 64);
      void* q = nullptr;
      if (cudaHostAlloc(&q, c * sizeof(*ptr), cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        q = std::malloc(c * sizeof(*ptr) + 64);
        if (!q) {
          cap = 0;
          throw ParseError{"host allocation failed for a batch buffer"};
        }
        std::lock_guard<std::mutex> g(pageable_mu());
        pageable().push_back(q);
      }
      ptr = static_cast<std::remove_reference_t<decltype(ptr)>>(q);
      cap = c;
    };
    grow(s.rowptr, s.cap_rp, (size_t)B + 1);
    grow(s.lptr, s.cap_lp, (size_t)B + 1);
    grow(s.idx, s.cap_idx, nnz);
    grow(s.val, s.cap_val, nnz);
    grow(s.labels, s.cap_lab, nl);
    int64_t a = 0, l = 0;
    s.rowptr[0] = 0;
    s.lptr[0] = 0;
    for (int i = 0; i < B; ++i) {
      const int64_t e = order[(size_t)(p0 + i)];
      const int64_t r0 = ds->rowptr[e], r1 = ds->rowptr[e + 1];
      std::memcpy(s.idx + a, ds->idx.data() + r0, (size_t)(r1 - r0) * 4);
      std::memcpy(s.val + a, ds->val.data() + r0, (size_t)(r1 - r0) * 4);
      a += r1 - r0;
      const int64_t q0 = ds->lptr[e], q1 = ds->lptr[e + 1];
      std::memcpy(s.labels + l, ds->labels.data() + q0, (size_t)(q1 - q0) * 4);
      l += q1 - q0;
      s.rowptr[i + 1] = (int32_t)a;
      s.lptr[i + 1] = (int32_t)l;
    }
    s.batch = B;
    s.nnz = (int32_t)a;
    s.nlab = (int32_t)l;
  }
  void run() {
    std::unique_lock<std::mutex> lk(mu);
    while (!stop) {
      BatchSlot& s = slot[fill];
      if (s.ready || pos >= (int64_t)order.size()) {
        cv.wait(lk);
        continue;
      }
      const int64_t p0 = pos;
      pos = std::min<int64_t>(pos + batch_size, (int64_t)order.size());
      lk.unlock();
      std::string err;
      try {
        assemble(s, p0);
      } catch (const ParseError& e) {
        err = e.msg;
      }
      lk.lock();
      if (!err.empty()) {
        werr = err;
        s.batch = 0;
      }
      s.ready = true;
      fill ^= 1;
      cv.notify_all();
    }
  }
  void start() {
    stop = false;
    if (prefetch) worker = std::thread([this] { run(); });
  }
  void halt() {
    if (worker.joinable()) {
      {
        std::lock_guard<std::mutex> g(mu);
        stop = true;
      }
      cv.notify_all();
      worker.join();
    }
    slot[0].ready = slot[1].ready = false;
    fill = take = 0;
    held = -1;
  }
  ~kl_batch_iter_s() {
    halt();
    slot[0].release();
    slot[1].release();
  }
};

#define KL_DATA_TRY try {
#define KL_DATA_CATCH                          \
  }                                            \
  catch (const ParseError& e) {                \
    kl::set_thread_error(e.msg);               \
    return KL_EINVAL;                          \
  }                                            \
  catch (const std::bad_alloc&) {              \
    kl::set_thread_error("host allocation failed"); \
    return KL_ENOMEM;                          \
  }

extern "C" kl_status kl_libsvm_parse(const char* text_host, size_t len, int64_t feature_dim, int64_t num_labels,
                                     int threads, kl_dataset_t* out) {
  if (!out || (!text_host && len)) return KL_EINVAL;
  KL_DATA_TRY
  *out = parse_text(text_host ? text_host : "", len, feature_dim, num_labels, threads);
  return KL_OK;
  KL_DATA_CATCH
}

extern "C" kl_status kl_libsvm_load(const char* path, int64_t feature_dim, int64_t num_labels, int threads,
                                    kl_dataset_t* out) {
  if (!out || !path) return KL_EINVAL;
  KL_DATA_TRY
  FILE* f = std::fopen(path, "rb");
  if (!f) throw ParseError{std::string("cannot open ") + path};
  std::vector<char> buf;
  char tmp[1 << 16];
  size_t n;
  while ((n = std::fread(tmp, 1, sizeof(tmp), f)) > 0) buf.insert(buf.end(), tmp, tmp + n);
  const bool bad = std::ferror(f) != 0;
  std::fclose(f);
  if (bad) throw ParseError{std::string("read error on ") + path};
  *out = parse_text(buf.data(), buf.size(), feature_dim, num_labels, threads);
  return KL_OK;
  KL_DATA_CATCH
}

extern "C" kl_status kl_dataset_from_csr(const int64_t* rowptr_host, const uint32_t* idx_host, const float* val_host,
                                         const int64_t* label_ptr_host, const uint32_t* labels_host, int64_t n,
                                         int64_t feature_dim, int64_t num_labels, kl_dataset_t* out) {
  if (!out || n < 0 || (n > 0 && (!rowptr_host || !label_ptr_host))) return KL_EINVAL;
  KL_DATA_TRY
  auto* ds = new kl_dataset_s();
  ds->feature_dim = feature_dim;
  ds->num_labels = num_labels;
  if (n > 0) {
    ds->rowptr.assign(rowptr_host, rowptr_host + n + 1);
    ds->lptr.assign(label_ptr_host, label_ptr_host + n + 1);
    const int64_t base = ds->rowptr[0], lbase = ds->lptr[0];
    for (auto& r : ds->rowptr) r -= base;
    for (auto& r : ds->lptr) r -= lbase;
    const int64_t nnz = ds->rowptr[(size_t)n], nl = ds->lptr[(size_t)n];
    if (nnz < 0 || nl < 0 || (nnz && (!idx_host || !val_host)) || (nl && !labels_host)) {
      delete ds;
      throw ParseError{"from_csr: inconsistent arrays"};
    }
    ds->idx.assign(idx_host + base, idx_host + base + nnz);
    ds->val.assign(val_host + base, val_host + base + nnz);
    ds->labels.assign(labels_host + lbase, labels_host + lbase + nl);
  }
  *out = ds;
  return KL_OK;
  KL_DATA_CATCH
}

extern "C" kl_status kl_dataset_destroy(kl_dataset_t ds) {
  if (!ds) return KL_EINVAL;  // as every other destroy call
  delete ds;
  return KL_OK;
}

extern "C" kl_status kl_dataset_info(kl_dataset_t ds, int64_t* len_host, int64_t* feature_dim_host,
                                     int64_t* num_labels_host, int64_t* nnz_host, int64_t* nlabels_host) {
  if (!ds) return KL_EINVAL;
  if (len_host) *len_host = ds->size();
  if (feature_dim_host) *feature_dim_host = ds->feature_dim;
  if (num_labels_host) *num_labels_host = ds->num_labels;
  if (nnz_host) *nnz_host = (int64_t)ds->idx.size();
  if (nlabels_host) *nlabels_host = (int64_t)ds->labels.size();
  return KL_OK;
}

extern "C" kl_status kl_dataset_csr(kl_dataset_t ds, const int64_t** rowptr, const uint32_t** idx, const float** val,
                                    const int64_t** label_ptr, const uint32_t** labels) {
  if (!ds) return KL_EINVAL;
  if (rowptr) *rowptr = ds->rowptr.data();
  if (idx) *idx = ds->idx.data();
  if (val) *val = ds->val.data();
  if (label_ptr) *label_ptr = ds->lptr.data();
  if (labels) *labels = ds->labels.data();
  return KL_OK;
}

extern "C" kl_status kl_batch_iter_create(kl_dataset_t ds, int batch_size, uint64_t seed, int prefetch,
                                          kl_batch_iter_t* out) {
  if (!ds || !out) return KL_EINVAL;
  if (batch_size < 1) {
    kl::set_thread_error("batch_size must be >= 1");
    return KL_EINVAL;
  }
  KL_DATA_TRY
  auto* it = new kl_batch_iter_s();
  it->ds = ds;
  it->batch_size = batch_size;
  it->prefetch = prefetch != 0;
  it->shuffle(seed);
  it->start();
  *out = it;
  return KL_OK;
  KL_DATA_CATCH
}

extern "C" kl_status kl_batch_iter_reset(kl_batch_iter_t it, uint64_t seed) {
  if (!it) return KL_EINVAL;
  KL_DATA_TRY
  it->halt();
  it->shuffle(seed);
  it->start();
  return KL_OK;
  KL_DATA_CATCH
}

extern "C" kl_status kl_batch_iter_next(kl_batch_iter_t it, kl_batch* batch_host) {
  if (!it || !batch_host) return KL_EINVAL;
  KL_DATA_TRY
  BatchSlot* s = nullptr;
  if (it->taken >= it->nbatches) {
    *batch_host = kl_batch{};  // the epoch is over
    return KL_OK;
  }
  if (it->prefetch) {
    std::unique_lock<std::mutex> lk(it->mu);
    if (it->held >= 0) {  // the previous call's batch goes back to the worker
      it->slot[it->held].ready = false;
      it->held = -1;
      it->cv.notify_all();
    }
    it->cv.wait(lk, [&] { return it->slot[it->take].ready; });
    s = &it->slot[it->take];
    if (!it->werr.empty()) {
      std::string m = it->werr;
      it->werr.clear();
      throw ParseError{m};
    }
    it->held = it->take;
    it->take ^= 1;
  } else {
    s = &it->slot[it->take];
    const int64_t p0 = it->pos;
    it->pos = std::min<int64_t>(it->pos + it->batch_size, (int64_t)it->order.size());
    it->assemble(*s, p0);
    it->take ^= 1;
  }
  it->taken += 1;
  kl_batch b{};
  b.batch = s->batch;
  b.rowptr = s->rowptr;
  b.idx = s->idx;
  b.val = s->val;
  b.label_ptr = s->lptr;
  b.labels = s->labels;
  b.nnz = s->nnz;
  b.nlabels = s->nlab;
  *batch_host = b;
  return KL_OK;
  KL_DATA_CATCH
}

extern "C" kl_status kl_batch_iter_destroy(kl_batch_iter_t it) {
  if (!it) return KL_EINVAL;
  delete it;
  return KL_OK;
}
