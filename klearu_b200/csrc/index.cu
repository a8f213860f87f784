// index.cu -- bucket tables of the LSH index: batched ordered inserts
// (rebuild), removals, and the per-query probe/union/select kernel.
//
// Reference semantics (crates/klearu-core/src):
//  * FifoBucket::insert (bucket/fifo.rs:27-33): a full bucket drops its
//    oldest id.  After inserting a sequence into a bucket holding `len0` ids,
//    the bucket holds the last `cap` ids of (old contents ++ new ids).
//  * ReservoirBucket::insert (bucket/reservoir.rs:50-67): count += 1; push
//    while len < cap; otherwise seed = count*0x517cc1b727220a95 + id,
//    j = splitmix(seed) % count, and if j < cap the id overwrites slot
//    splitmix(seed+1) % cap.  Each insertion's decision depends only on its
//    (count, id), so all insertions are evaluated in parallel and every slot
//    keeps its LAST writer (largest insertion rank) via a 64-bit atomicMax of
//    (rank+1) << 32 | id.
//  * LshIndex::insert / rebuild (lsh/index.rs:257-262, 302-307): items are
//    inserted in array order; bucket = hash & (2^K - 1).
// The per-bucket insertion rank of every item is computed by a stable
// counting sort: per-chunk bucket histograms, an exclusive scan over chunks,
// and a second pass that ranks items inside each chunk in order with
// __match_any_sync.
#include <cub/block/block_scan.cuh>

#include <algorithm>

#include "engine.h"

namespace kl {
namespace {

// ---- insert pass 1: per (table, chunk) bucket histogram (one warp per block)
__global__ void ins_count_kernel(DevTables T, const uint16_t* bkt, int64_t bkt_ld, int n,
                                 uint32_t* chunk_cnt, int nchunks) {
  extern __shared__ uint32_t hist[];  // [nb]
  const int t = blockIdx.y, c = blockIdx.x;
  for (int b = threadIdx.x; b < T.nb; b += 32) hist[b] = 0;
  __syncwarp();
  const int i0 = c * INSERT_CHUNK, i1 = min(n, i0 + INSERT_CHUNK);
  for (int base = i0; base < i1; base += 32) {
    const int i = base + threadIdx.x;
    const bool valid = i < i1;
    const int b = valid ? (int)bkt[(int64_t)t * bkt_ld + i] : -1;
    const unsigned peers = __match_any_sync(FULL, b);
    if (valid && (int)threadIdx.x == __ffs(peers) - 1) hist[b] += __popc(peers);
    __syncwarp();
  }
  uint32_t* dst = chunk_cnt + ((int64_t)t * nchunks + c) * T.nb;
  for (int b = threadIdx.x; b < T.nb; b += 32) dst[b] = hist[b];
}

// ---- insert pass 2: exclusive scan over chunks per (table, bucket), then the
// per-bucket plan: FIFO keeps `base` old ids (shifted to the front) and drops
// the first `skip` new ones; reservoir seeds the packed slot array.
// One warp per (table, bucket): the scan over the chunks runs 32 chunks at a
// time (a warp scan per round), so a rebuild of millions of rows (thousands
// of chunks) does not walk them one dependent load after another.
__global__ void ins_plan_kernel(DevTables T, uint32_t* chunk_cnt, int nchunks, uint32_t* total,
                                uint32_t* basev, uint32_t* skipv, unsigned long long* temp) {
  const int64_t g = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (g >= (int64_t)T.L * T.nb) return;
  const int t = (int)(g / T.nb), b = (int)(g % T.nb);
  uint32_t run = 0;
  for (int c0 = 0; c0 < nchunks; c0 += 32) {
    const int c = c0 + lane;
    uint32_t* p = chunk_cnt + ((int64_t)t * nchunks + c) * T.nb + b;
    const uint32_t v = c < nchunks ? *p : 0u;
    const uint32_t inc = (uint32_t)warp_incl_scan((int)v);
    if (c < nchunks) *p = run + inc - v;
    run += __shfl_sync(FULL, inc, 31);
  }
  if (lane != 0) return;
  total[g] = run;
  const uint32_t nnew = run;
  const uint32_t len0 = min(T.len[g], (uint32_t)T.cap);
  uint32_t* ids = T.ids + g * T.cap;
  if (T.type == KL_BUCKET_FIFO) {
    const uint32_t room = nnew >= (uint32_t)T.cap ? 0u : (uint32_t)T.cap - nnew;
    const uint32_t keep = min(len0, room);
    const uint32_t drop_old = len0 - keep;
    for (uint32_t j = 0; j < keep; ++j) ids[j] = ids[drop_old + j];  // ascending: src >= dst
    basev[g] = keep;
    skipv[g] = nnew > (uint32_t)T.cap ? nnew - (uint32_t)T.cap : 0u;
    T.len[g] = min((uint32_t)T.cap, keep + nnew);
  } else {
    unsigned long long* tp = temp + g * T.cap;
    for (int j = 0; j < T.cap; ++j) tp[j] = (j < (int)len0) ? (unsigned long long)ids[j] : 0ull;
  }
}

// ---- insert pass 3: stable in-chunk ranks, then placement
__global__ void ins_place_kernel(DevTables T, const uint32_t* idsin, const uint16_t* bkt,
                                 int64_t bkt_ld, int n, const uint32_t* chunk_cnt, int nchunks,
                                 const uint32_t* basev, const uint32_t* skipv,
                                 unsigned long long* temp) {
  extern __shared__ uint32_t run[];  // [nb]
  const int t = blockIdx.y, c = blockIdx.x;
  const uint32_t* src = chunk_cnt + ((int64_t)t * nchunks + c) * T.nb;
  for (int b = threadIdx.x; b < T.nb; b += 32) run[b] = src[b];
  __syncwarp();
  const int i0 = c * INSERT_CHUNK, i1 = min(n, i0 + INSERT_CHUNK);
  for (int base = i0; base < i1; base += 32) {
    const int i = base + threadIdx.x;
    const bool valid = i < i1;
    const int b = valid ? (int)bkt[(int64_t)t * bkt_ld + i] : -1;
    const unsigned peers = __match_any_sync(FULL, b);
    uint32_t r = 0;
    if (valid) r = run[b] + __popc(peers & lanemask_lt());
    __syncwarp();
    if (valid && (int)threadIdx.x == __ffs(peers) - 1) run[b] += __popc(peers);
    __syncwarp();
    if (!valid) continue;
    const uint32_t id = idsin ? idsin[i] : (uint32_t)i;
    const int64_t g = (int64_t)t * T.nb + b;
    if (T.type == KL_BUCKET_FIFO) {
      const uint32_t sk = skipv[g];
      if (r >= sk) T.ids[g * T.cap + basev[g] + (r - sk)] = id;
    } else {
      const uint32_t len0 = min(T.len[g], (uint32_t)T.cap);
      const unsigned long long key = ((unsigned long long)(r + 1) << 32) | id;
      if (len0 + r < (uint32_t)T.cap) {
        atomicMax(&temp[g * T.cap + len0 + r], key);
      } else {
        const uint64_t count = T.cnt[g] + (uint64_t)r + 1;
        const uint64_t seed = count * 0x517cc1b727220a95ULL + (uint64_t)id;
        const uint64_t j = splitmix_mod(seed, count);
        if (j < (uint64_t)T.cap) {
          const uint64_t slot = splitmix_mod(seed + 1, (uint64_t)T.cap);
          atomicMax(&temp[g * T.cap + slot], key);
        }
      }
    }
  }
}

// ---- insert pass 4 (reservoir): unpack slots, update len and count
__global__ void ins_res_finish_kernel(DevTables T, const uint32_t* total,
                                      const unsigned long long* temp) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)T.L * T.nb) return;
  const uint32_t len0 = min(T.len[g], (uint32_t)T.cap);
  const uint32_t nl = min((uint32_t)T.cap, len0 + total[g]);
  for (uint32_t j = 0; j < nl; ++j) T.ids[g * T.cap + j] = (uint32_t)(temp[g * T.cap + j] & 0xffffffffu);
  T.len[g] = nl;
  T.cnt[g] += total[g];
}

__global__ void clear_kernel(DevTables T) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)T.L * T.nb) return;
  T.len[g] = 0;
  T.cnt[g] = 0;
}

// swap_remove of the first occurrence (fifo.rs:35-42, reservoir.rs:69-76)
__device__ __forceinline__ void bucket_remove(uint32_t* ids, uint32_t* len, int cap, uint32_t id) {
  const uint32_t n = min(*len, (uint32_t)cap);
  for (uint32_t p = 0; p < n; ++p) {
    if (ids[p] == id) {
      ids[p] = ids[n - 1];
      *len = n - 1;
      return;
    }
  }
}
// LshIndexTrait::remove (index.rs:278-280): every bucket, ids in order.
__global__ void remove_all_kernel(DevTables T, const uint32_t* ids, int n) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)T.L * T.nb) return;
  for (int i = 0; i < n; ++i) bucket_remove(T.ids + g * T.cap, T.len + g, T.cap, ids[i]);
}
// remove_with_weights (index.rs:271-276): one thread per table, ids in order.
__global__ void remove_hashed_kernel(DevTables T, const uint32_t* ids, const uint16_t* bkt,
                                     int64_t bkt_ld, int n) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T.L) return;
  for (int i = 0; i < n; ++i) {
    const int64_t g = (int64_t)t * T.nb + bkt[(int64_t)t * bkt_ld + i];
    bucket_remove(T.ids + g * T.cap, T.len + g, T.cap, ids[i]);
  }
}

// ---------------------------------------------------------------------------
// Probe.  One 512-thread block per query:
//  1. gather the ids of its L buckets into shared memory (M <= L*cap);
//  2. stable LSD radix sort by id (8-bit digits, per-warp histograms ranked
//     with __match_any_sync);
//  3. run-length encode -> (id, count) sorted by id: the union and the
//     per-table multiplicities of collect_counts (lsh/index.rs:219-234);
//  4. selection: TopK by (count desc, id asc) (sampling/topk.rs:19-34),
//     Threshold with its top-1 fallback (threshold.rs:20-43) or Vanilla;
//     empty selection -> all N (layer.rs:82-84); retain(id < N) (layer.rs:87).
// ---------------------------------------------------------------------------
constexpr int PB_NT = 512;
constexpr int PB_NW = PB_NT / 32;
constexpr int PB_MAXM = 16384;  // largest L*cap: 3 arrays of u32 => 192 KB of shared memory
constexpr int PB_MAXWORDS = 3 * PB_MAXM;  // dynamic shared words beyond ProbeSmem
constexpr int PB_SMALLN = 8192;            // neuron counts handled by the count-array path

struct ProbeSmem {
  uint32_t hist[PB_NW][256];
  int tmp[40];
  int lens_off[1025];
  int bsel[1024];  // bucket probed in each table
};

__device__ void probe_radix_pass(const uint32_t* in, uint32_t* out, int M, int shift,
                                 uint32_t (*hist)[256], int* tmp) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int seg = (int)round_up(ceil_div(M, PB_NW), 32);
  const int s0 = w * seg, s1 = min(M, s0 + seg);
  for (int b = l; b < 256; b += 32) hist[w][b] = 0;
  __syncwarp();
  for (int base = s0; base < s1; base += 32) {
    const int i = base + l;
    const bool valid = i < s1;
    const int dg = valid ? (int)((in[i] >> shift) & 255u) : -1;
    const unsigned peers = __match_any_sync(FULL, dg);
    if (valid && l == __ffs(peers) - 1) hist[w][dg] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // exclusive scan over (digit-major, warp-minor): thread d < 256 owns digit d
  int mytot = 0;
  if (threadIdx.x < 256) {
    const int dg = threadIdx.x;
    for (int ww = 0; ww < PB_NW; ++ww) {
      uint32_t v = hist[ww][dg];
      hist[ww][dg] = mytot;
      mytot += v;
    }
  }
  int total;
  const int excl = block_excl_scan<PB_NT>(threadIdx.x < 256 ? mytot : 0, tmp, &total);
  if (threadIdx.x < 256)
    for (int ww = 0; ww < PB_NW; ++ww) hist[ww][threadIdx.x] += excl;
  __syncthreads();
  for (int base = s0; base < s1; base += 32) {
    const int i = base + l;
    const bool valid = i < s1;
    const uint32_t key = valid ? in[i] : 0u;
    const int dg = valid ? (int)((key >> shift) & 255u) : -1;
    const unsigned peers = __match_any_sync(FULL, dg);
    uint32_t pos = 0;
    if (valid) pos = hist[w][dg] + __popc(peers & lanemask_lt());
    __syncwarp();
    if (valid && l == __ffs(peers) - 1) hist[w][dg] += __popc(peers);
    __syncwarp();
    if (valid) out[pos] = key;
  }
  __syncthreads();
}

// Mode 2 (every candidate selected, no counts) as its own kernel with a
// block size chosen from the bitmap's size: the union sorted by id is the set
// bits of a presence bitmap over the N neuron ids.  A shard's small bitmap
// (N/P ids) gets 128-thread blocks, so that more queries run per SM.
template <int NT>
__global__ void __launch_bounds__(NT) probe_bitmap_kernel(ProbeArgs a) {
  extern __shared__ __align__(16) uint32_t bm[];
  __shared__ int tmp[40];
  constexpr int NW = NT / 32;
  const int q = blockIdx.x;
  const DevTables& T = a.T;
  const int w_ = threadIdx.x >> 5, l_ = threadIdx.x & 31;
  const int nwd = (a.N + 31) >> 5;
  for (int i = threadIdx.x; i < nwd; i += NT) bm[i] = 0;
  __syncthreads();
  for (int t = w_; t < T.L; t += NW) {
    const int b = a.bkt[(int64_t)t * a.bkt_ld + q];
    const int n = (int)min(T.len[(int64_t)t * T.nb + b], (uint32_t)T.cap);
    const uint32_t* src = T.ids + ((int64_t)t * T.nb + b) * T.cap;
    for (int j0 = 0; j0 < n; j0 += 128) {  // 4 loads in flight per lane
      uint32_t id[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) id[u] = j0 + u * 32 + l_ < n ? src[j0 + u * 32 + l_] : 0xffffffffu;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (id[u] < (uint32_t)a.N) atomicOr(&bm[id[u] >> 5], 1u << (id[u] & 31));
    }
  }
  __syncthreads();
  const int wpt = (nwd + NT - 1) / NT;  // contiguous words per thread
  const int w0 = threadIdx.x * wpt, w1 = min(nwd, w0 + wpt);
  int c = 0;
  for (int i = w0; i < w1; ++i) c += __popc(bm[i]);
  int nsel;
  int pos = block_excl_scan<NT>(c, tmp, &nsel);
  uint32_t* out_ids = a.out_ids + (int64_t)q * a.out_stride;
  int nout;
  if (nsel == 0 && a.fallback) {
    // fallback: every neuron (layer.rs:82-84)
    nout = min(a.N, a.out_stride);
    if (a.N > a.out_stride && threadIdx.x == 0) atomicOr(a.err, DERR_CAPACITY);
    for (int j = threadIdx.x; j < nout; j += NT) out_ids[j] = (uint32_t)j;
  } else {
    for (int i = w0; i < w1; ++i) {
      uint32_t bits = bm[i];
      while (bits) {
        const int j = __ffs(bits) - 1;
        bits &= bits - 1;
        if (pos < a.out_stride) out_ids[pos] = (uint32_t)(i * 32 + j);
        ++pos;
      }
    }
    nout = min(nsel, a.out_stride);
    if (nsel > a.out_stride && threadIdx.x == 0) atomicOr(a.err, DERR_CAPACITY);
  }
  if (threadIdx.x == 0) {
    a.out_n[q] = nout;
    if (a.stat_active) atomicAdd(a.stat_active, (unsigned long long)nout);
  }
}

__global__ void __launch_bounds__(PB_NT) probe_kernel(ProbeArgs a) {
  extern __shared__ __align__(16) unsigned char dyn[];
  ProbeSmem& S = *reinterpret_cast<ProbeSmem*>(dyn);
  uint32_t* A = reinterpret_cast<uint32_t*>(dyn + sizeof(ProbeSmem));
  uint32_t* Bf = A + a.maxm;
  uint32_t* C = Bf + a.maxm;
  const int q = blockIdx.x;
  const DevTables& T = a.T;

  // 1. bucket sizes and offsets
  int myoff = 0, tot = 0;
  {
    // L <= 1024: two passes of the 512-thread scan
    int carry = 0;
    for (int t0 = 0; t0 < T.L; t0 += PB_NT) {
      const int t = t0 + threadIdx.x;
      int len = 0;
      if (t < T.L) {
        const int b = a.bkt[(int64_t)t * a.bkt_ld + q];
        S.bsel[t] = b;
        len = (int)min(T.len[(int64_t)t * T.nb + b], (uint32_t)T.cap);
      }
      int chunk_tot;
      myoff = block_excl_scan<PB_NT>(len, S.tmp, &chunk_tot);
      if (t < T.L) S.lens_off[t] = carry + myoff;
      carry += chunk_tot;
    }
    tot = carry;
    if (threadIdx.x == 0) S.lens_off[T.L] = tot;
    __syncthreads();
  }
  const int M = tot;
  const int w_ = threadIdx.x >> 5, l_ = threadIdx.x & 31;
  // mode 2 (every candidate selected) runs in probe_bitmap_kernel
  uint32_t* uid;
  uint32_t* ucnt;
  int U;
  if (a.mode == 1) {
    // Small N: per-id counts in shared memory, compacted in id order into
    // (uid, ucnt) -- the union and collect_counts multiplicities
    // (lsh/index.rs:219-234) without a sort.  Ids >= N are dropped before
    // selection; the network's own tables never hold them.
    // layout: uid = A, ucnt = Bf, selection flags C, counts after C (maxm >= N)
    uint32_t* cntv = C + a.maxm;
    uid = A;
    ucnt = Bf;
    for (int i = threadIdx.x; i < a.N; i += PB_NT) cntv[i] = 0;
    __syncthreads();
    for (int t = w_; t < T.L; t += PB_NW) {
      const int b = S.bsel[t];
      const uint32_t* src = T.ids + ((int64_t)t * T.nb + b) * T.cap;
      const int n = S.lens_off[t + 1] - S.lens_off[t];
      for (int j0 = 0; j0 < n; j0 += 128) {  // 4 loads in flight per lane
        uint32_t id[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) id[u] = j0 + u * 32 + l_ < n ? src[j0 + u * 32 + l_] : 0xffffffffu;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (id[u] < (uint32_t)a.N) atomicAdd(&cntv[id[u]], 1u);
      }
    }
    __syncthreads();
    const int ipt = (a.N + PB_NT - 1) / PB_NT;
    const int i0 = threadIdx.x * ipt, i1 = min(a.N, i0 + ipt);
    int c = 0;
    for (int i = i0; i < i1; ++i) c += cntv[i] != 0;
    int pos = block_excl_scan<PB_NT>(c, S.tmp, &U);
    for (int i = i0; i < i1; ++i)
      if (cntv[i]) {
        uid[pos] = (uint32_t)i;
        ucnt[pos] = cntv[i];
        ++pos;
      }
    __syncthreads();
  } else {
    // 2. gather: warp w copies tables w, w+16, ...
    {
      const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
      for (int t = w; t < T.L; t += PB_NW) {
        const int b = S.bsel[t];
        const uint32_t* src = T.ids + ((int64_t)t * T.nb + b) * T.cap;
        const int o = S.lens_off[t], n = S.lens_off[t + 1] - o;
        for (int j = l; j < n; j += 32) A[o + j] = src[j];
      }
    }
    __syncthreads();
    // 3. radix sort by id
    uint32_t* cur = A;
    uint32_t* oth = Bf;
    for (int shift = 0; shift < a.id_bits; shift += 8) {
      probe_radix_pass(cur, oth, M, shift, S.hist, S.tmp);
      uint32_t* x = cur;
      cur = oth;
      oth = x;
    }
    // 4. run-length encode: heads -> unique ids (oth) and head positions (C)
    const int IPT = (int)ceil_div(M, PB_NT);
    int nheads = 0;
    for (int j = 0; j < IPT; ++j) {
      const int i = threadIdx.x * IPT + j;
      if (i < M && (i == 0 || cur[i] != cur[i - 1])) ++nheads;
    }
    int hoff = block_excl_scan<PB_NT>(nheads, S.tmp, &U);
    for (int j = 0; j < IPT; ++j) {
      const int i = threadIdx.x * IPT + j;
      if (i < M && (i == 0 || cur[i] != cur[i - 1])) {
        oth[hoff] = cur[i];
        C[hoff] = (uint32_t)i;
        ++hoff;
      }
    }
    __syncthreads();
    // counts into `cur` (no longer needed): count[u] = pos[u+1] - pos[u]
    for (int u = threadIdx.x; u < U; u += PB_NT) {
      const uint32_t nxt = (u + 1 < U) ? C[u + 1] : (uint32_t)M;
      cur[u] = nxt - C[u];
    }
    __syncthreads();
    uid = oth;
    ucnt = cur;
  }
  // 5. selection -> flags in C (1 = selected)
  const bool net = a.N > 0;
  int cstar = -1, need = 0;  // TopK threshold
  bool all = true;
  int thr_mode = 0;          // 1 = count >= threshold; 2 = single best
  uint32_t best_count = 0;
  if (net && U > 0) {
    if (a.sampling == KL_SAMPLING_TOPK && a.top_k < U) {
      all = false;
      // largest c with #(count >= c) >= k
      int maxc = 0;
      for (int u = threadIdx.x; u < U; u += PB_NT) maxc = max(maxc, (int)ucnt[u]);
      maxc = block_max<PB_NT>(maxc, S.tmp);
      int lo = 0, hi = maxc;  // #(>= lo) >= k holds for lo = 0 (k < U)
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        int c = 0;
        for (int u = threadIdx.x; u < U; u += PB_NT) c += (int)ucnt[u] >= mid;
        c = block_sum<PB_NT>(c, S.tmp);
        if (c >= a.top_k) lo = mid;
        else hi = mid - 1;
      }
      cstar = lo;
      int gt = 0;
      for (int u = threadIdx.x; u < U; u += PB_NT) gt += (int)ucnt[u] > cstar;
      gt = block_sum<PB_NT>(gt, S.tmp);
      need = a.top_k - gt;
    } else if (a.sampling == KL_SAMPLING_THRESHOLD) {
      all = false;
      int pass = 0, maxc = 0;
      for (int u = threadIdx.x; u < U; u += PB_NT) {
        pass += (int)ucnt[u] >= a.threshold;
        maxc = max(maxc, (int)ucnt[u]);
      }
      pass = block_sum<PB_NT>(pass, S.tmp);
      maxc = block_max<PB_NT>(maxc, S.tmp);
      thr_mode = pass > 0 ? 1 : 2;
      best_count = (uint32_t)maxc;
    }
  }
  // flags (blocked arrangement so that ranks follow id order)
  const int UPT = (int)ceil_div(U, PB_NT);
  int eq_local = 0;
  for (int j = 0; j < UPT; ++j) {
    const int u = threadIdx.x * UPT + j;
    if (u < U && cstar >= 0 && (int)ucnt[u] == cstar) ++eq_local;
  }
  int eq_tot;
  int eq_rank = block_excl_scan<PB_NT>(eq_local, S.tmp, &eq_tot);
  int sel_local = 0;
  int first_best = INT32_MAX;
  for (int j = 0; j < UPT; ++j) {
    const int u = threadIdx.x * UPT + j;
    if (u >= U) break;
    bool s = true;
    if (!all) {
      if (cstar >= 0) {
        const int c = (int)ucnt[u];
        if (c > cstar) s = true;
        else if (c == cstar) s = (eq_rank++ < need);
        else s = false;
      } else if (thr_mode == 1) {
        s = (int)ucnt[u] >= a.threshold;
      } else {
        s = false;
        if (ucnt[u] == best_count) first_best = min(first_best, u);
      }
    }
    C[u] = s ? 1u : 0u;
    sel_local += s;
  }
  if (!all && cstar < 0 && thr_mode == 2) {
    // single best: lowest id among the max count = first in id order
    int fb = first_best == INT32_MAX ? INT32_MAX : first_best;
    // block min via max of negatives
    fb = -block_max<PB_NT>(fb == INT32_MAX ? -INT32_MAX : -fb, S.tmp);
    __syncthreads();
    for (int u = threadIdx.x; u < U; u += PB_NT) C[u] = (u == fb) ? 1u : 0u;
    __syncthreads();
    sel_local = 0;
    for (int j = 0; j < UPT; ++j) {
      const int u = threadIdx.x * UPT + j;
      if (u < U) sel_local += C[u];
    }
  }
  __syncthreads();
  int nsel;
  int sel_off = block_excl_scan<PB_NT>(sel_local, S.tmp, &nsel);
  uint32_t* out_ids = a.out_ids + (int64_t)q * a.out_stride;
  uint32_t* out_cnt = a.out_counts ? a.out_counts + (int64_t)q * a.out_stride : nullptr;
  int nout = 0;
  if (net && nsel == 0 && a.fallback) {
    // fallback: every neuron (layer.rs:82-84)
    nout = a.N;
    if (nout > a.out_stride) {
      if (threadIdx.x == 0) atomicOr(a.err, DERR_CAPACITY);
      nout = a.out_stride;
    }
    for (int j = threadIdx.x; j < nout; j += PB_NT) {
      out_ids[j] = (uint32_t)j;
      if (out_cnt) out_cnt[j] = 0;
    }
  } else {
    for (int j = 0; j < UPT; ++j) {
      const int u = threadIdx.x * UPT + j;
      if (u < U && C[u]) {
        if (sel_off < a.out_stride) {
          out_ids[sel_off] = uid[u];
          if (out_cnt) out_cnt[sel_off] = ucnt[u];
        }
        ++sel_off;
      }
    }
    nout = nsel;
    if (nout > a.out_stride) {
      if (threadIdx.x == 0) atomicOr(a.err, DERR_CAPACITY);
      nout = a.out_stride;
    }
    if (net) {
      // retain(id < N): ids are sorted, so out-of-range ones form the tail
      __syncthreads();
      int bad = 0;
      for (int j = threadIdx.x; j < nout; j += PB_NT) bad += out_ids[j] >= (uint32_t)a.N;
      bad = block_sum<PB_NT>(bad, S.tmp);
      nout -= bad;
    }
  }
  if (threadIdx.x == 0) {
    a.out_n[q] = nout;
    if (a.stat_active) atomicAdd(a.stat_active, (unsigned long long)nout);
  }
}

// ---- scan of per-query counts (single block per 1M entries chunk) ----
__global__ void scan_kernel(const int32_t* counts, int32_t* offs, int n) {
  using BS = cub::BlockScan<int, 1024>;
  __shared__ typename BS::TempStorage ts;
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < n; base += 1024) {
    const int i = base + threadIdx.x;
    int v = i < n ? counts[i] : 0, ex, agg;
    BS(ts).ExclusiveSum(v, ex, agg);
    if (i < n) offs[i] = carry + ex;
    __syncthreads();
    if (threadIdx.x == 0) carry += agg;
    __syncthreads();
  }
  if (threadIdx.x == 0) offs[n] = carry;
}

__global__ void compact_kernel(const uint32_t* ids, const uint32_t* counts, int stride,
                               const int32_t* offs, int nq, uint32_t* out_ids,
                               uint32_t* out_counts, int32_t capacity, int32_t* overflow,
                               int* err) {
  const int q = blockIdx.x;
  const int o = offs[q], n = offs[q + 1] - o;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const int64_t dst = (int64_t)o + j;
    if (dst < capacity) {
      out_ids[dst] = ids[(int64_t)q * stride + j];
      if (out_counts && counts) out_counts[dst] = counts[(int64_t)q * stride + j];
    } else {
      if (overflow) *overflow = 1;
      atomicOr(err, DERR_CAPACITY);
    }
  }
}

}  // namespace

size_t insert_scratch_bytes(const DevTables& T, int n) {
  const int64_t nchunks = ceil_div(max(n, 1), INSERT_CHUNK);
  const int64_t LB = (int64_t)T.L * T.nb;
  size_t b = 0;
  b += round_up(LB * nchunks * 4, 256);
  b += 3 * round_up(LB * 4, 256);
  b += round_up(LB * T.cap * 8, 256);
  return b;
}
void carve_insert_scratch(const DevTables& T, int n, void* base, InsertScratch* s) {
  const int64_t nchunks = ceil_div(max(n, 1), INSERT_CHUNK);
  const int64_t LB = (int64_t)T.L * T.nb;
  char* p = static_cast<char*>(base);
  s->chunk_cnt = reinterpret_cast<uint32_t*>(p);
  p += round_up(LB * nchunks * 4, 256);
  s->total = reinterpret_cast<uint32_t*>(p);
  p += round_up(LB * 4, 256);
  s->base = reinterpret_cast<uint32_t*>(p);
  p += round_up(LB * 4, 256);
  s->skip = reinterpret_cast<uint32_t*>(p);
  p += round_up(LB * 4, 256);
  s->temp = reinterpret_cast<unsigned long long*>(p);
}

void launch_tables_insert(const DevTables& T, const uint32_t* ids, const uint16_t* bkt,
                          int64_t bkt_ld, int n, const InsertScratch& s, int* err,
                          cudaStream_t st) {
  (void)err;
  if (n <= 0) return;
  const int nchunks = (int)ceil_div(n, INSERT_CHUNK);
  const int64_t LB = (int64_t)T.L * T.nb;
  dim3 g(nchunks, T.L);
  const size_t sm = (size_t)T.nb * 4;
  ins_count_kernel<<<g, 32, sm, st>>>(T, bkt, bkt_ld, n, s.chunk_cnt, nchunks);
  count_launch();
  ins_plan_kernel<<<(unsigned)ceil_div(LB * 32, 256), 256, 0, st>>>(T, s.chunk_cnt, nchunks, s.total,
                                                               s.base, s.skip, s.temp);
  count_launch();
  ins_place_kernel<<<g, 32, sm, st>>>(T, ids, bkt, bkt_ld, n, s.chunk_cnt, nchunks, s.base,
                                      s.skip, s.temp);
  count_launch();
  if (T.type == KL_BUCKET_RESERVOIR)
    ins_res_finish_kernel<<<(unsigned)ceil_div(LB, 256), 256, 0, st>>>(T, s.total, s.temp);
  count_launch();
}

void launch_tables_clear(const DevTables& T, cudaStream_t st) {
  const int64_t LB = (int64_t)T.L * T.nb;
  clear_kernel<<<(unsigned)ceil_div(LB, 256), 256, 0, st>>>(T);
  count_launch();
}
void launch_tables_remove(const DevTables& T, const uint32_t* ids, int n, cudaStream_t st) {
  if (n <= 0) return;
  const int64_t LB = (int64_t)T.L * T.nb;
  remove_all_kernel<<<(unsigned)ceil_div(LB, 128), 128, 0, st>>>(T, ids, n);
  count_launch();
}
void launch_tables_remove_hashed(const DevTables& T, const uint32_t* ids, const uint16_t* bkt,
                                 int64_t bkt_ld, int n, cudaStream_t st) {
  if (n <= 0) return;
  remove_hashed_kernel<<<(unsigned)ceil_div(T.L, 64), 64, 0, st>>>(T, ids, bkt, bkt_ld, n);
  count_launch();
}

// ---------------------------------------------------------------------------
// BOLT sparse inference (crates/klearu-bolt/src/sparse_inference.rs:32-106):
// per input, the index's candidates with their table counts (sorted by id),
// ordered by count descending (ties by id ascending: a stable sort of the
// id-sorted list; the reference's ties follow HashMap order), the first
// effective_k kept, and for each kept neuron id < N the activation
// sum_j x[j] * W[id][j] (sequential f32, the reference's order) + bias[id],
// ReLU'd when `relu`.  One 512-thread block per input: the (count, position)
// keys go through one or two stable radix passes on the count digits; the dot
// products run one thread per kept neuron over x staged in shared memory.
// ---------------------------------------------------------------------------
template <class W>
__global__ void __launch_bounds__(PB_NT) bolt_kernel(BoltArgs a) {
  extern __shared__ __align__(16) unsigned char dyn[];
  ProbeSmem& S = *reinterpret_cast<ProbeSmem*>(dyn);
  float* xs = reinterpret_cast<float*>(dyn + sizeof(ProbeSmem));
  uint32_t* A = reinterpret_cast<uint32_t*>(xs + round_up(a.d, 4));
  uint32_t* Bf = A + a.maxm;
  const int q = blockIdx.x;
  const int M = min(a.cand_n[q], a.maxm);
  const uint32_t* ids = a.cand_ids + (int64_t)q * a.cand_stride;
  const uint32_t* cnt = a.cand_cnt + (int64_t)q * a.cand_stride;
  for (int j = threadIdx.x; j < a.d; j += PB_NT) xs[j] = a.X[(int64_t)q * a.ldx + j];
  // key: (L - count) above the 14-bit position, so an LSD sort of the count
  // digits orders by count descending and keeps id order among equal counts
  for (int i = threadIdx.x; i < M; i += PB_NT) {
    const uint32_t c = min(cnt[i], (uint32_t)a.L);
    A[i] = ((uint32_t)(a.L - c) << 14) | (uint32_t)i;
  }
  __syncthreads();
  uint32_t* cur = A;
  uint32_t* oth = Bf;
  for (int shift = 14; shift < 14 + a.count_bits; shift += 8) {
    probe_radix_pass(cur, oth, M, shift, S.hist, S.tmp);
    uint32_t* t = cur;
    cur = oth;
    oth = t;
  }
  const int K = min(M, a.k);
  // kept neurons with weights (id < N), compacted in order (neurons without
  // weights are skipped after the truncation, as `weights.find` does)
  const int IPT = (int)ceil_div(K, PB_NT);
  int mine = 0;
  for (int j = 0; j < IPT; ++j) {
    const int r = threadIdx.x * IPT + j;
    if (r < K && ids[cur[r] & 0x3FFFu] < (uint32_t)a.N) ++mine;
  }
  int total;
  int pos = block_excl_scan<PB_NT>(mine, S.tmp, &total);
  uint32_t* out_ids = a.out_ids + (int64_t)q * a.out_stride;
  float* out_act = a.out_act + (int64_t)q * a.out_stride;
  const W* Wp = static_cast<const W*>(a.W);
  for (int j = 0; j < IPT; ++j) {
    const int r = threadIdx.x * IPT + j;
    if (r >= K) break;
    const uint32_t id = ids[cur[r] & 0x3FFFu];
    if (id >= (uint32_t)a.N) continue;
    if (pos < a.out_stride) {
      const W* row = Wp + (int64_t)id * a.ldw;
      float acc = 0.0f;
      for (int e = 0; e < a.d; ++e) acc = __fadd_rn(acc, __fmul_rn(xs[e], to_f(row[e])));
      float v = __fadd_rn(acc, a.bias ? a.bias[id] : 0.0f);
      if (a.relu) v = fmaxf(v, 0.0f);
      out_ids[pos] = id;
      out_act[pos] = v;
    }
    ++pos;
  }
  if (threadIdx.x == 0) {
    a.out_n[q] = min(total, a.out_stride);
    if (total > a.out_stride) atomicOr(a.err, DERR_CAPACITY);
  }
}

void launch_bolt(const BoltArgs& a0, cudaStream_t st) {
  if (a0.nq <= 0) return;
  BoltArgs a = a0;
  a.maxm = (int)round_up(std::max(a.cand_stride, 1), 32);
  a.count_bits = 1;
  while ((1 << a.count_bits) <= a.L) ++a.count_bits;
  const size_t sm = sizeof(ProbeSmem) + (size_t)round_up(a.d, 4) * 4 + (size_t)2 * a.maxm * 4;
  static OncePerDevice attr;
  attr([&] {
    cudaFuncSetAttribute(bolt_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(bolt_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (a.wdtype == KL_DTYPE_BF16) bolt_kernel<__nv_bfloat16><<<a.nq, PB_NT, sm, st>>>(a);
  else bolt_kernel<float><<<a.nq, PB_NT, sm, st>>>(a);
  count_launch();
}
size_t bolt_smem_bytes(int d, int cand_stride) {
  return sizeof(ProbeSmem) + (size_t)round_up(d, 4) * 4 + (size_t)2 * round_up(std::max(cand_stride, 1), 32) * 4;
}

int probe_max_items() { return PB_MAXM; }

void launch_probe(const ProbeArgs& a, cudaStream_t st) {
  if (a.nq <= 0) return;
  ProbeArgs b = a;
  const int M = max(1, a.T.L * a.T.cap);
  b.maxm = (int)round_up(M, 32);
  size_t words = 3 * (size_t)b.maxm;
  b.mode = 0;
  if (a.N > 0) {
    const bool all = a.sampling == KL_SAMPLING_VANILLA || (a.sampling == KL_SAMPLING_TOPK && a.top_k >= M);
    if (all && !a.out_counts && a.N > PB_SMALLN && (size_t)(a.N + 31) / 32 <= (size_t)PB_MAXWORDS) {
      b.mode = 2;
      words = std::max(words, (size_t)(a.N + 31) / 32);
    } else if (a.N <= PB_SMALLN) {
      // uid, ucnt, selection flags and counts: [N] each
      b.mode = 1;
      b.maxm = (int)round_up(a.N, 32);
      words = 4 * (size_t)b.maxm;
    }
  }
  if (b.mode == 2) {
    const int nwd = (a.N + 31) / 32;
    const size_t bsm = (size_t)nwd * 4;
    static OncePerDevice battr;
    battr([&] {
      cudaFuncSetAttribute(probe_bitmap_kernel<1024>, cudaFuncAttributeMaxDynamicSharedMemorySize, PB_MAXWORDS * 4);
      cudaFuncSetAttribute(probe_bitmap_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, PB_MAXWORDS * 4);
      cudaFuncSetAttribute(probe_bitmap_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, PB_MAXWORDS * 4);
    });
    // threads per query grow with the bitmap (words cleared and scanned per thread)
    if (nwd >= 16384) probe_bitmap_kernel<1024><<<a.nq, 1024, bsm, st>>>(b);
    else if (nwd >= 8192) probe_bitmap_kernel<512><<<a.nq, 512, bsm, st>>>(b);
    else probe_bitmap_kernel<128><<<a.nq, 128, bsm, st>>>(b);
    count_launch();
    return;
  }
  const size_t sm = sizeof(ProbeSmem) + words * 4;
  static OncePerDevice attr;
  attr([&] {
    cudaFuncSetAttribute(probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)(sizeof(ProbeSmem) + (size_t)PB_MAXWORDS * 4));
  });
  probe_kernel<<<a.nq, PB_NT, sm, st>>>(b);
  count_launch();
}

size_t scan_scratch_bytes(int) { return 0; }
void launch_scan(const int32_t* counts, int32_t* offsets, int n, void*, cudaStream_t st) {
  scan_kernel<<<1, 1024, 0, st>>>(counts, offsets, n);
  count_launch();
}
void launch_compact(const uint32_t* ids, const uint32_t* counts, int stride, const int32_t* offs,
                    int nq, uint32_t* out_ids, uint32_t* out_counts, int32_t capacity,
                    int32_t* overflow, int* err, cudaStream_t st) {
  if (nq <= 0) return;
  compact_kernel<<<nq, 256, 0, st>>>(ids, counts, stride, offs, nq, out_ids, out_counts, capacity,
                                     overflow, err);
  count_launch();
}

}  // namespace kl
