// hash.cu -- batched LSH hash kernels for all five klearu hash families.
//
// Every kernel reproduces the reference's f32 arithmetic exactly:
//  * SimHash / SRP (crates/klearu-core/src/hash/simhash.rs:75-126,
//    srp.rs:93-162): each projection is a sequential f32 sum over the input in
//    index order; a plane entry p in {-1,0,+1} contributes fma(p, x, sum),
//    which rounds exactly like the reference's `sum += x` / `sum -= x` (p*x is
//    exact) and leaves the sum unchanged when p == 0 (up to the sign of a zero,
//    which the `>= 0` test does not see).  SRP is stored as a dense ternary
//    plane matrix, so it shares the SimHash kernels.
//  * WTA / DWTA (wta.rs:91-125, dwta.rs:86-164): first-max argmax over each
//    window, strict `>` from -inf.
//  * MinHash / DOPH (minhash.rs:67-153): per-bin minimum of permuted indices,
//    circular densification, polynomial combine.
#include <algorithm>

#include "engine.h"

namespace kl {
namespace {

template <class T>
__device__ __forceinline__ float ldx(const void* X, int64_t off) {
  return to_f(static_cast<const T*>(X)[off]);
}
__device__ __forceinline__ float ldx_dt(const void* X, int dtype, int64_t off) {
  return dtype == KL_DTYPE_BF16 ? ldx<__nv_bfloat16>(X, off) : ldx<float>(X, off);
}

__device__ __forceinline__ void write_out(const HashOut& o, int L, int i, int t, uint64_t code,
                                          float mn, bool has_mn) {
  const int64_t q = (int64_t)i * L + t;
  if (o.codes) o.codes[q] = code;
  if (o.min_abs && has_mn) o.min_abs[q] = mn;
  if (o.bkt) o.bkt[(int64_t)t * o.bkt_ld + i] = (uint16_t)(code & o.nb_mask);
}

// Stage a 32-row x `tw`-column tile of dense rows into shared memory as f32,
// dst[rr * rs + dd * ds].  Loads are issued STG_U at a time before their
// stores, so a thread keeps STG_U global loads in flight instead of one.
constexpr int STG_U = 8;
__device__ __forceinline__ void stage_rows(const DenseIn& in, int row0, int d0, int tw, float* dst, int rs, int ds) {
  const bool rowfast = in.ld_elem != 1;  // consecutive rows are adjacent in memory
  const int total = 32 * tw;
  for (int base = threadIdx.x; base < total; base += blockDim.x * STG_U) {
    float v[STG_U];
    int rr[STG_U], dd[STG_U];
#pragma unroll
    for (int u = 0; u < STG_U; ++u) {
      const int idx = base + u * blockDim.x;
      if (rowfast) { rr[u] = idx & 31; dd[u] = idx >> 5; }
      else { rr[u] = idx / tw; dd[u] = idx - rr[u] * tw; }
      v[u] = 0.0f;
      if (idx < total && row0 + rr[u] < in.n)
        v[u] = ldx_dt(in.X, in.dtype, (int64_t)(row0 + rr[u]) * in.ld_row + (int64_t)(d0 + dd[u]) * in.ld_elem);
    }
#pragma unroll
    for (int u = 0; u < STG_U; ++u)
      if (base + u * blockDim.x < total) dst[rr[u] * rs + dd[u] * ds] = v[u];
  }
}

// ---------------------------------------------------------------------------
// Projection hashing of dense rows over the planes' non-zero lists.  The
// reference's dot_ternary_dense (simhash.rs:75-85) adds x where the plane is
// +1, subtracts it where it is -1 and skips zeros; walking each projection's
// sorted non-zero list does exactly that, in the same order, with a third of
// the work (acc + (-x) is IEEE-identical to acc - x).  Block = 32 rows (one
// lane each) x TT*K projections (one warp each); the rows are staged in
// tiles of PL_T dimensions as xs[dim][row]:
//  * FMB (rows adjacent in memory, bf16 -- the feature-major layer-0 weights):
//    raw bf16 tiles copied with cp.async into two buffers, the next tile in
//    flight while the warps walk the current one;
//  * otherwise: converted to f32 by stage_rows (pitch 33).
// Each warp walks its list in windows of 32 entries (one per lane, broadcast
// by shuffle), prefetched two windows ahead.
// ---------------------------------------------------------------------------
constexpr int PL_PITCH = 33;

template <bool FMB>
__global__ void proj_list_kernel(DevHash h, DenseIn in, HashOut out, int TT) {
  extern __shared__ __align__(16) unsigned char dyn[];
  const int tdim = min(h.d, PL_T);
  // FMB: two bf16 buffers [tdim][32]; else one f32 buffer [tdim][PL_PITCH]
  const size_t xbytes = FMB ? (size_t)2 * tdim * 32 * 2 : (size_t)tdim * PL_PITCH * 4;
  float* sv = reinterpret_cast<float*>(dyn + round_up((int64_t)xbytes, 16));  // [TT*K][32]
  const int K = h.k;
  const int r = threadIdx.x & 31;
  const int q = threadIdx.x >> 5;
  const int tt = q / K, b = q % K;
  const int t = blockIdx.y * TT + tt;
  const int row0 = blockIdx.x * 32;
  const bool active = t < h.L;
  const uint32_t* toff = h.poff + (size_t)(active ? t * K + b : 0) * (h.nt + 1);
  auto stage_async = [&](int ti, int bf) {  // FMB only
    const int d0 = ti * PL_T, tw = min(PL_T, h.d - d0);
    unsigned char* dst = dyn + (size_t)bf * tdim * 64;
    const unsigned char* src = static_cast<const unsigned char*>(in.X);
    for (int c = threadIdx.x; c < tw * 4; c += blockDim.x) {
      const int dd = c >> 2, part = c & 3;  // 4 x 16 B = 32 bf16 rows per dimension
      const int rr = row0 + part * 8;
      if (rr + 8 <= in.ld_elem)
        cp_async16(dst + dd * 64 + part * 16, src + ((int64_t)(d0 + dd) * in.ld_elem + rr) * 2);
      else
        *reinterpret_cast<uint4*>(dst + dd * 64 + part * 16) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
  };
  uint32_t pos = toff[0];
  uint32_t wb = pos;
  uint32_t c0 = h.plist[wb + r], c1 = h.plist[wb + 32 + r], c2 = h.plist[wb + 64 + r];
  float acc = 0.0f;
  if (FMB) stage_async(0, 0);
  for (int ti = 0; ti < h.nt; ++ti) {
    const int d0 = ti * PL_T;
    const uint32_t E = active ? toff[ti + 1] : pos;
    if (FMB) {
      if (ti + 1 < h.nt) {
        stage_async(ti + 1, (ti + 1) & 1);
        cp_async_wait_group<1>();
      } else {
        cp_async_wait_group<0>();
      }
    } else {
      stage_rows(in, row0, d0, min(PL_T, h.d - d0), reinterpret_cast<float*>(dyn), 1, PL_PITCH);
    }
    __syncthreads();
    const uint16_t* xb = reinterpret_cast<const uint16_t*>(dyn + (size_t)(ti & 1) * tdim * 64) + r;
    const float* xf = reinterpret_cast<const float*>(dyn) + r;
    while (pos < E) {
      const int u0 = (int)(pos - wb);
      const int u1 = (int)min(32u, E - wb);
#pragma unroll 4
      for (int u = u0; u < u1; ++u) {
        const uint32_t ent = __shfl_sync(FULL, c0, u);
        const uint32_t dd = ent & 0x7fffu;
        const float x = FMB ? __uint_as_float((uint32_t)xb[dd * 32] << 16) : xf[dd * PL_PITCH];
        acc = __fadd_rn(acc, __int_as_float(__float_as_int(x) ^ (int)((ent & 0x8000u) << 16)));
      }
      pos = wb + (uint32_t)u1;
      if (u1 == 32) {
        c0 = c1;
        c1 = c2;
        wb += 32;
        c2 = h.plist[wb + 64 + r];
      }
    }
    __syncthreads();
  }
  const int nthr = blockDim.x;
  sv[q * 32 + r] = acc;
  __syncthreads();
  const int ncomb = TT * 32;
  for (int c = threadIdx.x; c < ncomb; c += nthr) {
    const int ct = c / 32, cr = c % 32;
    const int tab = blockIdx.y * TT + ct, i = row0 + cr;
    if (tab >= h.L || i >= in.n) continue;
    uint64_t code = 0;
    float mn = __int_as_float(0x7f800000);
    for (int bb = 0; bb < K; ++bb) {
      const float v = sv[(ct * K + bb) * 32 + cr];
      if (v >= 0.0f) code |= 1ULL << bb;
      mn = fminf(mn, fabsf(v));
    }
    write_out(out, h.L, i, tab, code, mn, true);
  }
}

// ---------------------------------------------------------------------------
// WTA / DWTA over dense rows, tiled: 32 rows staged as f32 in shared memory
// (pitch d+1), one warp per table at a time, one lane per row.  When only the
// bucket number is wanted (out.codes == NULL), only the windows whose bits
// survive `code & nb_mask` are evaluated (K=8, w=8, 256 buckets: 3 of 8).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) wta_tile_kernel(DevHash h, DenseIn in, HashOut out, int nwin) {
  extern __shared__ __align__(16) unsigned char dyn[];
  float* xs = reinterpret_cast<float*>(dyn);  // [32][d+1]
  const int pitch = h.d + 1;
  const int row0 = blockIdx.x * 32;
  const int nr = min(32, in.n - row0);
  stage_rows(in, row0, 0, h.d, xs, pitch, 1);
  __syncthreads();
  const int w = threadIdx.x >> 5, r = threadIdx.x & 31;
  const float* xr = xs + r * pitch;
  // tables of this block: [blockIdx.y * tpb, ...), one warp per table at a time
  const int tpb = (h.L + gridDim.y - 1) / gridDim.y;
  const int t0 = blockIdx.y * tpb, t1 = min(h.L, t0 + tpb);
  for (int t = t0 + w; t < t1; t += blockDim.x >> 5) {
    uint64_t code = 0;
    int shift = 0;
    for (int kk = 0; kk < nwin; ++kk) {
      const uint32_t* win = h.windows + ((int64_t)t * h.k + kk) * h.w;
      int best_pos = 0;
      float best = __int_as_float(0xff800000);
      for (int p = 0; p < h.w; ++p) {
        const float v = xr[__ldg(win + p)];
        if (v > best) {
          best = v;
          best_pos = p;
        }
      }
      code |= (uint64_t)best_pos << shift;
      shift += h.bpw;
    }
    if (r < nr) write_out(out, h.L, row0 + r, t, code, 0.0f, false);
  }
}

// Projection hashing of CSR rows: one block per row, one thread per projection.
// Chunks of PS_CH nonzeros: the plane bytes of their columns are staged in
// shared memory first, then each projection sums its chain in index order.
constexpr int PS_CH = 64;
__global__ void proj_sparse_kernel(DevHash h, SparseIn in, HashOut out) {
  extern __shared__ unsigned char dyn[];
  float* sv = reinterpret_cast<float*>(dyn);  // [LK]
  __shared__ uint32_t sidx[PS_CH];
  __shared__ float sval[PS_CH];
  uint32_t* spl = reinterpret_cast<uint32_t*>(dyn) + round_up(h.LK, 4);  // [PS_CH][lkpad] plane bytes
  const int i = blockIdx.x;
  const int tb = threadIdx.x;
  const int beg = in.rowptr[i], end = in.rowptr[i + 1];
  float acc = 0.0f;
  for (int c0 = beg; c0 < end; c0 += PS_CH) {
    const int m = min(PS_CH, end - c0);
    for (int e = threadIdx.x; e < m; e += blockDim.x) {
      sidx[e] = in.idx[c0 + e];
      sval[e] = in.val[c0 + e];
    }
    __syncthreads();
    // stage the plane bytes of this chunk's columns ([m][lkpad] int8, one
    // independent 4-byte load per thread at a time), then walk them in order
    const int wpc = h.lkpad / 4;  // 32-bit words per column
    for (int q0 = threadIdx.x; q0 < m * wpc; q0 += 4 * blockDim.x) {
      uint32_t v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = q0 + u * blockDim.x;
        v[u] = 0u;
        if (q < m * wpc) {
          const int e = q / wpc, wq = q - e * wpc;
          const uint32_t col = sidx[e];
          if (col < (uint32_t)h.d) v[u] = reinterpret_cast<const uint32_t*>(h.planesT + (int64_t)col * h.lkpad)[wq];
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (q0 + u * blockDim.x < m * wpc) spl[q0 + u * blockDim.x] = v[u];
    }
    __syncthreads();
    if (tb < h.LK) {
      const int8_t* pl = reinterpret_cast<const int8_t*>(spl);
      for (int e = 0; e < m; ++e) acc = __fmaf_rn((float)pl[e * h.lkpad + tb], sval[e], acc);
    }
    __syncthreads();
  }
  if (tb < h.LK) sv[tb] = acc;
  __syncthreads();
  for (int t = threadIdx.x; t < h.L; t += blockDim.x) {
    uint64_t code = 0;
    float mn = __int_as_float(0x7f800000);
    for (int b = 0; b < h.k; ++b) {
      float v = sv[t * h.k + b];
      if (v >= 0.0f) code |= 1ULL << b;
      mn = fminf(mn, fabsf(v));
    }
    write_out(out, h.L, i, t, code, mn, true);
  }
}

// WTA / DWTA over dense rows: thread per (row, table).
__global__ void wta_dense_kernel(DevHash h, DenseIn in, HashOut out) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)in.n * h.L) return;
  const int i = (int)(g / h.L), t = (int)(g % h.L);
  const int64_t rb = (int64_t)i * in.ld_row;
  uint64_t code = 0;
  int shift = 0;
  for (int kk = 0; kk < h.k; ++kk) {
    const uint32_t* win = h.windows + ((int64_t)t * h.k + kk) * h.w;
    int best_pos = 0;
    float best = __int_as_float(0xff800000);
    for (int p = 0; p < h.w; ++p) {
      float v = ldx_dt(in.X, in.dtype, rb + (int64_t)win[p] * in.ld_elem);
      if (v > best) {
        best = v;
        best_pos = p;
      }
    }
    code |= (uint64_t)best_pos << shift;
    shift += h.bpw;
  }
  write_out(out, h.L, i, t, code, 0.0f, false);
}

__device__ __forceinline__ int csr_find(const uint32_t* idx, int beg, int end, uint32_t key) {
  int lo = beg, hi = end;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (idx[mid] < key) lo = mid + 1;
    else hi = mid;
  }
  return (lo < end && idx[lo] == key) ? lo : -1;
}

// WTA (to_dense semantics, wta.rs:115-118) and DWTA (argmax_sparse with
// fallback, dwta.rs:104-137) over CSR rows: thread per (row, table).
__global__ void wta_sparse_kernel(DevHash h, SparseIn in, HashOut out) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)in.n * h.L) return;
  const int i = (int)(g / h.L), t = (int)(g % h.L);
  const int beg = in.rowptr[i], end = in.rowptr[i + 1];
  const bool dwta = h.kind == KL_HASH_DWTA;
  uint64_t code = 0;
  int shift = 0;
  for (int kk = 0; kk < h.k; ++kk) {
    const uint32_t* win = h.windows + ((int64_t)t * h.k + kk) * h.w;
    int best_pos = dwta ? -1 : 0;
    float best = __int_as_float(0xff800000);
    for (int p = 0; p < h.w; ++p) {
      int pos = csr_find(in.idx, beg, end, win[p]);
      float v;
      if (pos >= 0) v = in.val[pos];
      else if (dwta) continue;
      else v = 0.0f;
      if (v > best) {
        best = v;
        best_pos = p;
      }
    }
    if (best_pos < 0) best_pos = h.fallback[t * h.k + kk];
    code |= (uint64_t)best_pos << shift;
    shift += h.bpw;
  }
  write_out(out, h.L, i, t, code, 0.0f, false);
}

constexpr int MH_MAXK = 64;
__device__ uint64_t minhash_finish(uint32_t* mins, int K) {
  bool all_empty = true;
  for (int b = 0; b < K; ++b) all_empty &= (mins[b] == 0xffffffffu);
  if (all_empty) {
    for (int b = 0; b < K; ++b) mins[b] = 0;
  } else {
    for (int b = 0; b < K; ++b) {
      if (mins[b] == 0xffffffffu) {
        int j = (b + 1) % K;
        while (mins[j] == 0xffffffffu) j = (j + 1) % K;
        mins[b] = mins[j];
      }
    }
  }
  const uint64_t PRIME = 0x517cc1b727220a95ULL;
  const uint64_t mask = K >= 64 ? ~0ULL : ((1ULL << K) - 1);
  uint64_t hsh = 0, pp = 1;
  for (int b = 0; b < K; ++b) {
    hsh += (uint64_t)mins[b] * pp;
    pp *= PRIME;
  }
  return hsh & mask;
}

__global__ void minhash_dense_kernel(DevHash h, DenseIn in, HashOut out) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)in.n * h.L) return;
  const int i = (int)(g / h.L), t = (int)(g % h.L);
  uint32_t mins[MH_MAXK];
  for (int b = 0; b < h.k; ++b) mins[b] = 0xffffffffu;
  const uint32_t* perm = h.perms + (int64_t)t * h.d;
  for (int dim = 0; dim < h.d; ++dim) {
    float v = ldx_dt(in.X, in.dtype, (int64_t)i * in.ld_row + (int64_t)dim * in.ld_elem);
    if (v != 0.0f) {
      uint32_t pm = perm[dim];
      uint32_t bin = pm / (uint32_t)h.bin_size;
      if ((int)bin < h.k) mins[bin] = min(mins[bin], pm);
    }
  }
  write_out(out, h.L, i, t, minhash_finish(mins, h.k), 0.0f, false);
}

__global__ void minhash_sparse_kernel(DevHash h, SparseIn in, HashOut out) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)in.n * h.L) return;
  const int i = (int)(g / h.L), t = (int)(g % h.L);
  uint32_t mins[MH_MAXK];
  for (int b = 0; b < h.k; ++b) mins[b] = 0xffffffffu;
  const uint32_t* perm = h.perms + (int64_t)t * h.d;
  for (int e = in.rowptr[i]; e < in.rowptr[i + 1]; ++e) {
    uint32_t dim = in.idx[e];
    if (dim >= (uint32_t)h.d) continue;
    uint32_t pm = perm[dim];
    uint32_t bin = pm / (uint32_t)h.bin_size;
    if ((int)bin < h.k) mins[bin] = min(mins[bin], pm);
  }
  write_out(out, h.L, i, t, minhash_finish(mins, h.k), 0.0f, false);
}

}  // namespace

void launch_hash_dense(const DevHash& h, const DenseIn& in, const HashOut& out, cudaStream_t st) {
  if (in.n <= 0) return;
  switch (h.kind) {
    case KL_HASH_SIMHASH:
    case KL_HASH_SRP: {
      // bf16 row batches (table rebuilds) go to the tensor cores unless the
      // caller asked for the reference's sequential sums
      if (h.tc && h.tc->mode != KL_PROJ_SEQUENTIAL && (h.tc->mode == KL_PROJ_TENSOR || in.n >= 4096) &&
          launch_proj_tc(h, in, out, h.tc->err, st))
        break;
      const int TT = std::min(h.L, std::max(1, 12 / h.k));
      dim3 grid((unsigned)ceil_div(in.n, 32), (unsigned)ceil_div(h.L, TT));
      dim3 block(32 * TT * h.k);
      const int tdim = std::min(h.d, PL_T);
      const bool fmb = in.ld_row == 1 && in.dtype == KL_DTYPE_BF16 && in.ld_elem % 8 == 0 &&
                       (reinterpret_cast<uintptr_t>(in.X) & 15) == 0;
      const size_t xbytes = fmb ? (size_t)2 * tdim * 64 : (size_t)tdim * PL_PITCH * 4;
      const size_t sm = (size_t)round_up((int64_t)xbytes, 16) + (size_t)TT * h.k * 32 * sizeof(float);
      static OncePerDevice attr;
      attr([&] {
        cudaFuncSetAttribute(proj_list_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(proj_list_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      });
      if (fmb) proj_list_kernel<true><<<grid, block, sm, st>>>(h, in, out, TT);
      else proj_list_kernel<false><<<grid, block, sm, st>>>(h, in, out, TT);
      count_launch();
      break;
    }
    case KL_HASH_WTA:
    case KL_HASH_DWTA: {
      const size_t sm = (size_t)32 * (h.d + 1) * sizeof(float);
      if (sm <= 200 * 1024) {
        int nwin = h.k;
        if (!out.codes && !out.min_abs) {
          const int bits = __builtin_popcount(out.nb_mask);
          nwin = std::min(h.k, (bits + h.bpw - 1) / h.bpw);
        }
        static OncePerDevice attr;
        attr([&] {
          cudaFuncSetAttribute(wta_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        });
        // few row tiles (a query batch): spread the tables over more blocks
        const int rt = (int)ceil_div(in.n, 32);
        const int tg = std::max(1, std::min(h.L / 8, 296 / std::max(rt, 1)));
        wta_tile_kernel<<<dim3((unsigned)rt, (unsigned)tg), 256, sm, st>>>(h, in, out, nwin);
      } else {
        int64_t tot = (int64_t)in.n * h.L;
        wta_dense_kernel<<<(unsigned)ceil_div(tot, 256), 256, 0, st>>>(h, in, out);
      }
      count_launch();
      break;
    }
    case KL_HASH_MINHASH: {
      int64_t tot = (int64_t)in.n * h.L;
      minhash_dense_kernel<<<(unsigned)ceil_div(tot, 128), 128, 0, st>>>(h, in, out);
  count_launch();
      break;
    }
  }
}

void launch_hash_sparse(const DevHash& h, const SparseIn& in, const HashOut& out, cudaStream_t st) {
  if (in.n <= 0) return;
  switch (h.kind) {
    case KL_HASH_SIMHASH:
    case KL_HASH_SRP: {
      int nt = (int)round_up(h.LK, 32);
      const size_t sm = ((size_t)round_up(h.LK, 4) + (size_t)PS_CH * h.lkpad / 4) * sizeof(float);
      static OncePerDevice attr;
      attr([&] {
        cudaFuncSetAttribute(proj_sparse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      });
      proj_sparse_kernel<<<in.n, nt, sm, st>>>(h, in, out);
  count_launch();
      break;
    }
    case KL_HASH_WTA:
    case KL_HASH_DWTA: {
      int64_t tot = (int64_t)in.n * h.L;
      wta_sparse_kernel<<<(unsigned)ceil_div(tot, 256), 256, 0, st>>>(h, in, out);
  count_launch();
      break;
    }
    case KL_HASH_MINHASH: {
      int64_t tot = (int64_t)in.n * h.L;
      minhash_sparse_kernel<<<(unsigned)ceil_div(tot, 128), 128, 0, st>>>(h, in, out);
  count_launch();
      break;
    }
  }
}

}  // namespace kl
