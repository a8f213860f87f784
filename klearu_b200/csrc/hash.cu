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

// ---------------------------------------------------------------------------
// Projection hashing of dense rows.  Block = 32 rows x (TT tables x K bits);
// thread (row r, projection tb) owns one sequential f32 chain over d.  Input
// tiles of 64 columns are staged in shared memory (pitch 65 floats: lanes that
// read different rows hit different banks); plane rows are read 16 bytes at a
// time (all lanes of a warp share one projection -> broadcast).
// ---------------------------------------------------------------------------
constexpr int PJ_ROWS = 32;
constexpr int PJ_DT = 64;

__global__ void proj_dense_kernel(DevHash h, DenseIn in, HashOut out, int TT) {
  __shared__ float xs[PJ_ROWS][PJ_DT + 1];
  extern __shared__ unsigned char dyn[];
  const int K = h.k;
  const int nthr = blockDim.x;
  const int r = threadIdx.x & 31;
  const int q = threadIdx.x >> 5;  // projection within the block: tt*K + b
  const int tt = q / K, b = q % K;
  const int t = blockIdx.y * TT + tt;
  const int row0 = blockIdx.x * PJ_ROWS;
  const bool active = (t < h.L);
  const int tb = t * K + b;
  const int8_t* prow = h.planes + (int64_t)(active ? tb : 0) * h.dpad;
  float acc = 0.0f;
  for (int d0 = 0; d0 < h.d; d0 += PJ_DT) {
    // stage X[row0 .. row0+32)[d0 .. d0+64) as f32
    for (int e = threadIdx.x; e < PJ_ROWS * PJ_DT; e += nthr) {
      int rr, dd;
      if (in.ld_elem == 1) {
        rr = e / PJ_DT;
        dd = e % PJ_DT;
      } else {
        rr = e % PJ_ROWS;
        dd = e / PJ_ROWS;
      }
      float v = 0.0f;
      if (row0 + rr < in.n && d0 + dd < h.d)
        v = ldx_dt(in.X, in.dtype, (int64_t)(row0 + rr) * in.ld_row + (int64_t)(d0 + dd) * in.ld_elem);
      xs[rr][dd] = v;
    }
    __syncthreads();
    if (active) {
      const int dmax = min(PJ_DT, h.d - d0);
#pragma unroll 1
      for (int dd = 0; dd < dmax; dd += 16) {
        int4 pv = *reinterpret_cast<const int4*>(prow + d0 + dd);
        const int8_t* p8 = reinterpret_cast<const int8_t*>(&pv);
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          // columns beyond d are zero in both the plane padding and xs
          acc = __fmaf_rn((float)p8[u], xs[r][dd + u], acc);
        }
      }
    }
    __syncthreads();
  }
  // combine K sign bits per (row, table) through shared memory
  float* sv = reinterpret_cast<float*>(dyn);  // [TT*K][32]
  sv[q * 32 + r] = acc;
  __syncthreads();
  const int ncomb = TT * PJ_ROWS;
  for (int c = threadIdx.x; c < ncomb; c += nthr) {
    const int ct = c / PJ_ROWS, cr = c % PJ_ROWS;
    const int tab = blockIdx.y * TT + ct, i = row0 + cr;
    if (tab >= h.L || i >= in.n) continue;
    uint64_t code = 0;
    float mn = __int_as_float(0x7f800000);
    for (int bb = 0; bb < K; ++bb) {
      float v = sv[(ct * K + bb) * 32 + cr];
      if (v >= 0.0f) code |= 1ULL << bb;
      mn = fminf(mn, fabsf(v));
    }
    write_out(out, h.L, i, tab, code, mn, true);
  }
}

// Projection hashing of CSR rows: one block per row, one thread per projection.
__global__ void proj_sparse_kernel(DevHash h, SparseIn in, HashOut out) {
  extern __shared__ unsigned char dyn[];
  float* sv = reinterpret_cast<float*>(dyn);  // [LK]
  __shared__ uint32_t sidx[256];
  __shared__ float sval[256];
  const int i = blockIdx.x;
  const int tb = threadIdx.x;
  const int beg = in.rowptr[i], end = in.rowptr[i + 1];
  float acc = 0.0f;
  for (int c0 = beg; c0 < end; c0 += 256) {
    const int m = min(256, end - c0);
    for (int e = threadIdx.x; e < m; e += blockDim.x) {
      sidx[e] = in.idx[c0 + e];
      sval[e] = in.val[c0 + e];
    }
    __syncthreads();
    if (tb < h.LK) {
      for (int e = 0; e < m; ++e) {
        uint32_t col = sidx[e];
        float p = (col < (uint32_t)h.d) ? (float)h.planesT[(int64_t)col * h.lkpad + tb] : 0.0f;
        acc = __fmaf_rn(p, sval[e], acc);
      }
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
      int TT = max(1, 512 / (32 * h.k));
      TT = min(TT, h.L);
      dim3 grid((unsigned)ceil_div(in.n, PJ_ROWS), (unsigned)ceil_div(h.L, TT));
      dim3 block(32 * TT * h.k);
      size_t sm = (size_t)TT * h.k * 32 * sizeof(float);
      proj_dense_kernel<<<grid, block, sm, st>>>(h, in, out, TT);
  count_launch();
      break;
    }
    case KL_HASH_WTA:
    case KL_HASH_DWTA: {
      int64_t tot = (int64_t)in.n * h.L;
      wta_dense_kernel<<<(unsigned)ceil_div(tot, 256), 256, 0, st>>>(h, in, out);
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
      proj_sparse_kernel<<<in.n, nt, (size_t)h.LK * sizeof(float), st>>>(h, in, out);
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
