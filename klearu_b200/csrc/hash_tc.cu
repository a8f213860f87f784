// hash_tc.cu -- SimHash / SRP projection of bf16 rows on the tensor cores.
//
// Table rebuilds hash every row of a layer (crates/klearu-core/src/lsh/
// index.rs:302-316 after network/layer.rs:228-233): for row x and projection
// p, bit p of its table's code is (plane_p . x >= 0) (hash/simhash.rs:75-126).
// Over all rows that is the dense product X[n x d] . P^T[d x L*K] followed by
// a sign test, a GEMM that belongs on tcgen05:
//
//  * A operand: 128 rows of X per tile (bf16, K-major), streamed by TMA
//    (cp.async.bulk.tensor, 128-byte swizzle, no multicast) through a ring of
//    shared-memory stages;
//  * B operand: the ternary planes as exact bf16 (-1 / 0 / +1), K-major,
//    resident in shared memory for the whole kernel.  The tables are split
//    into H groups so that one group's planes fit beside the ring; CTA b
//    always serves group b % H, so it loads its planes once;
//  * accumulator: f32 in tensor memory, two buffers so that the epilogue of
//    one tile overlaps the MMAs of the next;
//  * epilogue (8 warps: one row per thread, the two warps of a TMEM lane
//    quadrant on half the tables each): tcgen05.ld of the row's
//    projections, sign-pack into each table's K-bit code, bucket index and
//    min |projection| written straight to the hash outputs.
//
// Warp roles: warp 0 issues the TMA loads, warp 1 owns tensor memory and
// issues the MMAs (one thread), warps 2..9 run the epilogue.  Every wait is
// bounded; a wait that gives up records DERR_TIMEOUT and the kernel winds
// down without leaving copies in flight.
//
// Numerics: every product of a bf16 row element and a plane entry is exact;
// the tensor core accumulates in f32 in its own order, so a projection
// within a few f32 ulps of zero may take the other sign than the reference's
// sequential sum.  Callers that need the reference's bits exactly use the
// sequential CUDA-core kernel (kl_hash_set_projection); min |projection| is
// written so that such rows can be identified.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "engine.h"
#include "tcgen05.cuh"

namespace kl {
namespace {

constexpr int TP_M = 128;          // rows per tile (MMA M)
constexpr int TP_KC = 64;          // K elements per TMA box / stage: 128-byte rows
constexpr int TP_ASTAGE = TP_M * TP_KC * 2;
constexpr int TP_NT = 320;         // 10 warps: TMA, MMA, 8 epilogue warps
constexpr int TP_SMEM_MAX = 213 * 1024;  // + ~9.5 KB static, under the 227 KB per block

__host__ __device__ constexpr uint32_t tp_idesc(int n) { return f16_idesc(TP_M, n); }
__device__ __forceinline__ void tp_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  tc5_ld16_async(taddr, v);
  tc5_ld_wait();
}

struct TpArgs {
  int n;        // rows
  int kc;       // K chunks of 64 (ceil(d / 64))
  int H;        // table groups
  int tph;      // tables per group
  int Nh;       // projection columns per group (multiple of 16, <= 256)
  int L, k;     // tables, bits per table
  int nst;      // A stages
  uint32_t tmem_cols;
  HashOut out;
  int* err;
};

// Shared memory: [B: kc chunks of Nh x 128 B][A ring: nst x 16 KB], 1024-aligned.
// MINABS: the per-table min |projection| is wanted (a column-by-column
// epilogue); otherwise the epilogue packs the sign bits of 64 columns at a
// time and cuts the tables' codes out of the packed words.
template <bool MINABS>
__global__ void __launch_bounds__(TP_NT, 1)
    proj_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap pmap, TpArgs a) {
  extern __shared__ unsigned char tp_dyn[];
  __shared__ uint64_t full[16], empty[16], bfull, acc_full[2], acc_empty[2];
  __shared__ uint32_t ebits[8][9][32];  // per epilogue warp: packed sign bits [word][lane] (+1 spare word)
  __shared__ uint32_t tmem_s;
  __shared__ int fail;
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tp_dyn) + 1023) & ~uintptr_t(1023));
  const int bbytes = a.kc * a.Nh * 128;
  unsigned char* sB = sm;
  unsigned char* sA = sm + bbytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x % a.H;
  const int tiles = (a.n + TP_M - 1) / TP_M;
  const int tstride = gridDim.x / a.H;
  const int t0 = blockIdx.x / a.H;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&bfull, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    fail = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&tmem_s)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc5_fence_before();
  __syncthreads();
  tc5_fence_after();
  const uint32_t tmem = tmem_s;

  if (warp == 0) {
    if (lane == 0) {
      // the group's planes, once
      mbar_arrive_expect_tx(&bfull, (uint32_t)bbytes);
      for (int c = 0; c < a.kc; ++c) tma_load_2d(sB + c * a.Nh * 128, &pmap, c * TP_KC, g * a.Nh, &bfull);
      uint32_t q = 0;  // chunks issued
      for (int t = t0; t < tiles && !*(volatile int*)&fail; t += tstride) {
        for (int c = 0; c < a.kc; ++c, ++q) {
          const int s = (int)(q % a.nst);
          const uint32_t round = q / a.nst;
          if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1u)) {
            atomicExch(&fail, 1);
            break;
          }
          mbar_arrive_expect_tx(&full[s], TP_ASTAGE);
          tma_load_2d(sA + s * TP_ASTAGE, &xmap, c * TP_KC, t * TP_M, &full[s]);
        }
      }
      // no copy may be left in flight when the CTA exits: wait (bounded) for the
      // last round of every stage and for the planes
      mbar_wait(&bfull, 0);
      for (uint32_t r = q > (uint32_t)a.nst ? q - a.nst : 0; r < q; ++r)
        mbar_wait(&full[r % a.nst], (r / a.nst) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(&bfull, 0);
      const uint32_t idesc = tp_idesc(a.Nh);
      const uint32_t sa0 = smem_u32(sA), sb0 = smem_u32(sB);
      uint32_t q = 0, j = 0;
      for (int t = t0; ok && t < tiles; t += tstride, ++j) {
        const uint32_t buf = j & 1u, use = j >> 1;
        if (use > 0 && !mbar_wait(&acc_empty[buf], (use - 1) & 1u)) {
          ok = false;
          break;
        }
        tc5_fence_after();
        const uint32_t d = tmem + buf * (uint32_t)a.Nh;
        for (int c = 0; c < a.kc; ++c, ++q) {
          const int s = (int)(q % a.nst);
          if (!mbar_wait(&full[s], (q / a.nst) & 1u)) {
            ok = false;
            break;
          }
          tc5_fence_after();
#pragma unroll
          for (int kk = 0; kk < TP_KC / 16; ++kk)
            tc5_mma(d, sw128_desc(sa0 + s * TP_ASTAGE + kk * 32), sw128_desc(sb0 + c * a.Nh * 128 + kk * 32), idesc,
                   (c | kk) != 0);
          tc5_commit(&empty[s]);
        }
        if (!ok) break;
        tc5_commit(&acc_full[buf]);
      }
      if (!ok) atomicExch(&fail, 1);
    }
  } else {
    // epilogue: warp w reads tensor-memory lanes 32 * (w % 4) .. + 31; the two
    // warps of a lane quadrant split the group's tables in halves
    const int quad = warp & 3, half = (warp - 2) >> 2;
    const int kbits = a.k;
    const int ntab_g = min(a.tph, a.L - g * a.tph);     // tables of this group
    const int lt_lo = half ? ntab_g / 2 : 0, lt_hi = half ? ntab_g : ntab_g / 2;
    const int c_lo = lt_lo * kbits, c_hi = lt_hi * kbits;  // this warp's projection columns
    uint32_t j = 0;
    for (int t = t0; t < tiles; t += tstride, ++j) {
      const uint32_t buf = j & 1u, use = j >> 1;
      if (!mbar_wait(&acc_full[buf], use & 1u)) {
        atomicExch(&fail, 1);
        break;
      }
      tc5_fence_after();
      const int row = t * TP_M + quad * 32 + lane;
      const uint32_t base = tmem + ((uint32_t)(quad * 32) << 16) + buf * (uint32_t)a.Nh;
      if (!MINABS) {
        // sign bits: 64 columns per round (4 loads, one wait), 2 words each
        uint32_t (*eb)[32] = ebits[warp - 2];
#pragma unroll
        for (int g64 = 0; g64 < 4; ++g64) {
          if (g64 * 64 < c_hi && g64 * 64 + 64 > c_lo) {
            uint32_t v[64];
#pragma unroll
            for (int u = 0; u < 4; ++u) tc5_ld16_async(base + (uint32_t)(g64 * 64 + u * 16), v + u * 16);
            tc5_ld_wait();
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int qq = 0; qq < 32; ++qq) {
              lo |= (__uint_as_float(v[qq]) >= 0.0f ? 1u : 0u) << qq;
              hi |= (__uint_as_float(v[32 + qq]) >= 0.0f ? 1u : 0u) << qq;
            }
            eb[2 * g64][lane] = lo;
            eb[2 * g64 + 1][lane] = hi;
          }
        }
        eb[8][lane] = 0u;
        tc5_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);  // the accumulator is free again
        if (row < a.n) {
          const uint32_t kmask = kbits >= 32 ? 0xffffffffu : (1u << kbits) - 1u;
          for (int lt = lt_lo; lt < lt_hi; ++lt) {
            const int p0 = lt * kbits, w0 = p0 >> 5, off = p0 & 31;
            const uint64_t win = (uint64_t)eb[w0][lane] | ((uint64_t)eb[w0 + 1][lane] << 32);
            const uint64_t code = (uint64_t)((uint32_t)(win >> off) & kmask);
            const int tab = g * a.tph + lt;
            if (a.out.codes) a.out.codes[(int64_t)row * a.L + tab] = code;
            if (a.out.bkt) a.out.bkt[(int64_t)tab * a.out.bkt_ld + row] = (uint16_t)(code & a.out.nb_mask);
          }
        }
        __syncwarp();  // eb is rewritten by the next tile
        continue;
      }
      int tab = g * a.tph + lt_lo, bit = 0;
      uint64_t code = 0;
      float mn = INFINITY;
      for (int cb = c_lo & ~15; cb < c_hi; cb += 16) {
        uint32_t v[16];
        tp_ld16(base + (uint32_t)cb, v);
#pragma unroll
        for (int qq = 0; qq < 16; ++qq) {
          if (cb + qq >= c_lo && cb + qq < c_hi) {
            const float p = __uint_as_float(v[qq]);
            if (p >= 0.0f) code |= 1ull << bit;
            mn = fminf(mn, fabsf(p));
            if (++bit == kbits) {
              if (row < a.n) {
                const int64_t o = (int64_t)row * a.L + tab;
                if (a.out.codes) a.out.codes[o] = code;
                if (a.out.min_abs) a.out.min_abs[o] = mn;
                if (a.out.bkt) a.out.bkt[(int64_t)tab * a.out.bkt_ld + row] = (uint16_t)(code & a.out.nb_mask);
              }
              ++tab;
              bit = 0;
              code = 0;
              mn = INFINITY;
            }
          }
        }
      }
      tc5_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc5_fence_before();
  __syncthreads();
  if (fail && threadIdx.x == 0) atomicOr(a.err, DERR_TIMEOUT);
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(a.tmem_cols)
                 : "memory");
}

}  // namespace

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool tma_map_bf16(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


// Host-side plane layout of the tensor-core projection: H groups of `tph`
// tables; group g's rows [g*Nh, g*Nh + tph*k) hold its tables' planes in
// (table, bit) order, the rest zero; K (dims) padded to a multiple of 64.
bool tc_plane_layout(int d, int k, int L, TcPlanes* tp) {
  const int kc = (d + TP_KC - 1) / TP_KC;
  const int dpad = kc * TP_KC;
  for (int H = 1; H <= 16; ++H) {
    const int tph = (L + H - 1) / H;
    const int Nh = (int)round_up((int64_t)tph * k, 16);
    if (Nh > 256) continue;
    const int bbytes = kc * Nh * 128;
    const int nst = (TP_SMEM_MAX - 1024 - bbytes) / TP_ASTAGE;
    if (nst < 3) continue;
    tp->H = H;
    tp->tph = tph;
    tp->Nh = Nh;
    tp->kc = kc;
    tp->dpad = dpad;
    tp->nst = nst < 16 ? nst : 16;
    return true;
  }
  return false;
}

bool tc_plane_map(TcPlanes* tp) {
  return tma_map_bf16(&tp->map, tp->planes, (int64_t)tp->H * tp->Nh, tp->dpad, tp->dpad, TP_KC, tp->Nh);
}

// Launches the tensor-core projection when the input allows it (bf16 rows,
// K-major with a 16-byte-multiple pitch, 16-byte-aligned base); returns
// false (nothing launched) otherwise.
bool launch_proj_tc(const DevHash& h, const DenseIn& in, const HashOut& out, int* err, cudaStream_t st) {
  const TcPlanes* tp = h.tc;
  if (!tp || !tp->ready || in.dtype != KL_DTYPE_BF16 || in.ld_elem != 1 || (in.ld_row * 2) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(in.X) & 15) != 0 || in.ld_row < h.d || in.n <= 0)
    return false;
  CUtensorMap xmap;
  if (!tma_map_bf16(&xmap, in.X, in.n, h.d, in.ld_row, TP_KC, TP_M)) return false;
  static OncePerDevice attr;
  attr([&] {
    cudaFuncSetAttribute(proj_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TP_SMEM_MAX);
    cudaFuncSetAttribute(proj_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TP_SMEM_MAX);
  });
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = (int)ceil_div(in.n, TP_M);
  const int per = std::max(1, sms / tp->H);
  const int grid = tp->H * std::min(per, tiles);
  TpArgs a;
  a.n = in.n;
  a.kc = tp->kc;
  a.H = tp->H;
  a.tph = tp->tph;
  a.Nh = tp->Nh;
  a.L = h.L;
  a.k = h.k;
  a.nst = tp->nst;
  uint32_t cols = 32;
  while (cols < 2u * (uint32_t)tp->Nh) cols <<= 1;
  a.tmem_cols = cols;
  a.out = out;
  a.err = err;
  const size_t smem = 1024 + (size_t)tp->kc * tp->Nh * 128 + (size_t)tp->nst * TP_ASTAGE;
  if (out.min_abs) proj_tc_kernel<true><<<grid, TP_NT, smem, st>>>(xmap, tp->map, a);
  else proj_tc_kernel<false><<<grid, TP_NT, smem, st>>>(xmap, tp->map, a);
  count_launch();
  return true;
}

}  // namespace kl
