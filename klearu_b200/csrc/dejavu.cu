// Deja Vu sparse FFN: the sparsity predictor (a two-layer MLP scoring the
// intermediate neurons, klearu-dejavu predictor/mlp_predictor.rs:102-132)
// and the SwiGLU MLP over the selected neurons (klearu-llm
// sparse/sparse_mlp.rs:4-37, klearu-dejavu mlp.rs:23-58).
//
// Predictor layers are tensor-core GEMMs: tcgen05.mma (kind::f16, bf16
// operands, f32 accumulator in tensor memory), operands staged into shared
// memory by cp.async in the canonical no-swizzle K-major layout, a 3-stage
// pipeline whose stages are released by tcgen05.commit on an mbarrier, and an
// epilogue that reads the accumulator with tcgen05.ld.  Weights are bf16.
// The f32 activations are split exactly into three bf16 pieces
// (x = hi + mid + lo), all three multiplied into the same accumulator, so
// every product is exact and only the f32 accumulation order differs from the
// reference's sequential sums.
#include <algorithm>

#include "engine.h"

namespace kl {
namespace {

constexpr int TC_M = 128;                  // accumulator rows (tokens, zero padded)
constexpr int TC_N = 128;                  // accumulator columns (output features per tile)
constexpr int TC_K = 64;                   // K elements per stage: 128-byte rows
constexpr int TC_ST = 3;                   // pipeline stages
constexpr int TC_NP = 3;                   // bf16 pieces of the f32 activations
constexpr int TC_TILE = TC_M * TC_K * 2;   // bytes of one 128 x 64 bf16 tile
constexpr int TC_STAGE = (TC_NP + 1) * TC_TILE;

// Canonical K-major layout without swizzle: 8-row x 16-byte core matrices,
// stored contiguously (128 B); the next 16 bytes of K are the next core
// matrix (leading byte offset 128 B); the next 8 rows start 8 core matrices
// later (stride byte offset 1024 B).
__device__ __forceinline__ uint32_t canon_off(int r, int c16) { return (r >> 3) * 1024 + c16 * 128 + (r & 7) * 16; }

// Shared-memory matrix descriptor: start address, leading and stride byte
// offsets (all >> 4), descriptor version 1, no swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46);
}
// Instruction descriptor: f32 accumulator, bf16 A and B, both K-major,
// N = TC_N, M = TC_M.
constexpr uint32_t TC_IDESC =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_N >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(da), "l"(db), "r"(TC_IDESC), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// P[split][TC_M][ldp] (f32 partial sums) = A . B^T over the split's K tiles.
// A: TC_NP pieces, each [TC_M][lda] bf16 (rows past the token count are zero);
// B: [nb][ldb] bf16, rows >= nb read as zero.  lda, ldb: multiples of TC_K.
// One CTA per (128-column tile, K split); 128 threads; warp 0 owns the
// tensor-memory allocation, thread 0 issues the MMAs.
__global__ void __launch_bounds__(128, 1)
    tc_gemm_kernel(const __nv_bfloat16* __restrict__ A, int64_t a_piece, int lda, const __nv_bfloat16* __restrict__ B,
                   int ldb, int nb, int ktiles, int kt_per_split, float* __restrict__ P, int ldp, int* err) {
  extern __shared__ __align__(1024) unsigned char tc_smem[];
  __shared__ uint64_t bar_mma[TC_ST];
  __shared__ uint64_t bar_done;
  __shared__ uint32_t tmem_s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * TC_N;
  const int kt0 = blockIdx.y * kt_per_split;
  const int nk = max(0, min(ktiles, kt0 + kt_per_split) - kt0);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&tmem_s)),
                 "r"(TC_N)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < TC_ST; ++s) mbar_init(&bar_mma[s], 1);
    mbar_init(&bar_done, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_s;
  bool ok = true;

  auto load_stage = [&](int i) {  // K tile kt0 + i into stage i % TC_ST
    unsigned char* st = tc_smem + (i % TC_ST) * TC_STAGE;
    const int k0 = (kt0 + i) * TC_K;
#pragma unroll
    for (int p = 0; p < TC_NP; ++p)
      for (int q = tid; q < TC_M * 8; q += 128) {
        const int r = q >> 3, c = q & 7;
        cp_async16(st + p * TC_TILE + canon_off(r, c), A + p * a_piece + (int64_t)r * lda + k0 + c * 8);
      }
    for (int q = tid; q < TC_N * 8; q += 128) {
      const int r = q >> 3, c = q & 7;
      unsigned char* dst = st + TC_NP * TC_TILE + canon_off(r, c);
      if (n0 + r < nb) cp_async16(dst, B + (int64_t)(n0 + r) * ldb + k0 + c * 8);
      else *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
  };

  for (int i = 0; i < TC_ST - 1; ++i) {
    if (i < nk) load_stage(i);
    cp_async_commit();
  }
  for (int i = 0; i < nk; ++i) {
    const int j = i + TC_ST - 1;
    if (j < nk) {
      // stage j % TC_ST last held tile j - TC_ST: wait until its MMAs are done
      if (j >= TC_ST && !mbar_wait(&bar_mma[j % TC_ST], (uint32_t)((j / TC_ST) - 1) & 1u)) ok = false;
      load_stage(j);
    }
    cp_async_commit();
    cp_async_wait_group<TC_ST - 1>();
    fence_proxy_async_smem();  // this thread's shared-memory writes, visible to the tensor core
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const unsigned char* st = tc_smem + (i % TC_ST) * TC_STAGE;
      const uint32_t sb = smem_u32(st + TC_NP * TC_TILE);
#pragma unroll
      for (int p = 0; p < TC_NP; ++p) {
        const uint32_t sa = smem_u32(st + p * TC_TILE);
#pragma unroll
        for (int kk = 0; kk < TC_K / 16; ++kk)
          tc_mma(tmem, smem_desc(sa + kk * 256), smem_desc(sb + kk * 256), (i | p | kk) != 0);
      }
      tc_commit(&bar_mma[i % TC_ST]);
    }
  }
  if (tid == 0) tc_commit(&bar_done);  // arrives when every MMA issued above has completed
  if (nk > 0 && !mbar_wait(&bar_done, 0)) ok = false;
  tc_fence_after();
  // epilogue: warp w owns accumulator rows (tensor-memory lanes) 32w .. 32w+31
  const int row = warp * 32 + lane;
  float* dst = P + ((int64_t)blockIdx.y * TC_M + row) * ldp + n0;
#pragma unroll 1
  for (int c0 = 0; c0 < TC_N; c0 += 32) {
    uint32_t v[32];
    tc_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
    for (int q = 0; q < 32; q += 4) {
      float4 f = nk > 0 ? make_float4(__uint_as_float(v[q]), __uint_as_float(v[q + 1]), __uint_as_float(v[q + 2]),
                                      __uint_as_float(v[q + 3]))
                        : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(dst + c0 + q) = f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TC_N) : "memory");
  if (!ok && tid == 0) atomicOr(err, DERR_TIMEOUT);
}

// x[T][n] f32 -> three bf16 pieces [3][TC_M][ld] with x = hi + mid + lo
// exactly (each piece holds the next 8 significant bits); rows >= T and
// columns >= n are zero.
__global__ void split3_kernel(const float* __restrict__ x, int T, int n, int ldx, __nv_bfloat16* __restrict__ out,
                              int ld) {
  const int t = blockIdx.y;
  const int64_t piece = (int64_t)TC_M * ld;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ld; i += gridDim.x * blockDim.x) {
    const float v = (t < T && i < n) ? x[(int64_t)t * ldx + i] : 0.0f;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const float r1 = __fsub_rn(v, __bfloat162float(hi));
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const float r2 = __fsub_rn(r1, __bfloat162float(mid));
    const __nv_bfloat16 lo = __float2bfloat16_rn(r2);
    const int64_t o = (int64_t)t * ld + i;
    out[o] = hi;
    out[piece + o] = mid;
    out[2 * piece + o] = lo;
  }
}

// y[t][j] = act(sum over splits of P[s][t][j] + bias[j]) for t < T, j < n;
// act 0 = ReLU (f32::max against 0), 1 = sigmoid.
__global__ void splitk_finish_kernel(const float* __restrict__ P, int splits, int ldp, const float* __restrict__ bias,
                                     int T, int n, int act, float* __restrict__ y, int ldy) {
  const int t = blockIdx.y;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int q = 0; q < splits; ++q) s = __fadd_rn(s, P[((int64_t)q * TC_M + t) * ldp + j]);
    const float v = __fadd_rn(s, bias[j]);
    y[(int64_t)t * ldy + j] = act == 0 ? fmaxf(v, 0.0f) : __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
  }
}

// ---------------------------------------------------------------------------
// select_top_k (mlp_predictor.rs:126-132): the k largest scores of a row in
// (score descending, index ascending) order -- the stable sort's order.
// Scores are sigmoid outputs, non-negative, so their bit patterns order like
// the values.  One block per token: a 4-pass 8-bit radix select finds the
// k-th largest key, the keys above it and the first ties (lowest indices)
// are gathered, and a bitonic sort of (~key, index) orders them.
// ---------------------------------------------------------------------------
constexpr int TK_NT = 1024;

__global__ void __launch_bounds__(TK_NT) topk_kernel(const float* __restrict__ scores, int n, int lds, int k,
                                                     uint32_t* __restrict__ idx, int ldi, int pow2) {
  extern __shared__ __align__(1024) unsigned char tk_smem[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(tk_smem);  // [pow2]
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel_prefix, sel_mask, need_s, n_gt, n_eq_taken;
  const int t = blockIdx.x, tid = threadIdx.x;
  const float* row = scores + (int64_t)t * lds;
  if (tid == 0) {
    sel_prefix = 0;
    sel_mask = 0;
    need_s = (uint32_t)k;
  }
  __syncthreads();
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += TK_NT) hist[b] = 0;
    __syncthreads();
    const uint32_t pre = sel_prefix, msk = sel_mask;
    for (int i = tid; i < n; i += TK_NT) {
      const uint32_t key = __float_as_uint(row[i]);
      if ((key & msk) == pre) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t need = need_s, b = 255;
      for (;; --b) {  // walk down from the largest digit
        if (hist[b] >= need || b == 0) break;
        need -= hist[b];
      }
      sel_prefix = pre | (b << shift);
      sel_mask = msk | (255u << shift);
      need_s = need;  // how many keys equal to the final threshold are still needed (after the last pass)
    }
    __syncthreads();
  }
  const uint32_t thr = sel_prefix;
  if (tid == 0) {
    n_gt = 0;
    n_eq_taken = 0;
  }
  for (int i = tid; i < pow2; i += TK_NT) keys[i] = ~0ull;
  __syncthreads();
  // keys above the threshold, in any order; then ties in index order
  for (int i = tid; i < n; i += TK_NT) {
    const uint32_t key = __float_as_uint(row[i]);
    if (key > thr) {
      const uint32_t pos = atomicAdd(&n_gt, 1u);
      keys[pos] = ((uint64_t)(~key) << 32) | (uint32_t)i;
    }
  }
  __syncthreads();
  const uint32_t ties = need_s;  // number of threshold-equal keys to take, lowest indices first
  for (int base = 0; base < n && n_eq_taken < ties; base += TK_NT) {
    const int i = base + tid;
    const bool eq = i < n && __float_as_uint(row[i]) == thr;
    // rank among the equal keys of this chunk (block-wide prefix via warp ballots)
    const uint32_t bal = __ballot_sync(0xffffffffu, eq);
    __shared__ uint32_t wcnt[TK_NT / 32];
    if ((tid & 31) == 0) wcnt[tid >> 5] = __popc(bal);
    __syncthreads();
    uint32_t before = 0;
    for (int w = 0; w < (tid >> 5); ++w) before += wcnt[w];
    before += __popc(bal & ((1u << (tid & 31)) - 1u));
    const uint32_t taken = n_eq_taken;
    if (eq && taken + before < ties) keys[n_gt + taken + before] = ((uint64_t)(~thr) << 32) | (uint32_t)i;
    __syncthreads();
    if (tid == 0) {
      uint32_t tot = 0;
      for (int w = 0; w < TK_NT / 32; ++w) tot += wcnt[w];
      n_eq_taken = min(ties, taken + tot);
    }
    __syncthreads();
  }
  // bitonic sort ascending of keys[0, pow2)
  for (int size = 2; size <= pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < pow2; i += TK_NT) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const uint64_t a = keys[i], b = keys[j];
          if ((a > b) == up) {
            keys[i] = b;
            keys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < k; i += TK_NT) idx[(int64_t)t * ldi + i] = (uint32_t)(keys[i] & 0xffffffffu);
}

// ---------------------------------------------------------------------------
// Sparse SwiGLU MLP over the selected neurons of each token.
// (1) dv_gateup_kernel: one warp per selected neuron i of token t:
//     a = silu(gate[i] . x) * (up[i] . x), 16-byte row loads, x in shared
//     memory, a warp-level reduction.
// (2) dv_down_kernel: out[t][j] = sum over the selection (in list order, per
//     split of the list) of downT[sel][j] * a; downT is the down projection
//     stored transposed ([inter][hidden]) so a selected neuron's weights are
//     one contiguous row.  Splits are added in order by dv_down_finish_kernel
//     (plus the optional bias).
// ---------------------------------------------------------------------------
constexpr int DV_WARPS = 8;

__global__ void __launch_bounds__(DV_WARPS * 32)
    dv_gateup_kernel(const __nv_bfloat16* __restrict__ gate, const __nv_bfloat16* __restrict__ up, int hid, int ldw,
                     const float* __restrict__ x, int ldx, const uint32_t* __restrict__ sel, int k, int inter,
                     float* __restrict__ a, int* err) {
  extern __shared__ __align__(1024) float xs[];
  const int t = blockIdx.y, w = threadIdx.x >> 5, l = threadIdx.x & 31;
  for (int i = threadIdx.x; i < ldw; i += blockDim.x) xs[i] = i < hid ? x[(int64_t)t * ldx + i] : 0.0f;
  __syncthreads();
  for (int s = blockIdx.x * DV_WARPS + w; s < k; s += gridDim.x * DV_WARPS) {
    uint32_t row = sel[(int64_t)t * k + s];
    if (row >= (uint32_t)inter) {
      if (l == 0) atomicOr(err, DERR_BOUNDS);
      row = 0;
    }
    const uint4* g4 = reinterpret_cast<const uint4*>(gate + (int64_t)row * ldw);
    const uint4* u4 = reinterpret_cast<const uint4*>(up + (int64_t)row * ldw);
    float g = 0.f, u = 0.f;
    for (int c = l; c < ldw / 8; c += 32) {
      const uint4 gr = g4[c], ur = u4[c];
      const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gr);
      const __nv_bfloat16* ue = reinterpret_cast<const __nv_bfloat16*>(&ur);
      const float4 xa = reinterpret_cast<const float4*>(xs)[2 * c], xb = reinterpret_cast<const float4*>(xs)[2 * c + 1];
      const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        g = fmaf(__bfloat162float(ge[q]), xv[q], g);
        u = fmaf(__bfloat162float(ue[q]), xv[q], u);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      g += __shfl_xor_sync(0xffffffffu, g, o);
      u += __shfl_xor_sync(0xffffffffu, u, o);
    }
    if (l == 0) a[(int64_t)t * k + s] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
  }
}

constexpr int DV_DN_T = 256;  // output columns per block
constexpr int DV_PF = 8;      // selected rows in flight per thread

__global__ void __launch_bounds__(DV_DN_T)
    dv_down_kernel(const __nv_bfloat16* __restrict__ downT, int hid, int ldw, const uint32_t* __restrict__ sel, int k,
                   int inter, const float* __restrict__ a, int splits, float* __restrict__ part) {
  const int t = blockIdx.z, sp = blockIdx.y;
  const int j = blockIdx.x * DV_DN_T + threadIdx.x;
  const int per = (k + splits - 1) / splits;
  const int s0 = sp * per, s1 = min(k, s0 + per);
  float acc = 0.0f;
  if (j < hid) {
    for (int s = s0; s < s1; s += DV_PF) {
      float wv[DV_PF], av[DV_PF];
#pragma unroll
      for (int u = 0; u < DV_PF; ++u) {
        if (s + u < s1) {
          uint32_t row = sel[(int64_t)t * k + s + u];
          if (row >= (uint32_t)inter) row = 0;
          wv[u] = __bfloat162float(downT[(int64_t)row * ldw + j]);
          av[u] = a[(int64_t)t * k + s + u];
        }
      }
#pragma unroll
      for (int u = 0; u < DV_PF; ++u)
        if (s + u < s1 && av[u] != 0.0f) acc = __fadd_rn(acc, __fmul_rn(wv[u], av[u]));
    }
    part[((int64_t)t * splits + sp) * ldw + j] = acc;
  }
}

__global__ void dv_down_finish_kernel(const float* __restrict__ part, int splits, int hid, int ldw,
                                      const float* __restrict__ bias, float* __restrict__ out) {
  const int t = blockIdx.y;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < hid; j += gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int q = 0; q < splits; ++q) s = __fadd_rn(s, part[((int64_t)t * splits + q) * ldw + j]);
    out[(int64_t)t * hid + j] = bias ? __fadd_rn(s, bias[j]) : s;
  }
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

}  // namespace

// K splits of the tcgen05 linear: enough CTAs to cover the SMs, at least two
// K tiles per split.  *per = K tiles per split.
int tc_linear_splits(int n, int ldw, int* per) {
  const int ntile = (int)ceil_div(n, TC_N);
  const int ktiles = ldw / TC_K;
  int splits = std::max(1, std::min(std::min(16, ktiles / 2), (int)ceil_div(sm_count(), ntile)));
  const int p = (int)ceil_div(ktiles, splits);
  if (per) *per = p;
  return (int)ceil_div(ktiles, p);
}
size_t tc_linear_scratch_floats(int n, int ldw) {
  return (size_t)tc_linear_splits(n, ldw, nullptr) * TC_M * ceil_div(n, TC_N) * TC_N;
}

// y[T][n] = act(x[T][d] . W^T + b) through the tcgen05 GEMM; T <= 128.
// W: [n][ldw] bf16 (ldw a multiple of 64, zero beyond d).  xs: split scratch
// [3][128][ldw] bf16; P: split-K scratch [splits][128][round_up(n, 128)] f32.
void launch_tc_linear(const float* x, int T, int d, int ldx, const __nv_bfloat16* W, int n, int ldw,
                      const float* bias, int act, float* y, int ldy, __nv_bfloat16* xs, float* P, int max_splits,
                      int* err, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_ST * TC_STAGE);
    attr = true;
  }
  split3_kernel<<<dim3((unsigned)ceil_div(ldw, 256), TC_M), 256, 0, st>>>(x, T, d, ldx, xs, ldw);
  count_launch();
  const int ntile = (int)ceil_div(n, TC_N);
  const int ktiles = ldw / TC_K;
  int per = 0;
  const int splits = tc_linear_splits(n, ldw, &per);
  (void)max_splits;
  const int ldp = ntile * TC_N;
  tc_gemm_kernel<<<dim3(ntile, splits), 128, TC_ST * TC_STAGE, st>>>(xs, (int64_t)TC_M * ldw, ldw, W, ldw, n, ktiles,
                                                                     per, P, ldp, err);
  count_launch();
  splitk_finish_kernel<<<dim3((unsigned)ceil_div(n, 256), T), 256, 0, st>>>(P, splits, ldp, bias, T, n, act, y, ldy);
  count_launch();
}

void launch_topk(const float* scores, int T, int n, int lds, int k, uint32_t* idx, int ldi, cudaStream_t st) {
  int pow2 = 1;
  while (pow2 < k) pow2 <<= 1;
  const size_t sm = (size_t)pow2 * 8;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr = true;
  }
  topk_kernel<<<T, TK_NT, sm, st>>>(scores, n, lds, k, idx, ldi, pow2);
  count_launch();
}

void launch_sparse_mlp(const __nv_bfloat16* gate, const __nv_bfloat16* up, const __nv_bfloat16* downT, int hid,
                       int ldw, int inter, const float* bias, const float* x, int T, const uint32_t* sel, int k,
                       float* a, float* part, int splits, float* out, int* err, cudaStream_t st) {
  const int gblocks = std::max(1, std::min((int)ceil_div(k, DV_WARPS), (int)ceil_div(sm_count() * 4, T)));
  dv_gateup_kernel<<<dim3(gblocks, T), DV_WARPS * 32, (size_t)ldw * 4, st>>>(gate, up, hid, ldw, x, hid, sel, k,
                                                                             inter, a, err);
  count_launch();
  dv_down_kernel<<<dim3((unsigned)ceil_div(hid, DV_DN_T), splits, T), DV_DN_T, 0, st>>>(downT, hid, ldw, sel, k,
                                                                                       inter, a, splits, part);
  count_launch();
  dv_down_finish_kernel<<<dim3((unsigned)ceil_div(hid, 256), T), 256, 0, st>>>(part, splits, hid, ldw, bias, out);
  count_launch();
}

}  // namespace kl
