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
#include "tcgen05.cuh"

namespace kl {
namespace {

constexpr int TC_M = 128;                  // accumulator rows: output features (weight rows) per tile
constexpr int TC_K = 64;                   // K elements per stage: 128-byte rows
constexpr int TC_NP = 3;                   // bf16 pieces of the f32 activations
constexpr int TC_TMAX = 85;                // tokens per call: 3 piece rows each, <= 256 accumulator columns
constexpr int TC_WTILE = TC_M * TC_K * 2;  // bytes of one 128 x 64 bf16 weight tile
constexpr int TC_SMEM = 200 * 1024;        // shared-memory budget of the stage ring

// P[split][t][n0 + m] (f32 partial sums, t < T) = sum over the split's K tiles
// of W[n0 + m] . x[t]: the weights are the MMA's A operand (M = 128 rows per
// tile), the token pieces its B operand: row 3t + p of X is piece p of token
// t, so one MMA per 16-wide K step covers every piece of every token, and the
// epilogue adds a token's three accumulator columns (hi + mid + lo).
// Both operands arrive by TMA (128-byte swizzle, no multicast): thread 0
// (warp 0) keeps NST stages of (128 x 64 weight tile + NT x 64 token tile)
// in flight, thread 32 (warp 1) issues the MMAs of a stage once its bytes
// have landed and releases the stage through tcgen05.commit.  Weight rows
// >= nw and token rows beyond the piece buffer read as zero; token-piece
// rows 3T .. NT-1 hold other data, whose accumulator columns the epilogue
// never reads.  One CTA per (128-row tile, K split); warp 1 owns the tensor
// memory; the epilogue reads row m = lane of warp m / 32.
template <int NT>
struct TcCfg {
  static constexpr int XTILE = NT * TC_K * 2;  // the token-piece rows
  static constexpr int STAGE = TC_WTILE + XTILE;
  // token tiles up to 64 wide: two CTAs per SM, so that two MMA chains and
  // their load rings share the SM
  static constexpr int CTAS = NT <= 64 ? 2 : 1;
  static constexpr int NST = ((TC_SMEM / CTAS - 1024) / STAGE) < 8 ? ((TC_SMEM / CTAS - 1024) / STAGE) : 8;
  static_assert(NST >= 2, "the ring needs two stages");
  static constexpr int TMEM_COLS = NT < 32 ? 32 : NT;
  static constexpr int SMEM = 1024 + NST * STAGE;
};

template <int NT>
__global__ void __launch_bounds__(128, TcCfg<NT>::CTAS)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, int T,
                   int ktiles, int kt_per_split, float* __restrict__ P, int ldp, int* err) {
  using Cfg = TcCfg<NT>;
  constexpr int NST = Cfg::NST;
  extern __shared__ unsigned char tc_dyn[];
  __shared__ uint64_t full[NST], empty[NST], done;
  __shared__ uint32_t tmem_s;
  __shared__ int fail;
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_dyn) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * TC_M;
  const int kt0 = blockIdx.y * kt_per_split;
  const int nk = max(0, min(ktiles, kt0 + kt_per_split) - kt0);
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fail = 0;
    fence_mbar_init();
  }
  if (warp == 1) tc5_alloc(&tmem_s, Cfg::TMEM_COLS);
  tc5_fence_before();
  __syncthreads();
  tc5_fence_after();
  const uint32_t tmem = tmem_s;
  if (tid == 0) {
    // producer
    int i = 0;
    for (; i < nk; ++i) {
      const int s = i % NST;
      const uint32_t round = (uint32_t)(i / NST);
      if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1u)) {
        atomicExch(&fail, 1);
        break;
      }
      unsigned char* st = sm + s * Cfg::STAGE;
      mbar_arrive_expect_tx(&full[s], (uint32_t)Cfg::STAGE);
      const int k0 = (kt0 + i) * TC_K;
      tma_load_2d(st, &wmap, k0, n0, &full[s]);
      tma_load_2d(st + TC_WTILE, &xmap, k0, 0, &full[s]);
    }
    // no copy may outlive the CTA: wait (bounded) for the last round of every stage
    for (int r = i > NST ? i - NST : 0; r < i; ++r) mbar_wait(&full[r % NST], (uint32_t)(r / NST) & 1u);
  } else if (tid == 32) {
    // MMA issuer
    const uint32_t sa0 = smem_u32(sm);
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int s = i % NST;
      if (!mbar_wait(&full[s], (uint32_t)(i / NST) & 1u)) {
        ok = false;
        break;
      }
      tc5_fence_after();
      const uint32_t sa = sa0 + s * Cfg::STAGE, sb = sa + TC_WTILE;
#pragma unroll
      for (int kk = 0; kk < TC_K / 16; ++kk)
        tc5_mma(tmem, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), f16_idesc(TC_M, NT), (i | kk) != 0);
      tc5_commit(&empty[s]);
    }
    tc5_commit(&done);  // arrives when every MMA issued above has completed
    if (!ok) atomicExch(&fail, 1);
  }
  __syncwarp();
  bool ok = nk == 0 || mbar_wait(&done, 0);
  tc5_fence_after();
  // epilogue: thread = weight row m (tensor-memory lane); column 3t + p holds
  // piece p of token t, summed as (hi + mid) + lo
  const int m = warp * 32 + lane;
  const int xr = TC_NP * T;
  float* dst = P + (int64_t)blockIdx.y * TC_TMAX * ldp + n0 + m;
  float acc = 0.0f;
#pragma unroll 1
  for (int c0 = 0; c0 < xr; c0 += 16) {
    uint32_t v[16];
    tc5_ld16_async(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
    tc5_ld_wait();
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const int col = c0 + q;
      if (col >= xr) break;
      const int p = col % TC_NP;
      acc = p == 0 ? __uint_as_float(v[q]) : __fadd_rn(acc, __uint_as_float(v[q]));
      if (p == TC_NP - 1) dst[(int64_t)(col / TC_NP) * ldp] = nk > 0 && ok ? acc : 0.0f;
    }
  }
  tc5_fence_before();
  __syncthreads();
  if (warp == 1) tc5_dealloc(tmem, Cfg::TMEM_COLS);
  if (tid == 0 && (!ok || fail)) atomicOr(err, DERR_TIMEOUT);
}

// x[T][n] f32 -> three bf16 pieces, row 3t + p of [3 * TC_TMAX][ld] holding
// piece p of token t, with x = hi + mid + lo exactly (each piece holds the
// next 8 significant bits); columns >= n are zero.
__global__ void split3_kernel(const float* __restrict__ x, int T, int n, int ldx, __nv_bfloat16* __restrict__ out,
                              int ld) {
  const int t = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ld; i += gridDim.x * blockDim.x) {
    const float v = (t < T && i < n) ? x[(int64_t)t * ldx + i] : 0.0f;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const float r1 = __fsub_rn(v, to_f(hi));
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const float r2 = __fsub_rn(r1, to_f(mid));
    const __nv_bfloat16 lo = __float2bfloat16_rn(r2);
    const int64_t o = (int64_t)(TC_NP * t) * ld + i;
    out[o] = hi;
    out[o + ld] = mid;
    out[o + 2 * (int64_t)ld] = lo;
  }
}

// y[t][j] = act(sum over splits of P[s][t][j] + bias[j]) for t < T, j < n;
// act 0 = ReLU (f32::max against 0), 1 = sigmoid, 2 = none; bias nullable.
// With xs_next, the result
// is also written as the next layer's three bf16 pieces (rows 3t .. 3t+2 of
// [3 * TC_TMAX][ld_next], columns n .. ld_next-1 zero).
__global__ void splitk_finish_kernel(const float* __restrict__ P, int splits, int ldp, const float* __restrict__ bias,
                                     int T, int n, int act, float* __restrict__ y, int ldy,
                                     __nv_bfloat16* __restrict__ xs_next, int ld_next) {
  const int t = blockIdx.y;
  const int lim = xs_next ? ld_next : n;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < lim; j += gridDim.x * blockDim.x) {
    float v = 0.0f;
    if (j < n) {
      float s = 0.0f;
      for (int q = 0; q < splits; ++q) s = __fadd_rn(s, P[((int64_t)q * TC_TMAX + t) * ldp + j]);
      v = bias ? __fadd_rn(s, bias[j]) : s;
      if (act == 0) v = fmaxf(v, 0.0f);
      else if (act == 1) v = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
      y[(int64_t)t * ldy + j] = v;
    }
    if (xs_next) {
      const int64_t o = (int64_t)(TC_NP * t) * ld_next + j;
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      const float r1 = __fsub_rn(v, to_f(hi));
      const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
      xs_next[o] = hi;
      xs_next[o + ld_next] = mid;
      xs_next[o + 2 * (int64_t)ld_next] = __float2bfloat16_rn(__fsub_rn(r1, to_f(mid)));
    }
  }
}

// y[t][j] = act(x[t] . W[j] + bias[j]) for a few tokens (TT <= GV_TMAX) on the
// CUDA cores: one warp per weight row, the row streamed once with 16-byte
// loads (8 bf16 per lane per chunk, GV_UNROLL chunks in flight), each bf16
// widened exactly by a 16-bit shift, f32 FMA accumulation, a shuffle-tree
// reduction.  x is staged once per block in shared memory as f32 [TT][ldw]
// (zero beyond d).  At one token the weight stream is the whole cost, so this
// replaces the tensor-core GEMM, its split-K scratch and its finish pass.
// act as in splitk_finish_kernel.
constexpr int GV_TMAX = 4;
constexpr int GV_WARPS = 4;
constexpr int GV_UNROLL = 8;
template <int TT>
__global__ void __launch_bounds__(GV_WARPS * 32)
    gemv_kernel(const float* __restrict__ x, int ldx, int d, const __nv_bfloat16* __restrict__ W, int ldw, int n,
                const float* __restrict__ bias, int act, float* __restrict__ y, int ldy) {
  extern __shared__ float4 gv_smem[];
  float* xs = reinterpret_cast<float*>(gv_smem);
  for (int i = threadIdx.x; i < TT * ldw; i += blockDim.x) {
    const int t = i / ldw, c = i - t * ldw;
    xs[i] = c < d ? x[(int64_t)t * ldx + c] : 0.0f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nch = ldw >> 3;  // 16-byte chunks per row (ldw is a multiple of 64)
  for (int j = blockIdx.x * GV_WARPS + warp; j < n; j += gridDim.x * GV_WARPS) {
    const uint4* wr = reinterpret_cast<const uint4*>(W + (int64_t)j * ldw);
    float acc[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) acc[t] = 0.0f;
    for (int c0 = lane; c0 < nch; c0 += 32 * GV_UNROLL) {
      uint4 q[GV_UNROLL];
#pragma unroll
      for (int u = 0; u < GV_UNROLL; ++u) {
        const int c = c0 + 32 * u;
        q[u] = c < nch ? __ldg(wr + c) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < GV_UNROLL; ++u) {
        const int c = c0 + 32 * u;
        if (c >= nch) break;
        const uint32_t wv[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          const float4* xv = reinterpret_cast<const float4*>(xs + (size_t)t * ldw + (size_t)c * 8);
          const float4 a = xv[0], b = xv[1];
          const float xe[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            acc[t] = fmaf(__uint_as_float(wv[h] << 16), xe[2 * h], acc[t]);
            acc[t] = fmaf(__uint_as_float(wv[h] & 0xffff0000u), xe[2 * h + 1], acc[t]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      float v = acc[t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) {
        if (bias) v = __fadd_rn(v, bias[j]);
        if (act == 0) v = fmaxf(v, 0.0f);
        else if (act == 1) v = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
        y[(int64_t)t * ldy + j] = v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// select_top_k (mlp_predictor.rs:126-132): the k largest scores of a row in
// (score descending, index ascending) order -- the stable sort's order.  One
// block per token, the row staged in shared memory:
//  1. min / max of the row;
//  2. a histogram over TK_NB equal-width bins of [min, max]; the bin map
//     (v - min) * scale, truncated, is monotonic in v, so every key of a
//     higher bin is larger than every key of a lower one;
//  3. a scan from the top bin finds bin b* where the count reaches k;
//  4. keys of bins above b* are taken, and the keys of b* are ranked exactly
//     among themselves (score desc, index asc) to take the rest;
//  5. a bitonic sort of (~score bits, index) orders the k taken keys.
// Scores are sigmoid outputs: non-negative and finite, so their bit
// patterns order like their values.
// ---------------------------------------------------------------------------
constexpr int TK_NT = 1024;
constexpr int TK_NB = 4096;
constexpr int TK_MAXC = 2048;  // candidates of the threshold bin ranked in shared memory

__global__ void __launch_bounds__(TK_NT) topk_kernel(const float* __restrict__ scores, int n, int lds, int k,
                                                     uint32_t* __restrict__ idx, int ldi, int pow2, int sorted) {
  extern __shared__ __align__(1024) unsigned char tk_smem[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(tk_smem);  // [pow2]
  float* row = reinterpret_cast<float*>(keys + pow2);     // [n]
  __shared__ uint32_t hist[TK_NB];
  __shared__ uint64_t cands[TK_MAXC];
  __shared__ float red_mn[TK_NT / 32], red_mx[TK_NT / 32];
  __shared__ uint32_t wsum[TK_NT / 32];
  __shared__ int bstar_s;
  __shared__ uint32_t above_s, n_taken, n_cand;
  const int t = blockIdx.x, tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const float* grow = scores + (int64_t)t * lds;
  float mn = INFINITY, mx = -INFINITY;
  if ((n & 3) == 0 && (lds & 3) == 0 && (reinterpret_cast<uintptr_t>(scores) & 15) == 0) {  // 16-byte loads
    for (int i = tid * 4; i < n; i += TK_NT * 4) {
      const float4 v = *reinterpret_cast<const float4*>(grow + i);
      *reinterpret_cast<float4*>(row + i) = v;
      mn = fminf(mn, fminf(fminf(v.x, v.y), fminf(v.z, v.w)));
      mx = fmaxf(mx, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    }
  } else {
    for (int i = tid; i < n; i += TK_NT) {
      const float v = grow[i];
      row[i] = v;
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
  }
  for (int i = tid; i < TK_NB; i += TK_NT) hist[i] = 0;
  for (int i = tid; i < pow2; i += TK_NT) keys[i] = ~0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (l == 0) {
    red_mn[w] = mn;
    red_mx[w] = mx;
  }
  if (tid == 0) {
    n_taken = 0;
    n_cand = 0;
  }
  __syncthreads();
  mn = red_mn[0];
  mx = red_mx[0];
  for (int q = 1; q < TK_NT / 32; ++q) {
    mn = fminf(mn, red_mn[q]);
    mx = fmaxf(mx, red_mx[q]);
  }
  const float scale = mx > mn ? (float)(TK_NB - 1) / (mx - mn) : 0.0f;
  auto bin_of = [&](float v) { return min(TK_NB - 1, (int)__fmul_rz(__fsub_rz(v, mn), scale)); };
  for (int i = tid; i < n; i += TK_NT) atomicAdd(&hist[bin_of(row[i])], 1u);
  __syncthreads();
  // suffix counts: thread j owns bins TK_NB-1-4j .. TK_NB-4-4j (descending)
  {
    uint32_t c[4], tot = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      c[q] = hist[TK_NB - 1 - 4 * tid - q];
      tot += c[q];
    }
    uint32_t incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (l >= o) incl += v;
    }
    if (l == 31) wsum[w] = incl;
    __syncthreads();
    uint32_t wbase = 0;
    for (int q = 0; q < w; ++q) wbase += wsum[q];
    const uint32_t before = wbase + incl - tot;  // keys in higher bins than this thread's
    if (before < (uint32_t)k && before + tot >= (uint32_t)k) {
      uint32_t run = before;
      for (int q = 0; q < 4; ++q) {
        if (run + c[q] >= (uint32_t)k) {
          bstar_s = TK_NB - 1 - 4 * tid - q;
          above_s = run;
          break;
        }
        run += c[q];
      }
    }
  }
  __syncthreads();
  const int bstar = bstar_s;
  const uint32_t above = above_s, need = (uint32_t)k - above;
  // keys above b*: taken in any order; keys of b*: candidates, ranked
  // exactly among themselves (score desc, index asc) for the remaining slots
  // warp-aggregated appends: one shared-memory atomic per warp and list
  for (int i0 = 0; i0 < n; i0 += TK_NT) {
    const int i = i0 + tid;
    const float v = i < n ? row[i] : 0.0f;
    const int b = i < n ? bin_of(v) : -1;
    const uint64_t key = ((uint64_t)(~__float_as_uint(v)) << 32) | (uint32_t)i;
    const int pt = warp_append(b > bstar, &n_taken);
    if (pt >= 0) keys[pt] = key;
    const int pc = warp_append(b == bstar, &n_cand);
    if (pc >= 0 && pc < TK_MAXC) cands[pc] = key;
  }
  __syncthreads();
  const uint32_t nc = n_cand;
  if (nc <= TK_MAXC) {
    for (uint32_t ci = tid; ci < nc; ci += TK_NT) {
      const uint64_t key = cands[ci];
      uint32_t rank = 0;
      for (uint32_t j = 0; j < nc; ++j) rank += cands[j] < key;
      if (rank < need) keys[above + rank] = key;
    }
  } else {  // a bin holding very many equal or near-equal scores: rank against the whole row
    for (int i = tid; i < n; i += TK_NT) {
      const float v = row[i];
      if (bin_of(v) != bstar) continue;
      const uint64_t key = ((uint64_t)(~__float_as_uint(v)) << 32) | (uint32_t)i;
      uint32_t rank = 0;
      for (int j = 0; j < n; ++j) {
        const float u = row[j];
        if (bin_of(u) == bstar) rank += (((uint64_t)(~__float_as_uint(u)) << 32) | (uint32_t)j) < key;
      }
      if (rank < need) keys[above + rank] = key;
    }
  }
  __syncthreads();
  if (!sorted) {
    // the selected set in ascending index order: a bitmap over the row (in the
    // histogram's words, free now) and a block scan of its popcounts
    __shared__ int scan_tmp[33];
    const int nwd = (n + 31) / 32;  // <= TK_NB (n <= 131072)
    for (int i = tid; i < nwd; i += TK_NT) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < k; i += TK_NT) {
      const uint32_t id = (uint32_t)(keys[i] & 0xffffffffu);
      atomicOr(&hist[id >> 5], 1u << (id & 31));
    }
    __syncthreads();
    const int WPT = (nwd + TK_NT - 1) / TK_NT;  // words per thread, contiguous
    int c = 0;
    for (int q = 0; q < WPT; ++q) {
      const int wi = tid * WPT + q;
      if (wi < nwd) c += __popc(hist[wi]);
    }
    int tot;
    int pos = block_excl_scan<TK_NT>(c, scan_tmp, &tot);
    for (int q = 0; q < WPT; ++q) {
      const int wi = tid * WPT + q;
      if (wi >= nwd) break;
      uint32_t bits = hist[wi];
      while (bits) {
        const int b = __ffs(bits) - 1;
        bits &= bits - 1;
        idx[(int64_t)t * ldi + pos++] = (uint32_t)(wi * 32 + b);
      }
    }
    return;
  }
  // bitonic sort ascending of keys[0, pow2)
  if (pow2 == 2 * TK_NT) {
    // two keys per thread (elements 2*tid, 2*tid+1; warp w holds 64w ..
    // 64w+63): strides below 64 in registers and shuffles, larger strides
    // through shared memory
    uint64_t v0 = keys[2 * tid], v1 = keys[2 * tid + 1];
    for (int size = 2; size <= pow2; size <<= 1) {
      int stride = size >> 1;
      if (stride >= 64) {
        keys[2 * tid] = v0;
        keys[2 * tid + 1] = v1;
        __syncthreads();
        for (; stride >= 64; stride >>= 1) {
          const int i = (tid / stride) * 2 * stride + (tid % stride), j = i + stride;
          const bool up = (i & size) == 0;
          const uint64_t a = keys[i], b = keys[j];
          if ((a > b) == up) {
            keys[i] = b;
            keys[j] = a;
          }
          __syncthreads();
        }
        v0 = keys[2 * tid];
        v1 = keys[2 * tid + 1];
        __syncthreads();
      }
      for (; stride >= 2; stride >>= 1) {
        const int lm = stride >> 1;  // partner lane offset
        const uint64_t o0 = __shfl_xor_sync(0xffffffffu, v0, lm), o1 = __shfl_xor_sync(0xffffffffu, v1, lm);
        const int e = 2 * tid;  // both keys share (e & stride) and (e & size)
        const bool keep_min = ((e & stride) == 0) == ((e & size) == 0);
        v0 = keep_min ? (v0 < o0 ? v0 : o0) : (v0 > o0 ? v0 : o0);
        v1 = keep_min ? (v1 < o1 ? v1 : o1) : (v1 > o1 ? v1 : o1);
      }
      {  // stride 1: the thread's own pair
        const bool up = ((2 * tid) & size) == 0;
        if ((v0 > v1) == up) {
          const uint64_t x = v0;
          v0 = v1;
          v1 = x;
        }
      }
    }
    keys[2 * tid] = v0;
    keys[2 * tid + 1] = v1;
    __syncthreads();
  } else {
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
  if ((hid & 3) == 0 && (ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {  // 16-byte loads
#pragma unroll 4
    for (int i = threadIdx.x * 4; i < ldw; i += blockDim.x * 4)
      *reinterpret_cast<float4*>(xs + i) =
          i < hid ? *reinterpret_cast<const float4*>(x + (int64_t)t * ldx + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  } else {
    for (int i = threadIdx.x; i < ldw; i += blockDim.x) xs[i] = i < hid ? x[(int64_t)t * ldx + i] : 0.0f;
  }
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
#pragma unroll 8
    for (int c = l; c < ldw / 8; c += 32) {
      const uint4 gr = g4[c], ur = u4[c];
      const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gr);
      const __nv_bfloat16* ue = reinterpret_cast<const __nv_bfloat16*>(&ur);
      const float4 xa = reinterpret_cast<const float4*>(xs)[2 * c], xb = reinterpret_cast<const float4*>(xs)[2 * c + 1];
      const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        g = fmaf(to_f(ge[q]), xv[q], g);
        u = fmaf(to_f(ue[q]), xv[q], u);
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

constexpr int DV_DN_T = 256;  // threads per block, 8 output columns each (16-byte row loads)
constexpr int DV_DN_C = 8 * DV_DN_T;
constexpr int DV_PF = 8;      // selected rows in flight per thread

__global__ void __launch_bounds__(DV_DN_T)
    dv_down_kernel(const __nv_bfloat16* __restrict__ downT, int hid, int ldw, const uint32_t* __restrict__ sel, int k,
                   int inter, const float* __restrict__ a, int splits, float* __restrict__ part) {
  const int t = blockIdx.z, sp = blockIdx.y;
  const int j0 = (blockIdx.x * DV_DN_T + threadIdx.x) * 8;
  const int per = (k + splits - 1) / splits;
  const int s0 = sp * per, s1 = min(k, s0 + per);
  if (j0 >= hid) return;
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
  for (int s = s0; s < s1; s += DV_PF) {
    uint4 wv[DV_PF];
    float av[DV_PF];
#pragma unroll
    for (int u = 0; u < DV_PF; ++u) {
      av[u] = 0.0f;
      if (s + u < s1) {
        uint32_t row = sel[(int64_t)t * k + s + u];
        if (row >= (uint32_t)inter) row = 0;
        wv[u] = *reinterpret_cast<const uint4*>(downT + (int64_t)row * ldw + j0);
        av[u] = a[(int64_t)t * k + s + u];
      }
    }
#pragma unroll
    for (int u = 0; u < DV_PF; ++u) {
      if (s + u < s1 && av[u] != 0.0f) {
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&wv[u]);
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = __fadd_rn(acc[c], __fmul_rn(to_f(e[c]), av[u]));
      }
    }
  }
  float4* dst = reinterpret_cast<float4*>(part + ((int64_t)t * splits + sp) * ldw + j0);
  dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

__global__ void dv_down_finish_kernel(const float* __restrict__ part, int splits, int hid, int ldw,
                                      const float* __restrict__ bias, float* __restrict__ out, int accumulate) {
  constexpr int FL = 32;  // partial sums in flight per thread, added in split order
  const int t = blockIdx.y;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < hid; j += gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int q0 = 0; q0 < splits; q0 += FL) {
      float v[FL];
#pragma unroll
      for (int u = 0; u < FL; ++u) v[u] = q0 + u < splits ? part[((int64_t)t * splits + q0 + u) * ldw + j] : 0.0f;
#pragma unroll
      for (int u = 0; u < FL; ++u)
        if (q0 + u < splits) s = __fadd_rn(s, v[u]);
    }
    const float v = bias ? __fadd_rn(s, bias[j]) : s;
    float* o = out + (int64_t)t * hid + j;
    *o = accumulate ? __fadd_rn(*o, v) : v;  // accumulate: the residual add h += mlp(x)
  }
}

// RMSNorm (klearu-llm model/rms_norm.rs): y = x * (1 / sqrt(mean(x^2) + eps))
// * w (or * (1 + w)), one block per token.  Each thread holds up to RN_V
// 4-element vectors of the row in registers, so the row is read once; the
// sum of squares is a block reduction (the reference sums sequentially:
// equal within f32 rounding).
constexpr int RN_NT = 1024, RN_V = 4;
__global__ void __launch_bounds__(RN_NT) rmsnorm_kernel(const float* x, int ld, int n, const float* w, float eps,
                                                        int one_plus, float* y) {
  __shared__ float red[RN_NT / 32];
  const int t = blockIdx.x;
  const float* xr = x + (int64_t)t * ld;
  const bool vec = (n & 3) == 0 && (ld & 3) == 0 && n <= RN_NT * 4 * RN_V &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) &
                    15) == 0;
  float4 v[RN_V];
  float ss = 0.f;
  if (vec) {
#pragma unroll
    for (int q = 0; q < RN_V; ++q) {
      const int i = (threadIdx.x + q * RN_NT) * 4;
      v[q] = i < n ? *reinterpret_cast<const float4*>(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int q = 0; q < RN_V; ++q) ss = fmaf(v[q].x, v[q].x, fmaf(v[q].y, v[q].y, fmaf(v[q].z, v[q].z, fmaf(v[q].w, v[q].w, ss))));
  } else {
    for (int i = threadIdx.x; i < n; i += RN_NT) ss = fmaf(xr[i], xr[i], ss);
  }
  ss = warp_sum_f(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float r = red[threadIdx.x];
    r = warp_sum_f(r);
    if (threadIdx.x == 0) red[0] = r;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(red[0] / (float)n + eps);
  float* yr = y + (int64_t)t * ld;
  if (vec) {
#pragma unroll
    for (int q = 0; q < RN_V; ++q) {
      const int i = (threadIdx.x + q * RN_NT) * 4;
      if (i < n) {
        float4 wv = *reinterpret_cast<const float4*>(w + i);
        if (one_plus) wv = make_float4(1.0f + wv.x, 1.0f + wv.y, 1.0f + wv.z, 1.0f + wv.w);
        *reinterpret_cast<float4*>(yr + i) =
            make_float4(v[q].x * inv * wv.x, v[q].y * inv * wv.y, v[q].z * inv * wv.z, v[q].w * inv * wv.w);
      }
    }
  } else {
    for (int i = threadIdx.x; i < n; i += RN_NT) {
      const float wi = one_plus ? 1.0f + w[i] : w[i];
      yr[i] = xr[i] * inv * wi;
    }
  }
}
__global__ void residual_add_kernel(float* h, const float* d, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) h[i] += d[i];
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

// K splits of the tcgen05 linear: as many CTAs as fit in one wave
// (ctas_per_sm per SM), at least two K tiles per split.  *per = K tiles per
// split.
int tc_linear_splits(int n, int ldw, int* per, int ctas_per_sm) {
  const int ntile = (int)ceil_div(n, TC_M);
  const int ktiles = ldw / TC_K;
  int splits = std::max(1, std::min(std::min(32, ktiles / 2), sm_count() * ctas_per_sm / ntile));
  const int p = (int)ceil_div(ktiles, splits);
  if (per) *per = p;
  return (int)ceil_div(ktiles, p);
}
size_t tc_linear_scratch_floats(int n, int ldw) {
  return (size_t)tc_linear_splits(n, ldw, nullptr, 2) * TC_TMAX * ceil_div(n, TC_M) * TC_M;
}

template <int NT>
static void tc_gemm_launch(dim3 grid, const __nv_bfloat16* W, int ldw, int nw, const __nv_bfloat16* xs, int T,
                           int ktiles, int per, float* P, int ldp, int* err, cudaStream_t st) {
  using Cfg = TcCfg<NT>;
  static OncePerDevice attr;
  attr([&] {
    cudaFuncSetAttribute(tc_gemm_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
  });
  CUtensorMap wmap, xmap;
  if (!tma_map_bf16(&wmap, W, nw, ldw, ldw, TC_K, TC_M) ||
      !tma_map_bf16(&xmap, xs, TC_NP * TC_TMAX, ldw, ldw, TC_K, NT)) {
    flag_error(err, DERR_TMA, st);
    return;
  }
  tc_gemm_kernel<NT><<<grid, 128, Cfg::SMEM, st>>>(wmap, xmap, T, ktiles, per, P, ldp, err);
}

// y[T][n] = act(x[T][d] . W^T + b) through the tcgen05 GEMM; T <= TC_TMAX.
// W: [n][ldw] bf16 (ldw a multiple of 64, zero beyond d).  xs: the split
// activations [3][128][ldw] bf16 -- written here from x, or, when x is
// null, already written by the previous layer's finish.  P: split-K scratch.
// xs_next (nullable): where the finish writes y's pieces for the next layer.
void launch_tc_linear(const float* x, int T, int d, int ldx, const __nv_bfloat16* W, int n, int ldw,
                      const float* bias, int act, float* y, int ldy, __nv_bfloat16* xs, float* P,
                      __nv_bfloat16* xs_next, int ld_next, int* err, cudaStream_t st) {
  if (x) {
    split3_kernel<<<dim3((unsigned)ceil_div(ldw, 256), T), 256, 0, st>>>(x, T, d, ldx, xs, ldw);
    count_launch();
  }
  const int ntile = (int)ceil_div(n, TC_M);
  const int ktiles = ldw / TC_K;
  const int xr = TC_NP * T;  // token-piece rows: the MMA's N, rounded up to 16
  int per = 0;
  const int splits = tc_linear_splits(n, ldw, &per, xr <= 64 ? 2 : 1);
  const int ldp = ntile * TC_M;
  const dim3 grid(ntile, splits);
  if (xr <= 16) tc_gemm_launch<16>(grid, W, ldw, n, xs, T, ktiles, per, P, ldp, err, st);
  else if (xr <= 32) tc_gemm_launch<32>(grid, W, ldw, n, xs, T, ktiles, per, P, ldp, err, st);
  else if (xr <= 64) tc_gemm_launch<64>(grid, W, ldw, n, xs, T, ktiles, per, P, ldp, err, st);
  else if (xr <= 128) tc_gemm_launch<128>(grid, W, ldw, n, xs, T, ktiles, per, P, ldp, err, st);
  else tc_gemm_launch<256>(grid, W, ldw, n, xs, T, ktiles, per, P, ldp, err, st);
  count_launch();
  const int lim = xs_next ? ld_next : n;
  splitk_finish_kernel<<<dim3((unsigned)ceil_div(lim, 256), T), 256, 0, st>>>(P, splits, ldp, bias, T, n, act, y, ldy,
                                                                            xs_next, ld_next);
  count_launch();
}

int gemv_linear_max_tokens() { return GV_TMAX; }

template <int TT>
static void gemv_launch(const float* x, int ldx, int d, const __nv_bfloat16* W, int n, int ldw, const float* bias,
                        int act, float* y, int ldy, cudaStream_t st) {
  const size_t sm = (size_t)TT * ldw * 4;
  static OncePerDevice attr;
  attr([&] { cudaFuncSetAttribute(gemv_kernel<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); });
  // enough warps to keep every SM's load queue full, and no more blocks than
  // rows need (each block stages x once)
  const int blocks = (int)std::min<int64_t>(ceil_div(n, GV_WARPS), (int64_t)sm_count() * 8);
  gemv_kernel<TT><<<blocks, GV_WARPS * 32, sm, st>>>(x, ldx, d, W, ldw, n, bias, act, y, ldy);
}

void launch_gemv_linear(const float* x, int T, int d, int ldx, const __nv_bfloat16* W, int n, int ldw,
                        const float* bias, int act, float* y, int ldy, cudaStream_t st) {
  if (T == 1) gemv_launch<1>(x, ldx, d, W, n, ldw, bias, act, y, ldy, st);
  else if (T == 2) gemv_launch<2>(x, ldx, d, W, n, ldw, bias, act, y, ldy, st);
  else if (T == 3) gemv_launch<3>(x, ldx, d, W, n, ldw, bias, act, y, ldy, st);
  else gemv_launch<4>(x, ldx, d, W, n, ldw, bias, act, y, ldy, st);
  count_launch();
}

void launch_topk(const float* scores, int T, int n, int lds, int k, uint32_t* idx, int ldi, cudaStream_t st,
                 bool sorted) {
  int pow2 = 2 * TK_NT;  // at least the register-sorted size
  while (pow2 < k) pow2 <<= 1;
  const size_t sm = (size_t)pow2 * 8 + (size_t)n * 4;
  static OncePerDevice attr;
  attr([&] {  // the kernel's static shared memory (~34 KB) counts against the 227 KB per block
    cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 190 * 1024);
  });
  topk_kernel<<<T, TK_NT, sm, st>>>(scores, n, lds, k, idx, ldi, pow2, sorted ? 1 : 0);
  count_launch();
}

namespace {
// mask[t][i] = 1 for the selected neurons of token t (mask zeroed before)
__global__ void dv_mask_kernel(const uint32_t* __restrict__ sel, int k, int inter, uint8_t* __restrict__ mask) {
  const int t = blockIdx.y;
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < k; s += gridDim.x * blockDim.x) {
    const uint32_t i = sel[(int64_t)t * k + s];
    if (i < (uint32_t)inter) mask[(int64_t)t * inter + i] = 1;
  }
}
// h[t][i] = mask ? silu(g) * u : 0, written as the down projection's three
// bf16 pieces (rows 3t .. 3t+2 of [3 * TC_TMAX][ldh], columns >= inter zero);
// the mask is cleared for the next call
__global__ void dv_swiglu_mask_kernel(const float* __restrict__ G, const float* __restrict__ U, int inter,
                                      uint8_t* __restrict__ mask, __nv_bfloat16* __restrict__ hs, int ldh) {
  const int t = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ldh; i += gridDim.x * blockDim.x) {
    float v = 0.0f;
    if (i < inter && mask[(int64_t)t * inter + i]) {
      const float g = G[(int64_t)t * inter + i], u = U[(int64_t)t * inter + i];
      v = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
      mask[(int64_t)t * inter + i] = 0;
    }
    const int64_t o = (int64_t)(TC_NP * t) * ldh + i;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const float r1 = __fsub_rn(v, to_f(hi));
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    hs[o] = hi;
    hs[o + ldh] = mid;
    hs[o + 2 * (int64_t)ldh] = __float2bfloat16_rn(__fsub_rn(r1, to_f(mid)));
  }
}
}  // namespace

// The selection as a mask over dense tensor-core GEMMs: G = gate . x,
// U = up . x over all neurons, h = silu(G) * U on the selected neurons and 0
// elsewhere, out = down . h (+ bias).  The zero terms leave every sum
// unchanged, so this equals the per-token gather; it reads each weight once
// per call instead of once per token.  T <= TC_TMAX.
void launch_sparse_mlp_dense(const __nv_bfloat16* gate, const __nv_bfloat16* up, const __nv_bfloat16* down,
                             int hid, int ldg, int inter, int ldd, const float* bias, const float* x, int T,
                             const uint32_t* sel, int k, float* G, float* U, uint8_t* mask, __nv_bfloat16* xs,
                             __nv_bfloat16* hs, float* P, float* out, int* err, cudaStream_t st) {
  // x's pieces once for gate and up
  split3_kernel<<<dim3((unsigned)ceil_div(ldg, 256), T), 256, 0, st>>>(x, T, hid, hid, xs, ldg);
  count_launch();
  launch_tc_linear(nullptr, T, hid, hid, gate, inter, ldg, nullptr, 2, G, inter, xs, P, nullptr, 0, err, st);
  launch_tc_linear(nullptr, T, hid, hid, up, inter, ldg, nullptr, 2, U, inter, xs, P, nullptr, 0, err, st);
  dv_mask_kernel<<<dim3((unsigned)ceil_div(k, 256), T), 256, 0, st>>>(sel, k, inter, mask);
  count_launch();
  dv_swiglu_mask_kernel<<<dim3((unsigned)ceil_div(ldd, 256), T), 256, 0, st>>>(G, U, inter, mask, hs, ldd);
  count_launch();
  launch_tc_linear(nullptr, T, inter, inter, down, hid, ldd, bias, 2, out, hid, hs, P, nullptr, 0, err, st);
}

void launch_sparse_mlp(const __nv_bfloat16* gate, const __nv_bfloat16* up, const __nv_bfloat16* downT, int hid,
                       int ldw, int inter, const float* bias, const float* x, int T, const uint32_t* sel, int k,
                       float* a, float* part, int splits, float* out, bool accumulate, int* err,
                       cudaStream_t st) {
  const int gblocks = std::max(1, std::min((int)ceil_div(k, DV_WARPS), (int)ceil_div(sm_count() * 4, T)));
  dv_gateup_kernel<<<dim3(gblocks, T), DV_WARPS * 32, (size_t)ldw * 4, st>>>(gate, up, hid, ldw, x, hid, sel, k,
                                                                             inter, a, err);
  count_launch();
  dv_down_kernel<<<dim3((unsigned)ceil_div(hid, DV_DN_C), splits, T), DV_DN_T, 0, st>>>(downT, hid, ldw, sel, k,
                                                                                       inter, a, splits, part);
  count_launch();
  dv_down_finish_kernel<<<dim3((unsigned)ceil_div(hid, 256), T), 256, 0, st>>>(part, splits, hid, ldw, bias, out,
                                                                            accumulate ? 1 : 0);
  count_launch();
}

void launch_rmsnorm(const float* x, int T, int n, const float* w, float eps, int one_plus, float* y,
                    cudaStream_t st) {
  if (T <= 0) return;
  rmsnorm_kernel<<<T, RN_NT, 0, st>>>(x, n, n, w, eps, one_plus, y);
  count_launch();
}
void launch_residual_add(float* h, const float* d, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  residual_add_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(h, d, n);
  count_launch();
}

}  // namespace kl
