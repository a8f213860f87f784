// layer.cu -- SLIDE layer kernels: active-row forward (gather + sequential f32
// dot), fused loss gradient and input gradient, softmax, and the sort-free
// segmented gradient reduction fused with lazy Adam / SGD.
//
// Reference (crates/klearu-core/src):
//  * Layer::forward (network/layer.rs:65-120), Neuron::forward
//    (network/neuron.rs:47-62): pre = sequential f32 sum of w*x, then + bias.
//    The kernels keep that order and use non-contracted __fmul_rn/__fadd_rn,
//    so pre-activations are bit-identical to the reference's.
//  * compute_loss / compute_loss_gradient (network/net.rs:180-230).
//  * Layer::backward (network/layer.rs:124-225): local gradients, the input
//    gradient from the rows BEFORE their update, per-row optimizer update.
//  * Adam::update (optim/adam.rs:27-76), Sgd::update (optim/sgd.rs:17-58):
//    evaluated with the same f32 operation sequence (IEEE div/sqrt, no FMA).
//  * Bf16Weights::update_from_f32 (klearu-accel/src/bf16/mod.rs:85-88):
//    bf16 rows are updated as bf16_rne(f32(w) + delta).
#include "engine.h"

namespace kl {
namespace {

template <class W>
__device__ __forceinline__ float wload(const void* base, int64_t off) {
  return to_f(static_cast<const W*>(base)[off]);
}

__device__ __forceinline__ float block_reduce_max_f(float v, float* tmp) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
  if (l == 0) tmp[w] = v;
  __syncthreads();
  if (w == 0) {
    float x = l < nw ? tmp[l] : __int_as_float(0xff800000);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(FULL, x, o));
    if (l == 0) tmp[32] = x;
  }
  __syncthreads();
  float r = tmp[32];
  __syncthreads();
  return r;
}
__device__ __forceinline__ float block_reduce_sum_f(float v, float* tmp) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  v = warp_sum_f(v);
  if (l == 0) tmp[w] = v;
  __syncthreads();
  if (w == 0) {
    float x = l < nw ? tmp[l] : 0.0f;
    x = warp_sum_f(x);
    if (l == 0) tmp[32] = x;
  }
  __syncthreads();
  float r = tmp[32];
  __syncthreads();
  return r;
}

// Optimizer step on one element (adam.rs:57-68 / sgd.rs:38-42).
__device__ __forceinline__ void opt_apply(float& w, float& m, float& v, float g, const OptStep& o) {
  if (o.opt == KL_OPT_ADAM) {
    m = __fadd_rn(__fmul_rn(o.b1, m), __fmul_rn(o.omb1, g));
    v = __fadd_rn(__fmul_rn(o.b2, v), __fmul_rn(__fmul_rn(o.omb2, g), g));
    // m == 0 makes the step lr * 0 / (sqrt(v_hat) + eps) a zero, so w keeps
    // its value (up to the sign of a zero weight); skipping the IEEE divisions
    // and sqrt is exact and keeps never-updated elements (m = v = 0) off the
    // slow paths of division and square root by zero.
    if (m == 0.0f) return;
    const float mh = __fdiv_rn(m, o.c1);
    const float vh = __fdiv_rn(v, o.c2);
    const float q = __fdiv_rn(__fmul_rn(o.lr, mh), __fadd_rn(__fsqrt_rn(vh), o.eps));
    w = __fadd_rn(w, -q);
  } else {
    const float vv = __fsub_rn(__fmul_rn(o.mom, m), __fmul_rn(o.lr, g));
    m = vv;
    w = __fadd_rn(w, vv);
  }
}

// ---------------------------------------------------------------------------
// Feature-major forward over CSR rows: block per sample, thread per active
// neuron (<= 1024 actives: up to 8 per thread).
// ---------------------------------------------------------------------------
template <class W>
__global__ void __launch_bounds__(128) fm_forward_kernel(const void* Wm, int ldw, int d,
                                                         const float* bias, int act, SparseIn in,
                                                         ActiveSet A, float* h, int ldh, int* err, int ch,
                                                         int gather) {
  // chunks of `ch` nonzeros: their whole feature rows (ldw weights each, one
  // contiguous line per nonzero) are staged in shared memory with coalesced,
  // independent 16-byte loads; then each active neuron's thread sums its
  // chain in nonzero order (bit-exact) from shared memory.
  constexpr int NT = 128, MAXJ = 8;
  extern __shared__ __align__(16) unsigned char dyn[];
  uint32_t* sidx = reinterpret_cast<uint32_t*>(dyn);
  const int chx = max(ch, 64);  // capacity of sidx / sval (64 in gather mode)
  float* sval = reinterpret_cast<float*>(sidx + chx);
  W* wt = reinterpret_cast<W*>(dyn + round_up((int64_t)chx * 8, 16));  // [ch][ldw]
  const int s = blockIdx.x;
  const int na = min(A.cnt[s], NT * MAXJ);
  // gather mode (see below) when this example's active neurons are few
  const bool use_gather = gather && (int64_t)na * 8 <= (int64_t)ldw;
  if (use_gather) ch = 64;
  const uint32_t* ids = A.ids + (int64_t)s * A.stride;
  float acc[MAXJ];
  uint32_t myid[MAXJ];
#pragma unroll
  for (int j = 0; j < MAXJ; ++j) {
    const int a = threadIdx.x + j * NT;
    myid[j] = a < na ? ids[a] : 0u;
    acc[j] = 0.0f;
  }
  const int beg = in.rowptr[s], end = in.rowptr[s + 1];
  const int vpr = (int)(((int64_t)ldw * sizeof(W)) / 16);  // 16-byte vectors per feature row
  for (int c0 = beg; c0 < end; c0 += ch) {
    const int m = min(ch, end - c0);
    for (int e = threadIdx.x; e < m; e += NT) {
      uint32_t col = in.idx[c0 + e];
      if (col >= (uint32_t)d) {
        atomicOr(err, DERR_BOUNDS);
        col = 0xffffffffu;
      }
      sidx[e] = col;
      sval[e] = in.val[c0 + e];
    }
    __syncthreads();
    if (use_gather) {
      // Wide rows with few active neurons (a dense input: every row is a
      // nonzero): each thread loads only its neurons' weights of the chunk's
      // rows, 32 independent loads ahead of the ordered sum.
#pragma unroll
      for (int j = 0; j < MAXJ; ++j) {
        const int a = threadIdx.x + j * NT;
        if (a < na) {
          float x = acc[j];
          const W* col = static_cast<const W*>(Wm) + myid[j];
          for (int e0 = 0; e0 < m; e0 += 32) {
            float wv[32];
#pragma unroll
            for (int u = 0; u < 32; ++u) {
              const uint32_t r = e0 + u < m ? sidx[e0 + u] : 0xffffffffu;
              wv[u] = r != 0xffffffffu ? to_f(col[(int64_t)r * ldw]) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 32; ++u)
              if (e0 + u < m && sidx[e0 + u] != 0xffffffffu) x = __fadd_rn(x, __fmul_rn(wv[u], sval[e0 + u]));
          }
          acc[j] = x;
        }
      }
      __syncthreads();
      continue;
    }
    for (int q0 = threadIdx.x; q0 < m * vpr; q0 += 4 * NT) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = q0 + u * NT;
        v[u] = make_uint4(0, 0, 0, 0);
        if (q < m * vpr) {
          const int e = q / vpr, c = q - e * vpr;
          const uint32_t col = sidx[e];
          if (col != 0xffffffffu) v[u] = reinterpret_cast<const uint4*>(static_cast<const W*>(Wm) + (int64_t)col * ldw)[c];
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (q0 + u * NT < m * vpr) reinterpret_cast<uint4*>(wt)[q0 + u * NT] = v[u];
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < MAXJ; ++j) {
      const int a = threadIdx.x + j * NT;
      if (a < na) {
        float x = acc[j];
        for (int e = 0; e < m; ++e) {
          if (sidx[e] == 0xffffffffu) continue;
          x = __fadd_rn(x, __fmul_rn(to_f(wt[(int64_t)e * ldw + myid[j]]), sval[e]));
        }
        acc[j] = x;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < MAXJ; ++j) {
    const int a = threadIdx.x + j * NT;
    if (a < na) {
      const float pre = __fadd_rn(acc[j], bias[myid[j]]);
      const float post = act == KL_ACT_SOFTMAX ? pre : act_apply(pre, act);
      A.pre[(int64_t)s * A.stride + a] = pre;
      A.post[(int64_t)s * A.stride + a] = post;
      if (h && act != KL_ACT_SOFTMAX) h[(int64_t)s * ldh + myid[j]] = post;
    }
  }
}

// ---------------------------------------------------------------------------
// Row-major active-row kernel.  Block = 8 warps x 32 active rows; grid =
// (row chunks, samples).  Each warp stages its 32 gathered rows, one
// TILEB-byte column tile at a time, into shared memory with 16-byte cp.async
// (coalesced: consecutive lanes fetch consecutive 16-byte pieces of a row).
// Lane r then computes row r's dot product sequentially from shared memory
// (bit-exact reference order); in FUSED mode it also forms the loss gradient
// and the warp accumulates dX = sum_r lg_r * W_r from the same staged tile,
// so every row is read from HBM once for forward + input gradient.
// ---------------------------------------------------------------------------
constexpr int RM_NWB = RM_RPB / 32;

template <class W, int TILEB>
__device__ __forceinline__ void rm_load_tile(unsigned char* mt, const unsigned char* Wb,
                                             int64_t rowbytes, int tI, uint32_t myid, int nw) {
  constexpr int CPR = TILEB / 16;
  constexpr int PITCH = TILEB + 16;
  const int l = threadIdx.x & 31;
#pragma unroll 4
  for (int c = l; c < 32 * CPR; c += 32) {
    const int r = c / CPR, q = c % CPR;
    const uint32_t rid = __shfl_sync(FULL, myid, r);
    const int64_t boff = (int64_t)tI * TILEB + q * 16;
    if (r < nw && boff < rowbytes) cp_async16(mt + r * PITCH + q * 16, Wb + (int64_t)rid * rowbytes + boff);
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncwarp();
}

template <class W, int MODE, int TILEB>
__global__ void __launch_bounds__(RM_RPB) rm_forward_kernel(RmArgs a) {
  constexpr int EPT = TILEB / (int)sizeof(W);
  constexpr int PITCH = TILEB + 16;
  constexpr int CPL = EPT / 32;
  extern __shared__ __align__(16) unsigned char dyn[];
  const int xs_bytes = (int)round_up((int64_t)a.ldx * 4, 16);
  float* xs = reinterpret_cast<float*>(dyn);
  unsigned char* tiles = dyn + xs_bytes;
  float* wpart = reinterpret_cast<float*>(tiles + RM_NWB * 32 * PITCH);
  const int s = blockIdx.y, chunk = blockIdx.x;
  if (a.only_empty && a.only_empty[s] != 0) return;
  const int na_tot = a.A.cnt[s];
  if (chunk * RM_RPB >= na_tot) return;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int a0 = chunk * RM_RPB + w * 32;
  const int nw = max(0, min(32, na_tot - a0));
  if (MODE != RM_DX)
    for (int k = threadIdx.x; k < a.ldx; k += RM_RPB) xs[k] = a.X[(int64_t)s * a.ldx + k];
  const int64_t arow = (int64_t)s * a.A.stride + a0 + l;
  const bool has = l < nw;
  const uint32_t myid = has ? a.A.ids[arow] : 0u;
  unsigned char* mt = tiles + w * 32 * PITCH;
  const int64_t rowbytes = (int64_t)a.ldw * sizeof(W);
  const int ntiles = (int)ceil_div(rowbytes, TILEB);
  const unsigned char* Wb = static_cast<const unsigned char*>(a.W);
  __syncthreads();
  float lgv = 0.0f;
  if (MODE != RM_DX) {
    float acc = 0.0f;
    for (int tI = 0; tI < ntiles; ++tI) {
      rm_load_tile<W, TILEB>(mt, Wb, rowbytes, tI, myid, nw);
      if (has) {
        // Sequential f32 dot in element order (bit-exact).  The loop runs to a
        // whole number of 16-byte vectors: row padding up to ldw is zero in W
        // and the staged x is zero beyond d, so the extra terms add +0.
        const int k0 = tI * EPT;
        constexpr int VE = 16 / (int)sizeof(W);
        const int kmax = (int)round_up(min(EPT, a.d - k0), VE);
        const uint4* rowp = reinterpret_cast<const uint4*>(mt + l * PITCH);
        const float4* x4 = reinterpret_cast<const float4*>(xs + k0);
        auto dot8 = [&](int kb) {  // VE elements from k0 + kb, in order
          const uint4 raw = rowp[kb / VE];
          const W* e = reinterpret_cast<const W*>(&raw);
          float xv[VE];
#pragma unroll
          for (int u4 = 0; u4 < VE / 4; ++u4) {
            const float4 t4 = x4[kb / 4 + u4];
            xv[4 * u4] = t4.x; xv[4 * u4 + 1] = t4.y; xv[4 * u4 + 2] = t4.z; xv[4 * u4 + 3] = t4.w;
          }
#pragma unroll
          for (int u = 0; u < VE; ++u) acc = __fadd_rn(acc, __fmul_rn(to_f(e[u]), xv[u]));
        };
        if (kmax == EPT) {  // a whole tile (C1/C2 rows: one tile of 128 / 256 elements): unrolled
#pragma unroll
          for (int kb = 0; kb < EPT; kb += VE) dot8(kb);
        } else {
          for (int kb = 0; kb < kmax; kb += VE) dot8(kb);
        }
      }
      __syncwarp();
    }
    if (has) {
      const float pre = __fadd_rn(acc, a.bias[myid]);
      const float post = a.act == KL_ACT_SOFTMAX ? pre : act_apply(pre, a.act);
      a.A.pre[arow] = pre;
      a.A.post[arow] = post;
      if (MODE == RM_FWD) {
        if (a.h && a.act != KL_ACT_SOFTMAX) a.h[(int64_t)s * a.ldh + myid] = post;
      } else {
        // compute_loss_gradient (net.rs:205-230) times the activation derivative
        const int lb = a.lab_ptr[s], le = a.lab_ptr[s + 1];
        float g = post;
        if (le == lb) {
          g = 0.0f;
        } else {
          const float lw = __fdiv_rn(1.0f, (float)(le - lb));
          for (int j = lb; j < le; ++j) {
            if (a.labels[j] == myid + a.id_base) {
              g = __fsub_rn(g, lw);
              a.labprob[j] = post;
            }
          }
        }
        lgv = __fmul_rn(g, act_deriv(pre, post, a.act));
        a.A.lg[arow] = lgv;
        if (a.lgd_dense) a.lgd_dense[(int64_t)a.slot_of[myid] * a.ldb + s] = lgv;
      }
    }
  } else if (has) {
    lgv = a.A.lg[arow];
  }
  if constexpr (MODE == RM_FWD) return;
  // input gradient of this block's rows (old weights, layer.rs:206-209)
  for (int tI = 0; tI < ntiles; ++tI) {
    if (MODE == RM_DX || ntiles > 1) rm_load_tile<W, TILEB>(mt, Wb, rowbytes, tI, myid, nw);
    float part[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) part[c] = 0.0f;
    // lane l owns the CPL consecutive columns l*CPL.. of the tile (columns
    // beyond d see zero row padding and are not written back)
    auto dx_row = [&](int r) {
      const float lr = __shfl_sync(FULL, lgv, r);
      const unsigned char* rowb = mt + r * PITCH + l * CPL * (int)sizeof(W);
      if constexpr (sizeof(W) == 2 && CPL == 4) {
        const uint2 raw = *reinterpret_cast<const uint2*>(rowb);
        const W* e = reinterpret_cast<const W*>(&raw);
#pragma unroll
        for (int c = 0; c < 4; ++c) part[c] = fmaf(lr, to_f(e[c]), part[c]);
      } else {
        const W* rowp = reinterpret_cast<const W*>(rowb);
#pragma unroll
        for (int c = 0; c < CPL; ++c) part[c] = fmaf(lr, to_f(rowp[c]), part[c]);
      }
    };
    if (nw == 32) {  // a full warp of rows: unrolled (constant shuffle lanes and offsets)
#pragma unroll
      for (int r = 0; r < 32; ++r) dx_row(r);
    } else {
      for (int r = 0; r < nw; ++r) dx_row(r);
    }
#pragma unroll
    for (int c = 0; c < CPL; ++c) wpart[w * EPT + l * CPL + c] = part[c];
    __syncthreads();
    for (int col = threadIdx.x; col < EPT; col += RM_RPB) {
      const int kg = tI * EPT + col;
      if (kg < a.ldx) {
        float v = 0.0f;
        for (int ww = 0; ww < RM_NWB; ++ww) v += wpart[ww * EPT + col];
        a.dxpart[((int64_t)s * a.nchunk + chunk) * a.ldx + kg] = v;
      }
    }
    __syncthreads();
  }
}

__global__ void reduce_dx_kernel(const float* dxpart, int nchunk, int ld, int d,
                                 const int32_t* cnt, float* dx) {
  const int s = blockIdx.x;
  const int nch = (int)ceil_div(cnt[s], RM_RPB);
  for (int k = threadIdx.x; k < ld; k += blockDim.x) {
    float v = 0.0f;
    if (k < d)
      for (int c = 0; c < nch; ++c) v += dxpart[((int64_t)s * nchunk + c) * ld + k];
    dx[(int64_t)s * ld + k] = v;
  }
}

// Softmax over the active set (layer.rs:286-308) and, with labels, the loss
// gradient through the softmax Jacobian (layer.rs:141-176):
// lg_i = sum_j g_j s_j (delta_ij - s_i) = s_i g_i - s_i * sum_j g_j s_j.
__global__ void softmax_kernel(ActiveSet A, float* h, int ldh, const int32_t* lab_ptr,
                               const uint32_t* labels, float* labprob) {
  __shared__ float tmp[40];
  const int s = blockIdx.x;
  const int na = A.cnt[s];
  const int64_t o = (int64_t)s * A.stride;
  float mx = __int_as_float(0xff800000);
  for (int a = threadIdx.x; a < na; a += blockDim.x) mx = fmaxf(mx, A.pre[o + a]);
  mx = block_reduce_max_f(mx, tmp);
  float sum = 0.0f;
  for (int a = threadIdx.x; a < na; a += blockDim.x) {
    const float e = expf(__fsub_rn(A.pre[o + a], mx));
    A.post[o + a] = e;
    sum += e;
  }
  sum = block_reduce_sum_f(sum, tmp);
  float S = 0.0f;
  for (int a = threadIdx.x; a < na; a += blockDim.x) {
    const float sv = sum > 0.0f ? __fdiv_rn(A.post[o + a], sum) : __fdiv_rn(1.0f, (float)na);
    A.post[o + a] = sv;
    const uint32_t id = A.ids[o + a];
    if (h) h[(int64_t)s * ldh + id] = sv;
    if (lab_ptr) {
      const int lb = lab_ptr[s], le = lab_ptr[s + 1];
      float g = sv;
      if (le == lb) {
        g = 0.0f;
      } else {
        const float lw = __fdiv_rn(1.0f, (float)(le - lb));
        for (int j = lb; j < le; ++j)
          if (labels[j] == id) {
            g = __fsub_rn(g, lw);
            labprob[j] = sv;
          }
      }
      A.lg[o + a] = g;  // temporarily the output gradient
      S += g * sv;
    }
  }
  if (!lab_ptr) return;
  S = block_reduce_sum_f(S, tmp);
  for (int a = threadIdx.x; a < na; a += blockDim.x) {
    const float sv = A.post[o + a], g = A.lg[o + a];
    A.lg[o + a] = __fsub_rn(__fmul_rn(sv, g), __fmul_rn(sv, S));
  }
}

// Local gradients of a non-output layer (layer.rs:177-193).
__global__ void local_grads_kernel(ActiveSet A, int act, const float* grad, int ldg, float* lgd,
                                   int ldl, uint32_t* touched_mask) {
  const int s = blockIdx.y;
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= A.cnt[s]) return;
  const int64_t o = (int64_t)s * A.stride + a;
  const uint32_t id = A.ids[o];
  const float lg = __fmul_rn(grad[(int64_t)s * ldg + id], act_deriv(A.pre[o], A.post[o], act));
  A.lg[o] = lg;
  if (lgd) {
    lgd[(int64_t)s * ldl + id] = lg;
    atomicOr(&touched_mask[id >> 5], 1u << (id & 31));
  }
}
// Softmax hidden layer: lg_i = s_i go_i - s_i sum_j go_j s_j.
__global__ void local_grads_softmax_kernel(ActiveSet A, const float* grad, int ldg, float* lgd,
                                           int ldl, uint32_t* touched_mask) {
  __shared__ float tmp[40];
  const int s = blockIdx.x;
  const int na = A.cnt[s];
  const int64_t o = (int64_t)s * A.stride;
  float S = 0.0f;
  for (int a = threadIdx.x; a < na; a += blockDim.x)
    S += grad[(int64_t)s * ldg + A.ids[o + a]] * A.post[o + a];
  S = block_reduce_sum_f(S, tmp);
  for (int a = threadIdx.x; a < na; a += blockDim.x) {
    const uint32_t id = A.ids[o + a];
    const float sv = A.post[o + a];
    const float lg = __fsub_rn(__fmul_rn(sv, grad[(int64_t)s * ldg + id]), __fmul_rn(sv, S));
    A.lg[o + a] = lg;
    if (lgd) {
      lgd[(int64_t)s * ldl + id] = lg;
      atomicOr(&touched_mask[id >> 5], 1u << (id & 31));
    }
  }
}

// compute_loss (net.rs:180-199): per sample, then summed in sample order.
__global__ void loss_kernel(const int32_t* lab_ptr, const float* labprob, int nq, float* accum) {
  extern __shared__ float ls[];
  const float eps = 1e-7f;
  for (int s = threadIdx.x; s < nq; s += blockDim.x) {
    const int lb = lab_ptr[s], le = lab_ptr[s + 1];
    float loss = 0.0f;
    for (int j = lb; j < le; ++j) loss = __fsub_rn(loss, logf(fmaxf(labprob[j], eps)));
    ls[s] = le > lb ? __fdiv_rn(loss, (float)(le - lb)) : 0.0f;
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // in example order; groups of 8 loads ahead of their adds
    float acc = *accum;
    int s = 0;
    for (; s + 8 <= nq; s += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = ls[s + u];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, v[u]);
    }
    for (; s < nq; ++s) acc = __fadd_rn(acc, ls[s]);
    *accum = acc;
  }
}

// ---------------------------------------------------------------------------
// Segmented gradient reduction without float atomics.  (1) every (sample,
// row) pair bumps a per-row counter; the first bump appends the row to the
// touched list; (2) each touched row reserves a contiguous segment;
// (3) pairs scatter (sample, coefficient) into their row's segment;
// (4) one warp per touched row rebuilds the segment as a per-sample bitmask
// in shared memory, so the gradient is summed in ascending sample order --
// deterministic and identical to the batched oracle -- and applies the
// optimizer to the row in the same pass (the gradient never touches HBM).
// ---------------------------------------------------------------------------
__global__ void rm_touch_kernel(ActiveSet A, uint32_t* hist, uint32_t* touched, uint32_t* ctr) {
  const int s = blockIdx.y;
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = a < A.cnt[s];
  uint32_t id = 0, old = 1;
  if (valid) {
    id = A.ids[(int64_t)s * A.stride + a];
    old = atomicAdd(&hist[id], 1u);
  }
  const int pos = warp_append(valid && old == 0, &ctr[0]);
  if (pos >= 0) touched[pos] = id;
}
// Feature rows [f0, f0 + nf) only (a rank's slice of a sharded hidden update).
__global__ void fm_touch_kernel(SparseIn in, uint32_t* hist, uint32_t* touched, uint32_t* ctr, uint32_t f0,
                                uint32_t nf) {
  const int s = blockIdx.x;
  const int beg = in.rowptr[s], end = in.rowptr[s + 1];
  for (int base = beg; base < end; base += blockDim.x) {
    const int e = base + threadIdx.x;
    bool valid = e < end;
    uint32_t f = 0, old = 1;
    if (valid) {
      f = in.idx[e];
      valid = f - f0 < nf;
      if (valid) old = atomicAdd(&hist[f], 1u);
    }
    const int pos = warp_append(valid && old == 0, &ctr[0]);
    if (pos >= 0) touched[pos] = f;
  }
}
__global__ void seg_alloc_kernel(const uint32_t* hist, const uint32_t* touched, uint32_t* cur,
                                 uint32_t* ctr, int maxn) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  const int n = (int)ctr[0];
  if (blockIdx.x * blockDim.x >= n) return;  // whole block idle
  const bool valid = k < n && k < maxn;
  const uint32_t row = valid ? touched[k] : 0u;
  const int len = valid ? (int)hist[row] : 0;
  const int inc = warp_incl_scan(len);
  const int wtot = __shfl_sync(FULL, inc, 31);
  uint32_t base = 0;
  if ((threadIdx.x & 31) == 31) base = atomicAdd(&ctr[1], (uint32_t)wtot);
  base = __shfl_sync(FULL, base, 31);
  if (valid) cur[row] = base + inc - len;
}
__global__ void rm_scatter_kernel(ActiveSet A, uint32_t* cur, uint32_t* ent_s, float* ent_v) {
  const int s = blockIdx.y;
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= A.cnt[s]) return;
  const int64_t o = (int64_t)s * A.stride + a;
  const uint32_t pos = atomicAdd(&cur[A.ids[o]], 1u);
  ent_s[pos] = (uint32_t)s;
  ent_v[pos] = A.lg[o];
}
__global__ void fm_scatter_kernel(SparseIn in, uint32_t* cur, uint32_t* ent_s, float* ent_v, uint32_t f0,
                                  uint32_t nf) {
  const int s = blockIdx.x;
  for (int e = in.rowptr[s] + threadIdx.x; e < in.rowptr[s + 1]; e += blockDim.x) {
    const uint32_t f = in.idx[e];
    if (f - f0 >= nf) continue;
    const uint32_t pos = atomicAdd(&cur[f], 1u);
    ent_s[pos] = (uint32_t)s;
    ent_v[pos] = in.val[e];
  }
}

// Load one segment into the warp's (coefficient, sample-bitmask) buffers.
__device__ __forceinline__ void seg_to_mask(const uint32_t* ent_s, const float* ent_v, uint32_t start,
                                            uint32_t len, float* coef, uint32_t* mask) {
  for (uint32_t e = threadIdx.x & 31; e < len; e += 32) {
    const uint32_t s = ent_s[start + e];
    coef[s] = ent_v[start + e];
    atomicOr(&mask[s >> 5], 1u << (s & 31));
  }
  __syncwarp();
}

template <class W>
__device__ __forceinline__ void load4(const void* Wm, int64_t off, float* w) {
  if (sizeof(W) == 4) {
    const float4 v = *reinterpret_cast<const float4*>(static_cast<const float*>(Wm) + off);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(Wm) + off);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
    w[0] = to_f(e[0]); w[1] = to_f(e[1]); w[2] = to_f(e[2]); w[3] = to_f(e[3]);
  }
}
template <class W>
__device__ __forceinline__ void store4(void* Wm, int64_t off, const float* w) {
  if (sizeof(W) == 4) {
    *reinterpret_cast<float4*>(static_cast<float*>(Wm) + off) = make_float4(w[0], w[1], w[2], w[3]);
  } else {
    __nv_bfloat16 e[4] = {__float2bfloat16_rn(w[0]), __float2bfloat16_rn(w[1]),
                          __float2bfloat16_rn(w[2]), __float2bfloat16_rn(w[3])};
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(Wm) + off) = *reinterpret_cast<uint2*>(e);
  }
}

// Apply the optimizer to 4 consecutive elements; lanes with !upd[i] keep
// their values (row padding, untouched neurons).
template <class W>
__device__ __forceinline__ void row_update4(void* Wm, float* m, float* v, int64_t off,
                                            const float* g, const bool* upd, const OptStep& o) {
  float w[4], mm[4], vv[4];
  load4<W>(Wm, off, w);
  const float4 m4 = *reinterpret_cast<const float4*>(m + off);
  mm[0] = m4.x; mm[1] = m4.y; mm[2] = m4.z; mm[3] = m4.w;
  float4 v4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (o.opt == KL_OPT_ADAM) v4 = *reinterpret_cast<const float4*>(v + off);
  vv[0] = v4.x; vv[1] = v4.y; vv[2] = v4.z; vv[3] = v4.w;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (upd[i]) opt_apply(w[i], mm[i], vv[i], g[i], o);
  store4<W>(Wm, off, w);
  *reinterpret_cast<float4*>(m + off) = make_float4(mm[0], mm[1], mm[2], mm[3]);
  if (o.opt == KL_OPT_ADAM) *reinterpret_cast<float4*>(v + off) = make_float4(vv[0], vv[1], vv[2], vv[3]);
}

__device__ __forceinline__ void bias_update(float* bias, float* mb, float* vb, uint32_t j, float gb,
                                            const OptStep& o) {
  float b = bias[j], m = mb[j], v = (o.opt == KL_OPT_ADAM) ? vb[j] : 0.0f;
  opt_apply(b, m, v, gb, o);
  bias[j] = b;
  mb[j] = m;
  if (o.opt == KL_OPT_ADAM) vb[j] = v;
}

constexpr int UPD_WARPS = 8;

// One warp per touched row.  The row's (sample, coefficient) pairs are
// marked in a per-warp sample bitmask, compacted into an ascending sample
// list, and the gradient is summed over that list in order, eight samples'
// X vectors loaded ahead of their sums (the loads are independent, the sums
// stay sequential: bit-exact).
constexpr int UPD_PF = 8;
template <class W>
__global__ void __launch_bounds__(UPD_WARPS * 32)
    rm_update_kernel(void* Wm, int ldw, int d, float* bias, float* m, float* v, float* mb, float* vb,
                     const float* X, int ldx, SegScratch S, int nwords, const OptStep* op,
                     unsigned long long* stat_touched) {
  const OptStep o = *op;
  extern __shared__ __align__(16) unsigned char dyn[];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  uint32_t* mask = reinterpret_cast<uint32_t*>(dyn) + w * nwords;
  float* coef = reinterpret_cast<float*>(dyn + (size_t)UPD_WARPS * nwords * 4) + (size_t)w * nwords * 32;
  uint16_t* list = reinterpret_cast<uint16_t*>(dyn + (size_t)UPD_WARPS * nwords * 4 * 33) + (size_t)w * nwords * 32;
  for (int i = l; i < nwords; i += 32) mask[i] = 0;
  __syncwarp();
  const int n = (int)S.ctr[0];
  if (blockIdx.x == 0 && threadIdx.x == 0 && stat_touched) atomicAdd(stat_touched, (unsigned long long)n);
  for (int k = blockIdx.x * UPD_WARPS + w; k < n; k += gridDim.x * UPD_WARPS) {
    const uint32_t row = S.touched[k];
    const uint32_t len = S.hist[row];
    const uint32_t start = S.cur[row] - len;
    seg_to_mask(S.ent_s, S.ent_v, start, len, coef, mask);
    // ascending sample list (and the mask cleared for the next row)
    int cnt = 0;
    for (int w0 = 0; w0 < nwords; w0 += 32) {
      const uint32_t mw = w0 + l < nwords ? mask[w0 + l] : 0u;
      const int c = __popc(mw);
      const int inc = warp_incl_scan(c);
      int pos = cnt + inc - c;
      uint32_t bb = mw;
      while (bb) {
        const int bit = __ffs(bb) - 1;
        bb &= bb - 1;
        list[pos++] = (uint16_t)((w0 + l) * 32 + bit);
      }
      cnt += __shfl_sync(FULL, inc, 31);
      if (w0 + l < nwords) mask[w0 + l] = 0;
    }
    __syncwarp();
    float gb = 0.0f;
    for (int g0 = 0; g0 < d; g0 += 128) {
      const int c = g0 + l * 4;
      float g[4] = {0.f, 0.f, 0.f, 0.f};
      for (int i0 = 0; i0 < cnt; i0 += UPD_PF) {
        float4 xv[UPD_PF];
        float cf[UPD_PF];
#pragma unroll
        for (int u = 0; u < UPD_PF; ++u) {
          if (i0 + u < cnt) {
            const uint32_t sidx = list[i0 + u];
            cf[u] = coef[sidx];
            xv[u] = c < d ? *reinterpret_cast<const float4*>(X + (int64_t)sidx * ldx + c)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int u = 0; u < UPD_PF; ++u) {
          if (i0 + u < cnt) {
            if (g0 == 0) gb = __fadd_rn(gb, cf[u]);
            g[0] = __fadd_rn(g[0], __fmul_rn(cf[u], xv[u].x));
            g[1] = __fadd_rn(g[1], __fmul_rn(cf[u], xv[u].y));
            g[2] = __fadd_rn(g[2], __fmul_rn(cf[u], xv[u].z));
            g[3] = __fadd_rn(g[3], __fmul_rn(cf[u], xv[u].w));
          }
        }
      }
      if (c < d) {
        const bool upd[4] = {c < d, c + 1 < d, c + 2 < d, c + 3 < d};
        row_update4<W>(Wm, m, v, (int64_t)row * ldw + c, g, upd, o);
      }
    }
    if (l == 0) {
      bias_update(bias, mb, vb, row, gb, o);
      S.hist[row] = 0;
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Dense-collision path of the row-major update, used when the layer's dense
// gradient matrix fits its memory budget.  In batched SLIDE steps many
// samples share active rows (C1: ~6 K distinct rows behind 1.5 M (sample,
// row) pairs), so instead of per-row segments built with contended atomics:
//  (1) rm_mark_kernel: a mark word per row; a lane whose row is already
//      marked only reads it, the lane that marks it first appends the row to the
//      touched list (slot = position) and records slot_of[row];
//  (2) rm_dense_scatter_kernel: LGd[slot][s] = local gradient of the row in
//      sample s, slot-major with a pitch of ldb >= max batch samples (the
//      step uses the first n rows; LGd is all zero between steps);
//  (3) rm_dense_update_kernel: a block owns RDU_ROWS consecutive slots (4 per
//      warp) of one 32-column block (a column per lane).  Chunks of RDU_S
//      samples of X and LGd are staged into shared memory by a 4-stage
//      cp.async pipeline; each lane sums g = sum_s lg_s * x_s in ascending s
//      with the non-fused f32 operations of the batched oracle (bit-exact),
//      applies the optimizer to its rows and biases, and clears their marks;
//  (4) rm_lg_zero_kernel zeroes the n x ldb block the step used.
// The slot-major layout keeps a step's gradients in one contiguous block: a
// sample-major [sample][slot] layout measured ~1.8x slower in the update and
// zeroing kernels at 2048-example batches.
// ---------------------------------------------------------------------------
// rm_dense_scatter_kernel gives each thread RM_PK pairs of one sample (stride
// blockDim), with the loads of all of them issued before any is used.
constexpr int RM_PK = 8;

// One pair per thread: blocks run in waves, and the plain read lets pairs of
// later waves skip the atomic on rows an earlier wave already set (batching
// pairs per thread puts them all in one wave and every pair then contends).
// One mark word per row: a few hundred samples of a large batch meet the same
// rows at once, and words shared by 32 rows would serialise their atomics.
__global__ void rm_mark_kernel(ActiveSet A, uint32_t* mark, uint32_t* touched, uint32_t* slot_of,
                               uint32_t* ctr, const int32_t* only_empty) {
  const int s = blockIdx.y;
  if (only_empty && only_empty[s] != 0) return;
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= A.cnt[s]) return;
  const uint32_t id = A.ids[(int64_t)s * A.stride + a];
  uint32_t* wp = mark + id;
  bool first = false;
  if (!*reinterpret_cast<volatile uint32_t*>(wp)) first = atomicExch(wp, 1u) == 0u;
  const int pos = warp_append(first, ctr);
  if (pos >= 0) {
    touched[pos] = id;
    slot_of[id] = (uint32_t)pos;
  }
}

__global__ void rm_dense_scatter_kernel(ActiveSet A, const uint32_t* slot_of, float* LGd, int64_t ldb) {
  const int s = blockIdx.y;
  const int n = A.cnt[s];
  const int a0 = blockIdx.x * blockDim.x * RM_PK + threadIdx.x;
  if (blockIdx.x * blockDim.x * RM_PK >= n) return;
  uint32_t id[RM_PK], sl[RM_PK];
  float lg[RM_PK];
#pragma unroll
  for (int u = 0; u < RM_PK; ++u) {
    const int a = a0 + u * blockDim.x;
    const int64_t o = (int64_t)s * A.stride + a;
    id[u] = a < n ? A.ids[o] : 0xffffffffu;
    lg[u] = a < n ? A.lg[o] : 0.0f;
  }
#pragma unroll
  for (int u = 0; u < RM_PK; ++u) sl[u] = id[u] != 0xffffffffu ? slot_of[id[u]] : 0u;
#pragma unroll
  for (int u = 0; u < RM_PK; ++u)
    if (id[u] != 0xffffffffu) LGd[(int64_t)sl[u] * ldb + s] = lg[u];
}

// Slots per warp RPW (a template parameter: 4, or 2 / 1 when a long sample
// loop meets few touched rows -- a shard over a large global batch -- so that
// more blocks share the work); 8 * RPW slots per block (8 warps).
constexpr int RDU_COLS = 32;             // columns per block (one per lane)
constexpr int RDU_S = 32;                // samples per staged chunk

// Block = (32 slots, 32 columns): warp w owns slots 4w .. 4w+3, lane l column
// cb*32 + l.  Column blocks multiply the parallelism when few rows meet many
// samples (a shard's union over a large global batch).  The sums start at
// +0 and a round-to-nearest sum is -0 only when both operands are, so a +-0
// term (a sample where the row is not active) leaves a sum unchanged: the sum
// over any superset of the active samples, in ascending order, equals the
// sum over the active samples (finite activations assumed).  The
// gradient matrix is left as read; rm_lg_zero_kernel restores its zeros.
// Samples are taken in groups of RDU_G whose shared-memory operands are all
// loaded before the group's arithmetic: the only loop-carried dependency is
// then the running sum itself.  ls is the staged gradient tile, slot-major
// ([slot][sample]); every lane of a warp reads the same ls words (broadcast).
constexpr int RDU_G = 8;
template <class W, bool BIAS, int RPW>
__device__ __forceinline__ void rdu_sum_chunk(const float (*xs)[RDU_COLS], const float (*ls)[RDU_S], int ns,
                                              int w, int l, float* g, float* gb) {
  int j = 0;
  for (; j + RDU_G <= ns; j += RDU_G) {
    float xv[RDU_G], lv[RPW][RDU_G];
#pragma unroll
    for (int u = 0; u < RDU_G; ++u) xv[u] = xs[j + u][l];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
#pragma unroll
      for (int u = 0; u < RDU_G; u += 4) {
        const float4 q = *reinterpret_cast<const float4*>(&ls[w * RPW + i][j + u]);
        lv[i][u] = q.x;
        lv[i][u + 1] = q.y;
        lv[i][u + 2] = q.z;
        lv[i][u + 3] = q.w;
      }
    }
#pragma unroll
    for (int u = 0; u < RDU_G; ++u) {
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        g[i] = __fadd_rn(g[i], __fmul_rn(lv[i][u], xv[u]));
        if (BIAS) gb[i] = __fadd_rn(gb[i], lv[i][u]);
      }
    }
  }
  for (; j < ns; ++j) {
    const float xv = xs[j][l];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const float lv = ls[w * RPW + i][j];
      g[i] = __fadd_rn(g[i], __fmul_rn(lv, xv));
      if (BIAS) gb[i] = __fadd_rn(gb[i], lv);
    }
  }
}

template <class W, int RPW, int NWB, int RDU_ST>
__global__ void __launch_bounds__(NWB * 32)
    rm_dense_update_kernel(void* Wm, int ldw, int d, float* bias, float* m, float* v, float* mb, float* vb,
                           const float* X, int ldx, uint32_t* mark, const uint32_t* touched, const uint32_t* ctr,
                           float* LGd, int64_t ldb, int nq, const OptStep* op) {
  constexpr int RDU_RPW = RPW;
  constexpr int RDU_ROWS = NWB * RPW;  // slots per block
  static_assert(RDU_ROWS % 4 == 0, "gradient tiles are staged in 16-byte pieces");
  constexpr int NT = NWB * 32;
  const OptStep o = *op;
  extern __shared__ __align__(16) float rdu_smem[];
  float(*xs)[RDU_S][RDU_COLS] = reinterpret_cast<float(*)[RDU_S][RDU_COLS]>(rdu_smem);
  float(*ls)[RDU_ROWS][RDU_S] = reinterpret_cast<float(*)[RDU_ROWS][RDU_S]>(rdu_smem + RDU_ST * RDU_S * RDU_COLS);
  const int t = threadIdx.x, w = t >> 5, l = t & 31;
  const int n = (int)ctr[0];
  const int nch = (nq + RDU_S - 1) / RDU_S;
  const int ncb = (d + RDU_COLS - 1) / RDU_COLS;
  const int ngroups = (n + RDU_ROWS - 1) / RDU_ROWS;
  for (int item = blockIdx.x; item < ngroups * ncb; item += gridDim.x) {
    const int k0 = (item / ncb) * RDU_ROWS, cb = item % ncb;
    const int c = cb * RDU_COLS + l;
    const bool cin = c < d;
    auto stage = [&](int ch) {  // 32 samples x 32 columns of X and RDU_ROWS slots x 32 samples of LGd
      const int bf = ch % RDU_ST;
      const int s0 = ch * RDU_S;
      for (int q = t; q < RDU_S * RDU_COLS / 4; q += NT) {
        const int r = q >> 3, c4 = (q & 7) * 4;
        float* dx = &xs[bf][r][c4];
        if (s0 + r < nq && cb * RDU_COLS + c4 < d)
          cp_async16(dx, X + (int64_t)(s0 + r) * ldx + cb * RDU_COLS + c4);
        else
          *reinterpret_cast<float4*>(dx) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      // slots k0 .. k0 + RDU_ROWS - 1 and samples s0 .. s0 + 31 lie inside the
      // allocation (round_up(rows, 32) slots, ldb a multiple of 32); slots past
      // the touched count and samples nq .. ldb - 1 are zero
      for (int q = t; q < RDU_S * RDU_ROWS / 4; q += NT) {
        const int lr = q / (RDU_S / 4), lc4 = (q % (RDU_S / 4)) * 4;
        cp_async16(&ls[bf][lr][lc4], LGd + (int64_t)(k0 + lr) * ldb + s0 + lc4);
      }
    };
    // optimizer state of this lane's elements, loaded now and used after the sum
    float wv[RDU_RPW], mv[RDU_RPW], vv[RDU_RPW];
    int64_t roff[RDU_RPW];
#pragma unroll
    for (int i = 0; i < RDU_RPW; ++i) {
      const int k = k0 + w * RDU_RPW + i;
      roff[i] = -1;
      if (k < n && cin) {
        roff[i] = (int64_t)touched[k] * ldw + c;
        wv[i] = to_f(static_cast<const W*>(Wm)[roff[i]]);
        mv[i] = m[roff[i]];
        vv[i] = o.opt == KL_OPT_ADAM ? v[roff[i]] : 0.f;
      }
    }
    float g[RDU_RPW], gb[RDU_RPW];
#pragma unroll
    for (int i = 0; i < RDU_RPW; ++i) g[i] = gb[i] = 0.f;
    __syncthreads();  // previous users of the buffers are done
#pragma unroll
    for (int p = 0; p < RDU_ST - 1; ++p) {
      if (p < nch) stage(p);
      cp_async_commit();  // one group per stage slot (possibly empty) keeps the wait count uniform
    }
    for (int ch = 0; ch < nch; ++ch) {
      const int bf = ch % RDU_ST;
      if (ch + RDU_ST - 1 < nch) stage(ch + RDU_ST - 1);
      cp_async_commit();
      cp_async_wait_group<RDU_ST - 1>();
      __syncthreads();
      const int ns = min(RDU_S, nq - ch * RDU_S);
      if (cb == 0) rdu_sum_chunk<W, true, RPW>(xs[bf], ls[bf], ns, w, l, g, gb);
      else rdu_sum_chunk<W, false, RPW>(xs[bf], ls[bf], ns, w, l, g, gb);
      __syncthreads();  // buffer bf is restaged RDU_ST - 1 chunks later
    }
    cp_async_wait_group<0>();
#pragma unroll
    for (int i = 0; i < RDU_RPW; ++i) {
      if (roff[i] < 0) continue;
      opt_apply(wv[i], mv[i], vv[i], g[i], o);
      static_cast<W*>(Wm)[roff[i]] = from_f<W>(wv[i]);
      m[roff[i]] = mv[i];
      if (o.opt == KL_OPT_ADAM) v[roff[i]] = vv[i];
    }
    if (cb == 0 && l < RDU_RPW) {
      const int k = k0 + w * RDU_RPW + l;
      if (k < n) {
        const uint32_t row = touched[k];
        float gbl = gb[0];
#pragma unroll
        for (int i = 1; i < RDU_RPW; ++i)
          if (l == i) gbl = gb[i];
        bias_update(bias, mb, vb, row, gbl, o);
        mark[row] = 0u;  // ready for the next step's mark
      }
    }
  }
}

// LGd[slot][*] = 0 for the touched slots (restores the zero invariant): one
// contiguous block of n x ldb floats.
__global__ void rm_lg_zero_kernel(float* LGd, int64_t ldb, const uint32_t* ctr) {
  const int64_t n4 = (int64_t)ctr[0] * ldb / 4;
  float4* p = reinterpret_cast<float4*>(LGd);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// Feature-major (layer 0) update, in two passes.
//
// (1) fm_grad_short_kernel / fm_grad_long_kernel: the gradient of neuron j
//     at feature row f is sum over the samples s that contain f of
//     x_s[f] * lg_s[j], in ascending s (the batched oracle's order).  The
//     segment's (sample, value) pairs arrive unordered.  Segments of at most
//     FM_SHORT pairs (nearly all of them) are put in order by ranking the
//     pairs inside one warp, which then sums 4 neurons per lane; longer ones
//     are queued and a block per feature orders them through a per-sample
//     bitmask.  The row goes to G[k] (k = position of f in the touched list)
//     and slot[f] becomes k + 1.
// (2) fm_adam_kernel: streams W, m, v of ALL d feature rows (Adam runs over
//     every element of a touched neuron, optim/adam.rs:57-68) with persistent
//     warps that keep their next items' loads in flight through a per-warp
//     shared-memory ring; rows with slot[f] != 0 read their gradient from G,
//     the rest use g = 0.  slot[f] and hist[f] are zeroed for the next step
//     (by fm_hist_clear_kernel when a row spans several items).
// ---------------------------------------------------------------------------
constexpr int FM_NT = 256;

constexpr int FM_SHORT = 32;  // segments up to this length are ranked inside one warp
constexpr int FM_GW = 8;      // warps per fm_grad_short block

__global__ void __launch_bounds__(FM_GW * 32)
    fm_grad_short_kernel(int N, const float* lgd, int ldl, SegScratch S, float* G, int ldg) {
  // one warp per touched feature.  Lane e holds the segment's e-th (sample,
  // value) pair; its rank among the pairs (sample id, then lane on a tie) is
  // its place in the ascending list.  Lane l then sums neurons [4l, 4l + 4)
  // of each 128-neuron chunk over the list.  Longer segments are queued for
  // fm_grad_long_kernel.
  __shared__ uint32_t ls[FM_GW][FM_SHORT];
  __shared__ float lv[FM_GW][FM_SHORT];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int n = (int)S.ctr[0];
  for (int k = blockIdx.x * FM_GW + w; k < n; k += gridDim.x * FM_GW) {
    const uint32_t f = S.touched[k];
    const int len = (int)S.hist[f];
    if (l == 0) S.slot[f] = (uint32_t)k + 1u;
    if (len > FM_SHORT) {
      if (l == 0) S.longk[atomicAdd(&S.ctr[2], 1u)] = (uint32_t)k;
      continue;
    }
    const uint32_t start = S.cur[f] - (uint32_t)len;
    uint32_t s = 0xffffffffu;
    float v = 0.f;
    if (l < len) {
      s = S.ent_s[start + l];
      v = S.ent_v[start + l];
    }
    int r = 0;
    for (int j = 0; j < len; ++j) {
      const uint32_t sj = __shfl_sync(FULL, s, j);
      r += (sj < s) | ((sj == s) & (j < l));
    }
    if (l < len) {
      ls[w][r] = s;
      lv[w][r] = v;
    }
    __syncwarp();
    for (int c0 = 0; c0 < ldg; c0 += 128) {
      const int c = c0 + 4 * l;
      float g[4] = {0.f, 0.f, 0.f, 0.f};
      if (c < N) {
        for (int i0 = 0; i0 < len; i0 += 8) {
          float4 q[8];
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (i0 + u < len) q[u] = *reinterpret_cast<const float4*>(lgd + (int64_t)ls[w][i0 + u] * ldl + c);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            if (i0 + u < len) {
              const float x = lv[w][i0 + u];
              g[0] = __fadd_rn(g[0], __fmul_rn(x, q[u].x));
              g[1] = __fadd_rn(g[1], __fmul_rn(x, q[u].y));
              g[2] = __fadd_rn(g[2], __fmul_rn(x, q[u].z));
              g[3] = __fadd_rn(g[3], __fmul_rn(x, q[u].w));
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (c + j >= N) g[j] = 0.f;
      }
      if (c < ldg) *reinterpret_cast<float4*>(G + (int64_t)k * ldg + c) = make_float4(g[0], g[1], g[2], g[3]);
    }
    __syncwarp();  // ls / lv reused by the warp's next feature
  }
}

__global__ void __launch_bounds__(1024)
    fm_grad_long_kernel(int N, const float* lgd, int ldl, SegScratch S, int nwords, float* G, int ldg, int chr) {
  // one block per queued feature (segment longer than FM_SHORT): the block
  // marks the samples in a bitmask, warp 0 compacts the set bits into an
  // ascending list, then warp w sums neuron 32w + lane over it
  extern __shared__ __align__(16) unsigned char dyn[];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  uint32_t* mask = reinterpret_cast<uint32_t*>(dyn);   // [nwords]
  float* coef = reinterpret_cast<float*>(mask + nwords);  // [32*nwords]
  uint32_t* list = mask + nwords + 32 * nwords;          // [32*nwords]
  float* rows = reinterpret_cast<float*>(dyn + round_up((int64_t)nwords * 4 * 65, 16));  // [2][chr][ldl]
  __shared__ int base_s;
  for (int i = threadIdx.x; i < nwords; i += blockDim.x) mask[i] = 0;
  __syncthreads();
  const int n = (int)S.ctr[2];
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const uint32_t k = S.longk[i];
    const uint32_t f = S.touched[k];
    const uint32_t len = S.hist[f];
    const uint32_t start = S.cur[f] - len;
    for (uint32_t e = threadIdx.x; e < len; e += blockDim.x) {
      const uint32_t s = S.ent_s[start + e];
      coef[s] = S.ent_v[start + e];
      atomicOr(&mask[s >> 5], 1u << (s & 31));
    }
    __syncthreads();
    if (w == 0) {
      int base = 0;
      for (int w0 = 0; w0 < nwords; w0 += 32) {
        const uint32_t mw = w0 + l < nwords ? mask[w0 + l] : 0u;
        const int c = __popc(mw);
        const int inc = warp_incl_scan(c);
        int pos = base + inc - c;
        uint32_t b = mw;
        while (b) {
          const int bit = __ffs(b) - 1;
          b &= b - 1;
          list[pos++] = (uint32_t)((w0 + l) * 32 + bit);
        }
        base += __shfl_sync(FULL, inc, 31);
        if (w0 + l < nwords) mask[w0 + l] = 0;
      }
      if (l == 0) base_s = base;
    }
    __syncthreads();
    const int base = base_s;
    // The listed samples' gradient rows come through shared memory in chunks
    // of `chr` rows, double-buffered with cp.async by the whole block
    // (coalesced 16-byte copies, one L2 round trip per chunk); thread c then
    // sums column c over the chunk in list order (bit-exact).
    const int c = threadIdx.x;  // one column per thread (blockDim >= ldg)
    float g = 0.f;
    const int vpr = ldl / 4;
    auto stage = [&](int i0, int b) {
      const int cn = min(chr, base - i0);
      float* dst = rows + (size_t)b * chr * ldl;
      for (int q = threadIdx.x; q < cn * vpr; q += blockDim.x) {
        const int r = q / vpr, c4 = (q - r * vpr) * 4;
        cp_async16(dst + r * ldl + c4, lgd + (int64_t)list[i0 + r] * ldl + c4);
      }
      cp_async_commit();
    };
    if (base > 0) stage(0, 0);
    for (int i0 = 0, b = 0; i0 < base; i0 += chr, b ^= 1) {
      if (i0 + chr < base) stage(i0 + chr, b ^ 1);
      else cp_async_commit();  // keeps one group per iteration
      cp_async_wait_group<1>();
      __syncthreads();
      if (c < N) {
        const float* src = rows + (size_t)b * chr * ldl + c;
        const int cn = min(chr, base - i0);
        for (int r = 0; r < cn; ++r) g = __fadd_rn(g, __fmul_rn(coef[list[i0 + r]], src[r * ldl]));
      }
      __syncthreads();  // buffer b is restaged two chunks later
    }
    if (c < ldg) G[(int64_t)k * ldg + c] = g;
    __syncthreads();  // list / coef reused by the next feature
  }
}

// One work item = rpw whole feature rows (vpr <= 32 vectors each: lane l
// holds vector l % vpr of row l / vpr) or, for vpr > 32, the k-th 32-vector
// slice of one row (nk slices per row).
__device__ __forceinline__ bool fm_item_pos(int i, int rpw, int nk, int vpr, int d, int r_l, int j_l, int& f,
                                            int& c) {
  int j;
  if (nk == 1) {
    f = i * rpw + r_l;
    j = j_l;
  } else {
    f = i / nk;
    j = (i - f * nk) * 32 + (int)(threadIdx.x & 31);
  }
  c = 4 * j;
  return r_l < rpw && f < d && j < vpr;
}

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem));
}

// Persistent warps walk items w, w + nwarps, ...  Each lane copies its own
// W / m / v / G vectors of the item FA_D - 1 items ahead into its warp's ring
// of FA_D stages in shared memory with cp.async, and reads back only what it
// copied itself, so a per-thread wait_group is the only synchronisation.
// The slot value that decides the G copy is loaded one item earlier still.
constexpr int FA_NT = 256;
constexpr int FA_D = 3;
constexpr int FA_STG = 32 * 16 * 4;  // one stage of one warp: W, m, v, G, 16 bytes per lane each

template <class W>
__global__ void __launch_bounds__(FA_NT, 4)
    fm_adam_kernel(void* Wm, int ldw, int d, int vpr, int rpw, int nk, int N, float* m, float* v,
                   const uint32_t* tmask, uint32_t* hist, uint32_t* slot, const float* G, int ldg, const OptStep* op) {
  extern __shared__ __align__(16) unsigned char dyn[];
  const OptStep o = *op;
  const bool adam = o.opt == KL_OPT_ADAM;
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  unsigned char* ring = dyn + (size_t)wib * FA_D * FA_STG;
  const int nwarps = gridDim.x * (FA_NT / 32);
  const int i0 = blockIdx.x * (FA_NT / 32) + wib;
  const int nitems = nk == 1 ? (int)ceil_div(d, rpw) : d * nk;
  const int r_l = nk == 1 ? lane / vpr : 0;
  const int j_l = nk == 1 ? lane - r_l * vpr : lane;
  auto upd_bits = [&](int c) {
    if (c >= N) return 0u;
    const uint32_t tw = tmask[c >> 5] >> (c & 31);
    uint32_t u = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (c + q < N && ((tw >> q) & 1u)) u |= 1u << q;
    return u;
  };
  auto slot_of = [&](int t) -> uint32_t {
    const int i = i0 + t * nwarps;
    int f, c;
    if (i < nitems && fm_item_pos(i, rpw, nk, vpr, d, r_l, j_l, f, c)) return slot[f];
    return 0u;
  };
  // copies item t (slot value hv) into stage t % FA_D; always commits a group
  auto issue = [&](int t, uint32_t hv) {
    const int i = i0 + t * nwarps;
    int f, c;
    if (i < nitems && fm_item_pos(i, rpw, nk, vpr, d, r_l, j_l, f, c) && upd_bits(c)) {
      unsigned char* st = ring + (t % FA_D) * FA_STG + lane * 16;
      const int64_t off = (int64_t)f * ldw + c;
      if (sizeof(W) == 2) cp_async8(st, static_cast<const W*>(Wm) + off);
      else cp_async16(st, static_cast<const W*>(Wm) + off);
      cp_async16(st + 512, m + off);
      if (adam) cp_async16(st + 1024, v + off);
      if (hv) cp_async16(st + 1536, G + (int64_t)(hv - 1) * ldg + c);
    }
    cp_async_commit();
  };
  uint32_t hvq[FA_D];  // slot values of items t .. t + FA_D - 1 (ring of registers)
#pragma unroll
  for (int u = 0; u < FA_D; ++u) hvq[u] = slot_of(u);
#pragma unroll
  for (int u = 0; u < FA_D - 1; ++u) issue(u, hvq[u]);
  for (int t = 0; i0 + t * nwarps < nitems; ++t) {
    // hvq[u] holds the slot of item t + u; fetch item t + FA_D - 1 and the
    // slot of item t + FA_D
    issue(t + FA_D - 1, hvq[FA_D - 1]);
    const uint32_t hv = hvq[0];
#pragma unroll
    for (int u = 0; u < FA_D - 1; ++u) hvq[u] = hvq[u + 1];
    hvq[FA_D - 1] = slot_of(t + FA_D);
    cp_async_wait_group<FA_D - 1>();  // item t's copies of this lane have landed
    const int i = i0 + t * nwarps;
    int f, c;
    const bool valid = fm_item_pos(i, rpw, nk, vpr, d, r_l, j_l, f, c);
    __syncwarp();  // every lane of the item's rows has used its slot value
    if (!valid) continue;
    if (nk == 1 && j_l == 0 && hv) {  // ready for the next step
      slot[f] = 0;
      hist[f] = 0;
    }
    const uint32_t upd = upd_bits(c);
    if (!upd) continue;
    const unsigned char* st = ring + (t % FA_D) * FA_STG + lane * 16;
    float w[4], mm[4], vv[4], g[4] = {0.f, 0.f, 0.f, 0.f};
    load4<W>(st, 0, w);
    const float4 m4 = *reinterpret_cast<const float4*>(st + 512);
    mm[0] = m4.x; mm[1] = m4.y; mm[2] = m4.z; mm[3] = m4.w;
    if (adam) {
      const float4 v4 = *reinterpret_cast<const float4*>(st + 1024);
      vv[0] = v4.x; vv[1] = v4.y; vv[2] = v4.z; vv[3] = v4.w;
    } else {
      vv[0] = vv[1] = vv[2] = vv[3] = 0.f;
    }
    if (hv) {
      const float4 g4 = *reinterpret_cast<const float4*>(st + 1536);
      g[0] = g4.x; g[1] = g4.y; g[2] = g4.z; g[3] = g4.w;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if ((upd >> q) & 1u) opt_apply(w[q], mm[q], vv[q], g[q], o);
    const int64_t off = (int64_t)f * ldw + c;
    store4<W>(Wm, off, w);
    *reinterpret_cast<float4*>(m + off) = make_float4(mm[0], mm[1], mm[2], mm[3]);
    if (adam) *reinterpret_cast<float4*>(v + off) = make_float4(vv[0], vv[1], vv[2], vv[3]);
  }
  cp_async_wait_group<0>();
}

// hist[f] = slot[f] = 0 for the touched features (rows split over several
// items of fm_adam_kernel, which cannot clear them in place).
__global__ void fm_hist_clear_kernel(SegScratch S) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k < (int)S.ctr[0]) {
    S.hist[S.touched[k]] = 0;
    S.slot[S.touched[k]] = 0;
  }
}

// Bias gradient over a long batch: block b owns neurons [8b, 8b + 8).  Its 8
// warps stage the samples' 8-column row segments through shared memory in
// chunks of FB_CH rows, double-buffered with cp.async (many blocks with large
// chunks keep enough bytes in flight); lane j of warp 0 then adds column j in
// ascending sample order (bit-exact).
constexpr int FB_CB = 8, FB_CH = 1024, FB_NT = 256;
constexpr size_t FB_SMEM = (size_t)2 * FB_CH * FB_CB * 4;
__global__ void __launch_bounds__(FB_NT) fm_bias_stream_kernel(float* bias, float* mb, float* vb, const float* lgd,
                                                              int ldl, int nq, int N, const uint32_t* tmask,
                                                              const OptStep* op, unsigned long long* stat_touched) {
  extern __shared__ __align__(16) float brows[];  // [2][FB_CH][FB_CB]
  const OptStep o = *op;
  const int j0 = blockIdx.x * FB_CB;  // ldl is a multiple of 8: the block's 8 columns lie inside the row pitch
  auto stage = [&](int s0, int b) {
    const int cn = min(FB_CH, nq - s0);
    for (int q = threadIdx.x; q < cn * 2; q += FB_NT) {
      const int r = q >> 1, c4 = (q & 1) * 4;
      cp_async16(&brows[((size_t)b * FB_CH + r) * FB_CB + c4], lgd + (int64_t)(s0 + r) * ldl + j0 + c4);
    }
    cp_async_commit();
  };
  float gb = 0.0f;
  stage(0, 0);
  for (int s0 = 0, b = 0; s0 < nq; s0 += FB_CH, b ^= 1) {
    if (s0 + FB_CH < nq) stage(s0 + FB_CH, b ^ 1);
    else cp_async_commit();
    cp_async_wait_group<1>();
    __syncthreads();
    if (threadIdx.x < FB_CB) {
      const int cn = min(FB_CH, nq - s0);
      const float* col = brows + (size_t)b * FB_CH * FB_CB + threadIdx.x;
      int r = 0;
      for (; r + 8 <= cn; r += 8) {  // the group's loads first: only the sum is a chain
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = col[(size_t)(r + u) * FB_CB];
#pragma unroll
        for (int u = 0; u < 8; ++u) gb = __fadd_rn(gb, v[u]);
      }
      for (; r < cn; ++r) gb = __fadd_rn(gb, col[(size_t)r * FB_CB]);
    }
    __syncthreads();
  }
  const int j = j0 + (int)threadIdx.x;
  if (threadIdx.x < FB_CB && j < N && ((tmask[j >> 5] >> (j & 31)) & 1u)) {
    if (stat_touched) atomicAdd(stat_touched, 1ull);
    bias_update(bias, mb, vb, (uint32_t)j, gb, o);
  }
}

// Bias gradient of every touched neuron: one warp per neuron loads 32
// samples' gradients at a time and adds them in ascending sample order.
__global__ void fm_bias_kernel(float* bias, float* mb, float* vb, const float* lgd, int ldl, int nq,
                               int N, const uint32_t* tmask, const OptStep* op,
                               unsigned long long* stat_touched) {
  const OptStep o = *op;
  const int j = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int l = threadIdx.x & 31;
  if (j >= N) return;
  if (!((tmask[j >> 5] >> (j & 31)) & 1u)) return;
  float gb = 0.0f;
  constexpr int R = 8;  // rounds of 32 samples loaded before they are summed
  for (int s00 = 0; s00 < nq; s00 += 32 * R) {
    float mine[R];
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const int sidx = s00 + u * 32 + l;
      mine[u] = sidx < nq ? lgd[(int64_t)sidx * ldl + j] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const int ns = min(32, nq - (s00 + u * 32));
      for (int v = 0; v < ns; ++v) gb = __fadd_rn(gb, __shfl_sync(FULL, mine[u], v));
    }
  }
  if (l == 0) {
    if (stat_touched) atomicAdd(stat_touched, 1ull);
    bias_update(bias, mb, vb, (uint32_t)j, gb, o);
  }
}

// Matrix conversion between reference f32 rows and device storage.
template <class W>
__global__ void f32_to_w_kernel(const float* src, int64_t n_rows, int d, int64_t ld_src, W* dst,
                                int64_t ld_dst, bool transpose) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n_rows * d) return;
  const int64_t r = g / d, c = g % d;
  const W val = from_f<W>(src[r * ld_src + c]);
  if (transpose) dst[c * ld_dst + r] = val;
  else dst[r * ld_dst + c] = val;
}

template <class W>
__global__ void w_to_f32_kernel(const W* src, int64_t ld_src, bool transpose, float* dst, int64_t n_rows,
                                int d) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n_rows * d) return;
  const int64_t r = g / d, c = g % d;
  dst[g] = to_f(transpose ? src[c * ld_src + r] : src[r * ld_src + c]);
}

// Top-k of one sample: actives sorted by (score desc, id asc) with a bitonic
// sort in shared memory; the score-0 tier merges active zeros with inactive
// ids in id order.
constexpr int TK_MAX = 4096;
__global__ void __launch_bounds__(1024) topk_kernel(ActiveSet A, int N, int k, uint32_t* top_ids,
                                                    float* top_scores) {
  __shared__ float sc[TK_MAX];
  __shared__ uint32_t id[TK_MAX];
  const int s = blockIdx.x;
  const int na = min(A.cnt[s], TK_MAX);
  int P = 1;
  while (P < na) P <<= 1;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    if (i < na) {
      sc[i] = A.post[(int64_t)s * A.stride + i];
      id[i] = A.ids[(int64_t)s * A.stride + i];
    } else {
      sc[i] = __int_as_float(0xff800000);
      id[i] = 0xffffffffu;
    }
  }
  __syncthreads();
  // "a before b" if a.score > b.score or (== and a.id < b.id)
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const bool before_ji = sc[j] > sc[i] || (sc[j] == sc[i] && id[j] < id[i]);
          if (before_ji == up) {
            float t = sc[i]; sc[i] = sc[j]; sc[j] = t;
            uint32_t u = id[i]; id[i] = id[j]; id[j] = u;
          }
        }
      }
      __syncthreads();
    }
  }
  if (threadIdx.x != 0) return;
  uint32_t* oi = top_ids + (int64_t)s * k;
  float* os = top_scores ? top_scores + (int64_t)s * k : nullptr;
  int o = 0, p = 0;
  while (o < k && p < na && sc[p] > 0.0f) {
    oi[o] = id[p];
    if (os) os[o] = sc[p];
    ++o; ++p;
  }
  // zero tier: ids (active with score 0, or inactive) ascending
  const uint32_t* act_ids = A.ids + (int64_t)s * A.stride;  // sorted by id
  int q = 0;
  for (uint32_t cand = 0; o < k && cand < (uint32_t)N; ++cand) {
    while (q < na && act_ids[q] < cand) ++q;
    bool active = q < na && act_ids[q] == cand;
    if (active) {
      const float v = A.post[(int64_t)s * A.stride + q];
      if (!(v == 0.0f)) continue;
    }
    oi[o] = cand;
    if (os) os[o] = 0.0f;
    ++o;
  }
  while (o < k && p < na) {
    if (sc[p] < 0.0f) {
      oi[o] = id[p];
      if (os) os[o] = sc[p];
      ++o;
    }
    ++p;
  }
}

}  // namespace

void launch_topk(ActiveSet A, int N, int k, uint32_t* top_ids, float* top_scores, int nq,
                 cudaStream_t st) {
  if (nq <= 0 || k <= 0) return;
  topk_kernel<<<nq, 1024, 0, st>>>(A, N, k, top_ids, top_scores);
  count_launch();
}

void launch_w_to_f32(const void* src, int wdtype, int64_t ld_src, bool transpose, float* dst,
                     int64_t n_rows, int d, cudaStream_t st) {
  const int64_t tot = n_rows * d;
  if (tot <= 0) return;
  const unsigned g = (unsigned)ceil_div(tot, 256);
  if (wdtype == KL_DTYPE_BF16)
    w_to_f32_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(src), ld_src,
                                                       transpose, dst, n_rows, d);
  else
    w_to_f32_kernel<float><<<g, 256, 0, st>>>(static_cast<const float*>(src), ld_src, transpose, dst,
                                              n_rows, d);
  count_launch();
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
void launch_fm_forward(const void* W, int wdtype, int ldw, int d, const float* bias, int act,
                       SparseIn in, ActiveSet A, float* h, int ldh, int* err, cudaStream_t st) {
  if (in.n <= 0) return;
  const size_t rowb = (size_t)ldw * (wdtype == KL_DTYPE_BF16 ? 2 : 4);
  // Wide rows of which only a small part is active (the README MLP's dense
  // 784-dim input against 1024 neurons, ~10 % active) gather the active
  // columns instead of staging whole rows.
  const int gather = rowb > 1024 ? 1 : 0;  // decided per example from its active count
  const int ch = (int)std::max<size_t>(8, std::min<size_t>(64, (size_t)(48 * 1024) / rowb));
  const size_t sm = (size_t)round_up((int64_t)std::max(ch, 64) * 8, 16) + (size_t)ch * rowb;
  static OncePerDevice attr;
  attr([&] {
    cudaFuncSetAttribute(fm_forward_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(fm_forward_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (wdtype == KL_DTYPE_BF16)
    fm_forward_kernel<__nv_bfloat16><<<in.n, 128, sm, st>>>(W, ldw, d, bias, act, in, A, h, ldh, err, ch, gather);
  else
    fm_forward_kernel<float><<<in.n, 128, sm, st>>>(W, ldw, d, bias, act, in, A, h, ldh, err, ch, gather);
  count_launch();
}

template <class W, int MODE, int TILEB>
static void rm_launch(const RmArgs& a, int nq, cudaStream_t st) {
  constexpr int PITCH = TILEB + 16;
  constexpr int EPT = TILEB / (int)sizeof(W);
  const size_t sm = (size_t)round_up((int64_t)a.ldx * 4, 16) + (size_t)RM_NWB * 32 * PITCH +
                    (size_t)RM_NWB * EPT * 4;
  static OncePerDevice attr;
  attr([&] {
    cudaFuncSetAttribute(rm_forward_kernel<W, MODE, TILEB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         200 * 1024);
  });
  dim3 grid(a.nchunk, nq);
  rm_forward_kernel<W, MODE, TILEB><<<grid, RM_RPB, sm, st>>>(a);
  count_launch();
}
template <class W, int MODE>
static void rm_launch_t(const RmArgs& a, int nq, cudaStream_t st) {
  // 256-byte column tiles for every width: wider rows take several tiles, and
  // the smaller staging buffers keep three blocks (24 warps) per SM
  rm_launch<W, MODE, 256>(a, nq, st);
}
void launch_rm_forward(const RmArgs& a, int nq, int mode, cudaStream_t st) {
  if (nq <= 0) return;
  const bool bf = a.wdtype == KL_DTYPE_BF16;
  switch (mode) {
    case RM_FWD:
      bf ? rm_launch_t<__nv_bfloat16, RM_FWD>(a, nq, st) : rm_launch_t<float, RM_FWD>(a, nq, st);
      break;
    case RM_FUSED:
      bf ? rm_launch_t<__nv_bfloat16, RM_FUSED>(a, nq, st) : rm_launch_t<float, RM_FUSED>(a, nq, st);
      break;
    default:
      bf ? rm_launch_t<__nv_bfloat16, RM_DX>(a, nq, st) : rm_launch_t<float, RM_DX>(a, nq, st);
      break;
  }
}
void launch_reduce_dx(const float* dxpart, int nchunk, int ld, int d, const int32_t* cnt, float* dx,
                      int nq, cudaStream_t st) {
  if (nq <= 0) return;
  reduce_dx_kernel<<<nq, 256, 0, st>>>(dxpart, nchunk, ld, d, cnt, dx);
  count_launch();
}
void launch_softmax(ActiveSet A, float* h, int ldh, const int32_t* lab_ptr, const uint32_t* labels,
                    float* labprob, int nq, cudaStream_t st) {
  if (nq <= 0) return;
  softmax_kernel<<<nq, 256, 0, st>>>(A, h, ldh, lab_ptr, labels, labprob);
  count_launch();
}
void launch_local_grads(ActiveSet A, int act, const float* grad, int ldg, float* lgd, int ldl,
                        uint32_t* touched_mask, int nq, cudaStream_t st) {
  if (nq <= 0) return;
  if (act == KL_ACT_SOFTMAX) {
    local_grads_softmax_kernel<<<nq, 256, 0, st>>>(A, grad, ldg, lgd, ldl, touched_mask);
  count_launch();
  } else {
    dim3 grid((unsigned)ceil_div(A.stride, 128), nq);
    local_grads_kernel<<<grid, 128, 0, st>>>(A, act, grad, ldg, lgd, ldl, touched_mask);
  count_launch();
  }
}
void launch_loss(const int32_t* lab_ptr, const float* labprob, int nq, float* accum, cudaStream_t st) {
  if (nq <= 0) return;
  loss_kernel<<<1, 1024, (size_t)nq * 4, st>>>(lab_ptr, labprob, nq, accum);
  count_launch();
}

static int upd_grid() {
  static int g = 0;
  if (!g) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    g = sms * 8;
  }
  return g;
}

__global__ void count_touched_kernel(const uint32_t* ctr, unsigned long long* stat) { *stat += ctr[0]; }
void launch_count_touched(const uint32_t* ctr, unsigned long long* stat, cudaStream_t st) {
  if (!stat) return;
  count_touched_kernel<<<1, 1, 0, st>>>(ctr, stat);
  count_launch();
}

void launch_rm_mark(ActiveSet A, int nq, DenseScratch D, cudaStream_t st, const int32_t* only_empty) {
  if (nq <= 0) return;
  rm_mark_kernel<<<dim3((unsigned)ceil_div(A.stride, 256), nq), 256, 0, st>>>(A, D.mark, D.touched, D.slot_of, D.ctr,
                                                                           only_empty);
  count_launch();
}

bool rm_dense_fits(int64_t rows, int nb, int64_t max_bytes) {
  if (max_bytes < 0) return false;
  if (max_bytes == 0) max_bytes = (int64_t)2 << 30;
  return rows * (int64_t)nb * 4 <= max_bytes;
}

void launch_rm_update_dense(const void* W, int wdtype, int ldw, int d, float* bias, float* m, float* v,
                            float* mb, float* vb, const float* X, int ldx, ActiveSet A, int nq, int N,
                            DenseScratch D, const OptStep* o, unsigned long long* stat_touched,
                            cudaStream_t st, bool premarked) {
  (void)stat_touched;
  if (nq <= 0) return;
  if (!premarked) {
    launch_rm_mark(A, nq, D, st);
    rm_dense_scatter_kernel<<<dim3((unsigned)ceil_div(A.stride, 256 * RM_PK), nq), 256, 0, st>>>(A, D.slot_of, D.LGd,
                                                                                                 D.ldb);
    count_launch();
  }
  const int64_t maxn = std::min<int64_t>((int64_t)N, (int64_t)nq * A.stride);
  const int ncb = (int)ceil_div(d, RDU_COLS);
  // Long sample loops (large batches) meet few touched rows per shard: blocks
  // of 2 warps x 4 rows (8 rows each) give 4x the blocks of 8 x 4 while each
  // thread keeps 4 rows per staged sample.
  const int nwb = nq >= 512 ? 2 : 8;
  constexpr int NST = 4;  // cp.async stages (deeper pipelines measured no faster)
  const int grid = (int)std::min<int64_t>((int64_t)upd_grid() * 8 / nwb, ceil_div(maxn, 4 * nwb) * ncb);
  void* Wv = const_cast<void*>(W);
#define KL_RDU(WT, NW)                                                                                        \
  do {                                                                                                        \
    const size_t sm = (size_t)NST * RDU_S * (RDU_COLS + NW * 4) * 4;                                          \
    static OncePerDevice a_;                                                                                  \
    a_([&] {                                                                                                  \
      cudaFuncSetAttribute(rm_dense_update_kernel<WT, 4, NW, NST>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           (int)sm);                                                                          \
    });                                                                                                       \
    rm_dense_update_kernel<WT, 4, NW, NST><<<grid, NW * 32, sm, st>>>(Wv, ldw, d, bias, m, v, mb, vb, X, ldx,   \
                                                                       D.mark, D.touched, D.ctr, D.LGd, D.ldb, nq, o); \
  } while (0)
  if (wdtype == KL_DTYPE_BF16) {
    if (nwb == 2) KL_RDU(__nv_bfloat16, 2);
    else KL_RDU(__nv_bfloat16, 8);
  } else {
    if (nwb == 2) KL_RDU(float, 2);
    else KL_RDU(float, 8);
  }
#undef KL_RDU
  count_launch();
  rm_lg_zero_kernel<<<upd_grid(), 256, 0, st>>>(D.LGd, D.ldb, D.ctr);
  count_launch();
}

void launch_rm_update(const void* W, int wdtype, int ldw, int d, float* bias, float* m, float* v,
                      float* mb, float* vb, const float* X, int ldx, ActiveSet A, int nq, int N,
                      SegScratch S, const OptStep* o, unsigned long long* stat_touched,
                      cudaStream_t st) {
  if (nq <= 0) return;
  dim3 g2((unsigned)ceil_div(A.stride, 256), nq);
  rm_touch_kernel<<<g2, 256, 0, st>>>(A, S.hist, S.touched, S.ctr);
  count_launch();
  const int maxn = (int)std::min<int64_t>((int64_t)N, (int64_t)nq * A.stride);
  seg_alloc_kernel<<<(unsigned)ceil_div(maxn, 256), 256, 0, st>>>(S.hist, S.touched, S.cur, S.ctr, maxn);
  count_launch();
  rm_scatter_kernel<<<g2, 256, 0, st>>>(A, S.cur, S.ent_s, S.ent_v);
  count_launch();
  const int nwords = (int)ceil_div(nq, 32);
  // per warp: mask, coefficients and the 16-bit sample list (<= 200 KB at 4096 samples)
  const size_t sm = (size_t)UPD_WARPS * nwords * (4 * 33 + 2 * 32);
  const int grid = (int)std::min<int64_t>(upd_grid(), ceil_div(maxn, UPD_WARPS));
  if (wdtype == KL_DTYPE_BF16) {
    cudaFuncSetAttribute(rm_update_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    rm_update_kernel<__nv_bfloat16><<<grid, UPD_WARPS * 32, sm, st>>>(
        const_cast<void*>(W), ldw, d, bias, m, v, mb, vb, X, ldx, S, nwords, o, stat_touched);
  count_launch();
  } else {
    cudaFuncSetAttribute(rm_update_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    rm_update_kernel<float><<<grid, UPD_WARPS * 32, sm, st>>>(
        const_cast<void*>(W), ldw, d, bias, m, v, mb, vb, X, ldx, S, nwords, o, stat_touched);
  count_launch();
  }
}

void launch_fm_update(const void* W, int wdtype, int ldw, int d, int f0, int nf, int N, float* bias, float* m,
                      float* v, float* mb, float* vb, SparseIn in, const float* lgd, int ldl,
                      const uint32_t* touched_mask, SegScratch S, float* G, const OptStep* o,
                      unsigned long long* stat_touched, int* err, cudaStream_t st,
                      void (*around_adam)(void*, int), void* hook_arg) {
  const int nq = in.n;
  if (nq <= 0) return;
  (void)d;
  fm_touch_kernel<<<nq, 256, 0, st>>>(in, S.hist, S.touched, S.ctr, (uint32_t)f0, (uint32_t)nf);
  count_launch();
  seg_alloc_kernel<<<(unsigned)ceil_div(std::max(nf, 1), 256), 256, 0, st>>>(S.hist, S.touched, S.cur, S.ctr, nf);
  count_launch();
  fm_scatter_kernel<<<nq, 256, 0, st>>>(in, S.cur, S.ent_s, S.ent_v, (uint32_t)f0, (uint32_t)nf);
  count_launch();
  const int ggrid = (int)std::min<int64_t>((int64_t)upd_grid() * 2, ceil_div(std::max(nf, 1), FM_GW));
  fm_grad_short_kernel<<<ggrid, FM_GW * 32, 0, st>>>(N, lgd, ldl, S, G, ldl);
  count_launch();
  const int nwords = (int)ceil_div(nq, 32);
  // staged gradient rows: two chunks of `chr` rows, at most 64 KB
  const int chr = std::max(4, std::min(64, (int)((32 * 1024) / ((size_t)ldl * 4))));
  const size_t sm = (size_t)round_up((int64_t)nwords * 4 * 65, 16) + (size_t)2 * chr * ldl * 4;
  static OncePerDevice attr;
  attr([&] {
    cudaFuncSetAttribute(fm_grad_long_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  const int lthreads = std::min(1024, 32 * (int)ceil_div(N, 32));
  fm_grad_long_kernel<<<upd_grid(), lthreads, sm, st>>>(N, lgd, ldl, S, nwords, G, ldl, chr);
  count_launch();
  const int vpr = ldl / 4;  // vectors per feature row (ldw == ldl == pitch of N)
  const int rpw = vpr <= 32 ? 32 / vpr : 1;
  const int nk = vpr <= 32 ? 1 : (int)ceil_div(vpr, 32);
  const size_t smem = (size_t)(FA_NT / 32) * FA_D * FA_STG;
  static OncePerDevice attr_adam;
  attr_adam([&] {
    cudaFuncSetAttribute(fm_adam_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(fm_adam_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int agrid = sms * 4;  // resident blocks per SM under the kernel's launch bounds
  (void)err;
  if (around_adam) around_adam(hook_arg, 0);
  // the slice's rows: row pointers, optimizer state and per-feature slots offset by f0
  const int64_t ro = (int64_t)f0 * ldw;
  if (wdtype == KL_DTYPE_BF16)
    fm_adam_kernel<__nv_bfloat16><<<agrid, FA_NT, smem, st>>>(
        const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(W)) + ro, ldw, nf, vpr, rpw, nk, N, m + ro,
        v + ro, touched_mask, S.hist + f0, S.slot + f0, G, ldl, o);
  else
    fm_adam_kernel<float><<<agrid, FA_NT, smem, st>>>(const_cast<float*>(static_cast<const float*>(W)) + ro, ldw, nf,
                                                      vpr, rpw, nk, N, m + ro, v + ro, touched_mask, S.hist + f0,
                                                      S.slot + f0, G, ldl, o);
  count_launch();
  if (around_adam) around_adam(hook_arg, 1);
  if (nk > 1) {
    fm_hist_clear_kernel<<<(unsigned)ceil_div(std::max(nf, 1), 256), 256, 0, st>>>(S);
    count_launch();
  }
  if (nq >= 512) {
    // long batches: 32 neurons per block, gradient rows streamed through shared memory
    static OncePerDevice fbattr;
    fbattr([&] {
      cudaFuncSetAttribute(fm_bias_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FB_SMEM);
    });
    fm_bias_stream_kernel<<<(unsigned)ceil_div(N, FB_CB), FB_NT, FB_SMEM, st>>>(bias, mb, vb, lgd, ldl, nq, N,
                                                                               touched_mask, o,
                                                                      stat_touched);
  } else {
    fm_bias_kernel<<<(unsigned)ceil_div(N, 8), 256, 0, st>>>(bias, mb, vb, lgd, ldl, nq, N, touched_mask, o,
                                                             stat_touched);
  }
  count_launch();
}

void launch_f32_to_w(const float* src, int64_t n_rows, int d, int64_t ld_src, void* dst, int wdtype,
                     int64_t ld_dst, bool transpose, cudaStream_t st) {
  const int64_t tot = n_rows * d;
  if (tot <= 0) return;
  const unsigned g = (unsigned)ceil_div(tot, 256);
  if (wdtype == KL_DTYPE_BF16)
    f32_to_w_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(src, n_rows, d, ld_src,
                                                       static_cast<__nv_bfloat16*>(dst), ld_dst, transpose);
  else
    f32_to_w_kernel<float><<<g, 256, 0, st>>>(src, n_rows, d, ld_src, static_cast<float*>(dst), ld_dst,
                                              transpose);
  count_launch();
}

}  // namespace kl
