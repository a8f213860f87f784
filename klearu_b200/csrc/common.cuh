// common.cuh -- shared device helpers for the klearu B200 engine (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/klearu_gpu.h"

namespace kl {

// Function attributes such as the dynamic shared memory limit apply to the
// device that is current when they are set.  A launch site keeps one
// OncePerDevice and runs its set-up through it: the set-up runs once on each
// device the process launches on, under a lock shared by the host threads.
struct OncePerDevice {
  std::mutex mu;
  unsigned long long done = 0;
  template <class F>
  void operator()(F&& f) {
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    std::lock_guard<std::mutex> g(mu);
    if (!(done & bit)) {
      f();
      done |= bit;
    }
  }
};

// Device-side error word bits (never __trap: kernels record and return).
enum : int {
  DERR_BOUNDS = 1,    // id / index outside its array
  DERR_CAPACITY = 2,  // an output did not fit its buffer (truncated)
  DERR_TIMEOUT = 4,   // a bounded wait gave up
  DERR_TMA = 8,       // a TMA tensor map could not be encoded (nothing was launched)
};

constexpr int WARP = 32;
constexpr unsigned FULL = 0xffffffffu;

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

// Row pitch (elements) of every weight / activation matrix: rows start on
// 32-byte boundaries so 16-byte vector loads and cp.async are always aligned.
__host__ __device__ inline int pitch_of(int n) { return (int)round_up(n, 8); }

// ---- weight element access (f32 or bf16 storage, f32 arithmetic) ----
__device__ __forceinline__ float to_f(float x) { return x; }
// bf16 -> f32 is exact: a bf16 value is the upper half of the f32 with the
// same bits, so the widening is a 16-bit shift on the integer pipe.
__device__ __forceinline__ float to_f(__nv_bfloat16 x) {
  return __uint_as_float((uint32_t)__bfloat16_as_ushort(x) << 16);
}
template <class W>
__device__ __forceinline__ W from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// ---- warp / block scans ----
__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ unsigned lanemask_lt() { return (1u << lane_id()) - 1u; }

__device__ __forceinline__ int warp_incl_scan(int v) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(FULL, v, o);
    if ((int)lane_id() >= o) v += t;
  }
  return v;
}
__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ int warp_max(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(FULL, v, o));
  return v;
}

// Exclusive block scan of one int per thread; `tmp` holds >= 33 ints.
// Returns the exclusive prefix; *total receives the block sum.
template <int NT>
__device__ __forceinline__ int block_excl_scan(int v, int* tmp, int* total) {
  constexpr int NW = NT / 32;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  int inc = warp_incl_scan(v);
  if (l == 31) tmp[w] = inc;
  __syncthreads();
  if (w == 0) {
    int x = l < NW ? tmp[l] : 0;
    int xi = warp_incl_scan(x);
    if (l < NW) tmp[l] = xi - x;
    if (l == NW - 1) tmp[32] = xi;
  }
  __syncthreads();
  int r = tmp[w] + inc - v;
  *total = tmp[32];
  __syncthreads();
  return r;
}
template <int NT>
__device__ __forceinline__ int block_sum(int v, int* tmp) {
  int tot;
  block_excl_scan<NT>(v, tmp, &tot);
  return tot;
}
template <int NT>
__device__ __forceinline__ int block_max(int v, int* tmp) {
  constexpr int NW = NT / 32;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  v = warp_max(v);
  if (l == 0) tmp[w] = v;
  __syncthreads();
  if (w == 0) {
    int x = l < NW ? tmp[l] : INT32_MIN;
    x = warp_max(x);
    if (l == 0) tmp[32] = x;
  }
  __syncthreads();
  int r = tmp[32];
  __syncthreads();
  return r;
}

// Warp-aggregated append: every lane with `pred` gets a unique slot in
// [*counter, *counter + popc).  One atomic per warp.
__device__ __forceinline__ int warp_append(bool pred, unsigned* counter) {
  unsigned m = __ballot_sync(__activemask(), pred);
  if (!pred) return -1;
  int leader = __ffs(m) - 1;
  unsigned base = 0;
  if ((int)lane_id() == leader) base = atomicAdd(counter, (unsigned)__popc(m));
  base = __shfl_sync(m, base, leader);
  return (int)(base + __popc(m & lanemask_lt()));
}

// ---- cp.async (Ampere+ LDGSTS, 16 bytes, L2-only caching) ----
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ---- mbarriers in shared memory (completion of TMA copies and tensor-core
// work).  No cluster multicast anywhere in this library. ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// makes initialised barriers visible to the async proxy
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
// orders earlier generic-proxy shared-memory accesses before later async-proxy ones
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
// Waits for the barrier phase of parity `parity` to complete; gives up after
// about limit_ns nanoseconds and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 20000000ull) {
  const uint32_t a = smem_u32(bar);
  uint64_t t0 = 0;
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    const uint64_t t = global_ns();
    if (t0 == 0) t0 = t;
    else if (t - t0 > limit_ns) return false;
  }
}

// ---- SplitMix64 mixer of ReservoirBucket::deterministic_rand
// (crates/klearu-core/src/bucket/reservoir.rs:36-44) ----
__host__ __device__ __forceinline__ uint64_t splitmix_mod(uint64_t seed, uint64_t bound) {
  uint64_t z = seed + 0x9e3779b97f4a7c15ULL;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  z = z ^ (z >> 31);
  return z % bound;
}

// ---- activations (crates/klearu-core/src/network/layer.rs:250-283) ----
__device__ __forceinline__ float act_apply(float x, int act) {
  switch (act) {
    case KL_ACT_RELU: return fmaxf(x, 0.0f);
    case KL_ACT_SIGMOID: return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
    case KL_ACT_TANH: return tanhf(x);
    default: return x;
  }
}
__device__ __forceinline__ float act_deriv(float pre, float post, int act) {
  switch (act) {
    case KL_ACT_RELU: return pre > 0.0f ? 1.0f : 0.0f;
    case KL_ACT_SIGMOID: return __fmul_rn(post, __fsub_rn(1.0f, post));
    case KL_ACT_TANH: return __fsub_rn(1.0f, __fmul_rn(post, post));
    default: return 1.0f;
  }
}

}  // namespace kl
