// tcgen05.cuh -- the Blackwell tensor-core and TMA primitives shared by the
// engine's GEMM kernels (hash_tc.cu, dejavu.cu): UMMA shared-memory
// descriptors for the 128-byte-swizzled K-major layout that TMA writes,
// kind::f16 instruction descriptors, tcgen05.mma / commit / ld, 2-D tiled TMA
// loads (never with cluster multicast) and the host-side tensor-map encoder.
#pragma once

#include <cuda.h>

#include <cstdint>

#include "common.cuh"

namespace kl {

__device__ __forceinline__ void tc5_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc5_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// UMMA shared-memory descriptor, K-major, 128-byte swizzle: 8-row groups of
// 1024 bytes (stride byte offset), descriptor version 1, layout type 2.  The
// tile must start on a 1024-byte boundary; a K step of 16 bf16 inside the
// 128-byte swizzle atom adds 32 bytes to the start address.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}
// kind::f16 instruction descriptor: f32 accumulator, bf16 A and B, both
// K-major, M = m (64 or 128), N = n (a multiple of 16 up to 256).
__host__ __device__ constexpr uint32_t f16_idesc(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void tc5_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}
// arrives on `bar` when every MMA this thread issued before it has completed
__device__ __forceinline__ void tc5_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}
// 16 consecutive accumulator columns of the calling thread's lane (32x32b
// shape: warp w reads lanes 32 * (w % 4) ..); tc5_ld_wait() before use.
__device__ __forceinline__ void tc5_ld16_async(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tc5_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tc5_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst_smem)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tc5_dealloc(uint32_t tmem, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(cols) : "memory");
}
// 2-D tiled TMA load into this CTA's shared memory (no multicast): the box at
// element coordinates (x, y) completes on `bar`.  x * 2 bytes must be a
// multiple of 16 (callers pass multiples of 64 bf16).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

// Host: tensor map of a bf16 matrix [rows][cols] with a row pitch of `ld`
// elements, box = box_cols x box_rows, 128-byte swizzle, zero fill outside
// the matrix.  False when the driver entry point is missing or the encoder
// refuses the arguments (base or pitch not 16-byte aligned, box too large).
bool tma_map_bf16(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols,
                  int box_rows);

}  // namespace kl
