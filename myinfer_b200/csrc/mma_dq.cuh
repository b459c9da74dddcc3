// Shared pieces of the register-prefetch tensor-core GEMVs (gemv_mma.cu,
// moe_mma.cu): 4-bit codes as bf16 MMA operands and non-caching weight loads.
#pragma once

#include "common.cuh"

namespace m5 {

// bf16 pair (128 + q_i, 128 + q_{i+4}) of nibbles i and i+4 of w, exactly.
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int i) {
  return ((w >> (4 * i)) & 0x000F000Fu) | 0x43004300u;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint2 ldg_nc_u2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint16_t ldg_nc_u16(const void* p) {
  uint16_t r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

}  // namespace m5
