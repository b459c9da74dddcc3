// Shared helpers for libm5cuda: status codes, error text, bf16 conversions,
// warp reductions and the 128-bit streaming loads used by the decode kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/m5cuda.h"

namespace m5 {

// Per-thread text of the last failure; read through m5_last_error().
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define M5_CHECK_ARG(cond, msg)                                   \
  do {                                                            \
    if (!(cond)) return ::m5::fail(M5_ERR_INVALID, (msg));        \
  } while (0)

#define M5_CUDA(call)                                             \
  do {                                                            \
    cudaError_t _e = (call);                                      \
    if (_e != cudaSuccess) return ::m5::cuda_fail(_e, #call);     \
  } while (0)

// A launch error is reported without synchronising the stream.
#define M5_LAUNCH_CHECK(what)                                     \
  do {                                                            \
    cudaError_t _e = cudaGetLastError();                          \
    if (_e != cudaSuccess) return ::m5::cuda_fail(_e, (what));    \
  } while (0)

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ bf16 f2bf(float v) { return __float2bfloat16_rn(v); }
// Round an fp32 value to the nearest bf16 and return it as fp32.
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 16-byte read-only load that does not allocate in L1: packed weights are
// streamed exactly once per token.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Packed fp32x2 FMA (sm_100): d = a * b + c on two lanes of a 64-bit register.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long ra = *reinterpret_cast<unsigned long long*>(&a);
  unsigned long long rb = *reinterpret_cast<unsigned long long*>(&b);
  unsigned long long rc = *reinterpret_cast<unsigned long long*>(&c);
  unsigned long long rd;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
  return *reinterpret_cast<float2*>(&rd);
}

// 4-bit code held in byte j of `lo` (0..15) -> the fp32 value 128 + code.
// 0x43 in the top byte is the exponent of 128.0f; the code lands on mantissa
// bits 16..19, whose unit is exactly 1.0 in that binade.
template <int J>
__device__ __forceinline__ float nib128(uint32_t lo) {
  return __uint_as_float(__byte_perm(lo, 0x43u, 0x4055u | (J << 8)));
}
// 8-bit code in byte j -> the fp32 value 32768 + code (exponent of 32768.0f,
// code on mantissa bits 8..15 whose unit is 1.0).
template <int J>
__device__ __forceinline__ float byte32768(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x47u, 0x4505u | (J << 4)));
}

inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

// Runs a per-device set-up step (cudaFuncSetAttribute and the like, whose
// effect belongs to the current device's context) once for each device, from
// any number of host threads.  One instance per call site:
//   static DeviceOnce once;
//   M5_CUDA(once.run([&] { return cudaFuncSetAttribute(...); }));
// A failed step is not recorded, so the next call retries it.
struct DeviceOnce {
  std::atomic<unsigned long long> done{0};
  std::mutex mu;
  template <class Fn>
  cudaError_t run(Fn&& fn) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return fn();  // beyond the mask: set every time
    const unsigned long long bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    std::lock_guard<std::mutex> lk(mu);
    if (done.load(std::memory_order_relaxed) & bit) return cudaSuccess;
    e = fn();
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
    return e;
  }
};

int sm_count();  // SMs of the current device (cached)

// Programmatic dependent launch.  A kernel launched with launch_pdl() may start
// while the previous kernel on the stream is still running: it must execute
// pdl_wait() before touching anything an earlier kernel writes (or reading
// what it reads and later kernels write), and it lets the next kernel start
// early with pdl_launch_dependents().  Work that depends on nothing earlier
// (streaming constant weights into shared memory) goes before the wait.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

bool pdl_enabled();  // true only when M5_PDL=1 is set in the environment

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace m5
