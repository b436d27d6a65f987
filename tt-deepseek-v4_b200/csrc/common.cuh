// Shared helpers for the dsv4attn sm_100a kernels: status plumbing, bf16 /
// e4m3 conversions, warp reductions, cp.async and programmatic dependent
// launch.  Everything here is header-only device/host code.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdio.h>
#include <string>
#include <algorithm>
#include <utility>

#include "../../include/dsv4attn.h"

namespace dsa {

// ---------------------------------------------------------------- status
void set_error(const char* fmt, ...);
void clear_error();

#define DSA_CHECK_ARG(cond, ...)                 \
  do {                                           \
    if (!(cond)) {                               \
      ::dsa::set_error(__VA_ARGS__);             \
      return DSA_ERR_ARG;                        \
    }                                            \
  } while (0)

#define DSA_CHECK_LAUNCH(what)                                              \
  do {                                                                      \
    cudaError_t e__ = cudaGetLastError();                                   \
    if (e__ != cudaSuccess) {                                               \
      ::dsa::set_error("%s: launch failed: %s", what, cudaGetErrorString(e__)); \
      return DSA_ERR_CUDA;                                                  \
    }                                                                       \
  } while (0)

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int num_sms();  // cached per device

// Spin budget, in SM clock cycles, of every bounded device-side wait the
// library's kernels take (mbarrier waits, grid barriers, peer flags); set
// with dsa_set_wait_limit, about one second by default.  Passed to each
// kernel as an argument at launch.
long long wait_limit_cycles();

// ----------------------------------------------------------- conversions
__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }

// unpack 8 bf16 packed in a uint4 to fp32
__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------- reductions
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ----------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte async global->shared copy; src_bytes = 0 zero-fills the destination
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ---------------------------------------------- programmatic dependent launch
// Kernels of the decode chain are launched with programmatic stream
// serialisation: the next kernel of the stream may start (set up shared
// memory, barriers, TMEM) while this one drains.  Every such kernel calls
// pdl_wait() before its first global-memory access - it returns once the
// previous kernel of the stream has completed and its writes are visible
// (immediately when the launch had no programmatic dependency) - and then
// pdl_launch_dependents(), which lets the next kernel be scheduled once all
// CTAs of this one have reached it.  No CTA touches global memory before its
// wait, so reads after writes and writes after reads across the chain keep
// stream order.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
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
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// order-preserving map float -> uint32 (larger float -> larger key)
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

}  // namespace dsa
