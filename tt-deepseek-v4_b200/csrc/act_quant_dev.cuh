// attn.kv's block-wise FP8-E4M3 round trip of one warp's block and the
// window-ring write of one sequence's row as device functions: used by
// act_quant.cu's kernels and by the decode layer's prologue kernel
// (prologue.cu).  Semantics in act_quant.cu.
#pragma once

#include "common.cuh"

namespace dsa {

template <int EPL>
__device__ __forceinline__ void quant_block_lane(const __nv_bfloat16* __restrict__ src,
                                                 __nv_bfloat16* __restrict__ dst, float* scale_out,
                                                 uint8_t* codes_out, int lane, float fp8_max,
                                                 float inv_max, float eps) {
  float v[EPL];
  if constexpr (EPL == 2) {
    __nv_bfloat162 h = reinterpret_cast<const __nv_bfloat162*>(src)[lane];
    float2 f = __bfloat1622float2(h);
    v[0] = f.x;
    v[1] = f.y;
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = bf2f(src[lane * EPL + i]);
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = warp_max(amax);
  const float s = __fmul_rn(fmaxf(amax, eps), inv_max);
  uint8_t qb[EPL];
  float o[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    float y = __fdiv_rn(v[i], s);
    y = fminf(fmaxf(y, -fp8_max), fp8_max);
    __nv_fp8_storage_t q = __nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3);
    qb[i] = static_cast<uint8_t>(q);
    __half_raw hr = __nv_cvt_fp8_to_halfraw(q, __NV_E4M3);
    o[i] = __half2float(__half(hr)) * s;
  }
  if constexpr (EPL == 2) {
    reinterpret_cast<__nv_bfloat162*>(dst)[lane] = __floats2bfloat162_rn(o[0], o[1]);
    if (codes_out) {
      uint16_t pk = (uint16_t)qb[0] | ((uint16_t)qb[1] << 8);
      reinterpret_cast<uint16_t*>(codes_out)[lane] = pk;
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      dst[lane * EPL + i] = f2bf(o[i]);
      if (codes_out) codes_out[lane * EPL + i] = qb[i];
    }
  }
  if (scale_out && lane == 0) *scale_out = s;
}

// One sequence's row (D = nope + rope dims) into ring slot pos[b] % win:
// warps [0, nope/64) quantise a block each (the rest of the CTA's warps
// take further blocks), then the rope dims are copied.  Any whole number of
// warps per CTA.
__device__ __forceinline__ void kv_window_write_row(const __nv_bfloat16* __restrict__ kv,
                                                    __nv_bfloat16* __restrict__ cache, float* __restrict__ scales,
                                                    const int32_t* __restrict__ pos, int D, int rope_dim,
                                                    int64_t cache_bstride, int win, float fp8_max, float inv_max,
                                                    float eps, int b) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nope = D - rope_dim;
  const int nblk = nope / 64;
  const int p = pos[b];
  const int slot = ((p % win) + win) % win;
  const __nv_bfloat16* src = kv + int64_t(b) * D;
  __nv_bfloat16* dst = cache + int64_t(b) * cache_bstride + int64_t(slot) * D;
  const int nwarps = blockDim.x >> 5;
  for (int blk = warp; blk < nblk; blk += nwarps)
    quant_block_lane<2>(src + blk * 64, dst + blk * 64, scales ? scales + int64_t(b) * nblk + blk : nullptr,
                        nullptr, lane, fp8_max, inv_max, eps);
  for (int c = threadIdx.x; c < rope_dim; c += blockDim.x) dst[nope + c] = src[nope + c];
}

}  // namespace dsa
