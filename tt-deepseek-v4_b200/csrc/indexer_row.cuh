// The indexer score of ONE key row (inference.py:5260-5275 for a single t):
// sum_h w[h] relu(q[h, :] . key) over the 64 heads of one sequence, used by
// the top-k kernels to recompute the newest compressed row's score, which
// the indexer compressor may write after the score matrix was computed.
#pragma once

#include "common.cuh"

namespace dsa {

constexpr int kRowHeads = 64;
constexpr int kRowDim = 128;

// q [64 x 128] bf16, key [128] bf16 (8-byte aligned), w [64] fp32.  Called by
// every thread of the block (any whole number of warps); each warp takes
// heads warp, warp + nwarps, ...; lane l covers dims 4l .. 4l + 3, a fixed
// shuffle tree sums them; the heads are accumulated in order h = 0..63 like
// the score kernel's epilogue.  s_dot: 64 floats of shared memory.  Every
// thread returns the score.
__device__ __forceinline__ float indexer_row_score(const __nv_bfloat16* __restrict__ q,
                                                   const __nv_bfloat16* __restrict__ key,
                                                   const float* __restrict__ w, float* s_dot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const uint2 kraw = *reinterpret_cast<const uint2*>(key + 4 * lane);
  const float2 k01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kraw.x));
  const float2 k23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kraw.y));
  for (int h = warp; h < kRowHeads; h += nwarps) {
    const uint2 qraw = *reinterpret_cast<const uint2*>(q + int64_t(h) * kRowDim + 4 * lane);
    const float2 q01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qraw.x));
    const float2 q23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qraw.y));
    float d = q01.x * k01.x;
    d = fmaf(q01.y, k01.y, d);
    d = fmaf(q23.x, k23.x, d);
    d = fmaf(q23.y, k23.y, d);
    d = warp_sum(d);
    if (lane == 0) s_dot[h] = d;
  }
  __syncthreads();
  float sc = 0.f;
  for (int h = 0; h < kRowHeads; ++h) sc = fmaf(w[h], fmaxf(s_dot[h], 0.f), sc);
  return sc;
}

// The score of sequence b's newest live row, t = min(t_active[b], T) - 1,
// into score[b, t] (nothing when t < 0): indexer_score_newest_kernel
// (indexer.cu) and the decode layer's prologue kernel (prologue.cu).
__device__ __forceinline__ void score_newest_row(const __nv_bfloat16* __restrict__ q,
                                                 const __nv_bfloat16* __restrict__ k, int64_t k_bstride,
                                                 const float* __restrict__ w, const int32_t* __restrict__ t_active,
                                                 float* __restrict__ score, int64_t ld_score, int T, int b,
                                                 float* s_dot) {
  const int t = min(t_active[b], T) - 1;
  if (t < 0) return;  // uniform across the block
  const float sc = indexer_row_score(q + int64_t(b) * kRowHeads * kRowDim, k + int64_t(b) * k_bstride +
                                     int64_t(t) * kRowDim, w + int64_t(b) * kRowHeads, s_dot);
  if (threadIdx.x == 0) score[int64_t(b) * ld_score + t] = sc;
}

}  // namespace dsa
