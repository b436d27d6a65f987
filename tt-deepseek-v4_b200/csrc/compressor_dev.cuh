// attn.compress's per-sequence step as a device function: the body of
// compressor_step_kernel (compressor.cu) and of the decode layer's prologue
// kernel (prologue.cu).  One CTA of kCmpThreads threads per sequence.
#pragma once

#include "common.cuh"

namespace dsa {


constexpr int kCmpThreads = 256;
constexpr int kCmpMaxD = 1024;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (warp == 0) {
    t = (lane < (int)(blockDim.x >> 5)) ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  t = red[0];
  __syncthreads();
  return t;
}

// Softmax over the slot axis of the (overlap) view and the weighted sum for
// this thread's columns; returns the thread's sum of squares.  With NS > 0
// the slot count is a compile-time constant, so each column's NS scores and
// values are loaded together instead of as a chain of dependent loads.
template <int NS>
__device__ __forceinline__ float emit_columns(const float* kvs, const float* scs, float* s_row, int d, int cd,
                                              int ratio, int overlap, int nslots_rt = 0) {
  float ss = 0.f;
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float v;
    if constexpr (NS > 0) {
      float sc[NS], kv[NS];
#pragma unroll
      for (int i = 0; i < NS; ++i) {
        const int col = (overlap && i >= ratio) ? d + c : c;
        sc[i] = scs[int64_t(i) * cd + col];
        kv[i] = kvs[int64_t(i) * cd + col];
      }
      float m = -INFINITY;
#pragma unroll
      for (int i = 0; i < NS; ++i) m = fmaxf(m, sc[i]);
      float den = 0.f, num = 0.f;
#pragma unroll
      for (int i = 0; i < NS; ++i) {
        const float e = expf(sc[i] - m);
        den += e;
        num = fmaf(e, kv[i], num);
      }
      v = __fdiv_rn(num, den);
    } else {
      float m = -INFINITY;
      for (int i = 0; i < nslots_rt; ++i) {
        const int col = (overlap && i >= ratio) ? d + c : c;
        m = fmaxf(m, scs[int64_t(i) * cd + col]);
      }
      float den = 0.f, num = 0.f;
      for (int i = 0; i < nslots_rt; ++i) {
        const int col = (overlap && i >= ratio) ? d + c : c;
        const float e = expf(scs[int64_t(i) * cd + col] - m);
        den += e;
        num = fmaf(e, kvs[int64_t(i) * cd + col], num);
      }
      v = __fdiv_rn(num, den);
    }
    s_row[c] = v;
    ss = fmaf(v, v, ss);
  }
  return ss;
}

// Arguments of one compressor step (see dsa_compressor_step).
struct CmpStep {
  const __nv_bfloat16* kv_row;
  const __nv_bfloat16* score_row;
  int64_t ld_row;
  const float* ape;
  float* kv_state;
  float* score_state;
  const float* gamma;
  const float* cos_tab;
  const float* sin_tab;
  int n_pos;
  __nv_bfloat16* cache;
  int64_t cache_bstride, cache_rows;
  int slot_offset;
  const int32_t* pos;
  int32_t* emitted;
  int d, rope_dim, ratio, overlap, rotate, write_state;
  float had_scale, eps;
};

// The step for sequence b: state write, and on emit steps the softmax-sum,
// RMSNorm, rotary, optional Hadamard, the compressed row's write and the
// slot shift.  Called by every thread of the CTA; s_row: kCmpMaxD floats,
// s_red: 32 floats of shared memory.
__device__ __forceinline__ void compressor_step_row(const CmpStep& a, int b, float* s_row, float* s_red) {
  const __nv_bfloat16* __restrict__ kv_row = a.kv_row;
  const __nv_bfloat16* __restrict__ score_row = a.score_row;
  const int64_t ld_row = a.ld_row;
  const float* __restrict__ ape = a.ape;
  float* __restrict__ kv_state = a.kv_state;
  float* __restrict__ score_state = a.score_state;
  const float* __restrict__ gamma = a.gamma;
  const float* __restrict__ cos_tab = a.cos_tab;
  const float* __restrict__ sin_tab = a.sin_tab;
  const int n_pos = a.n_pos;
  __nv_bfloat16* __restrict__ cache = a.cache;
  const int64_t cache_bstride = a.cache_bstride, cache_rows = a.cache_rows;
  const int slot_offset = a.slot_offset;
  const int32_t* __restrict__ pos = a.pos;
  int32_t* __restrict__ emitted = a.emitted;
  const int d = a.d, rope_dim = a.rope_dim, ratio = a.ratio, overlap = a.overlap, rotate = a.rotate;
  const int write_state = a.write_state;
  const float had_scale = a.had_scale, eps = a.eps;
  const int tid = threadIdx.x;
  const int p = pos[b];
  const int coff = overlap ? 2 : 1;
  const int cd = coff * d;
  const int nslots = coff * ratio;
  float* kvs = kv_state + int64_t(b) * nslots * cd;
  float* scs = score_state + int64_t(b) * nslots * cd;
  const int pr = p % ratio;
  const int slot = overlap ? ratio + pr : pr;

  // ---- state write (score gets the absolute-position embedding ape[pos % r])
  const __nv_bfloat16* kr = kv_row + int64_t(b) * ld_row;
  const __nv_bfloat16* sr = score_row + int64_t(b) * ld_row;
  const float* ape_row = ape + int64_t(pr) * cd;
  if (write_state) {
    for (int c = tid; c < cd; c += blockDim.x) {
      kvs[int64_t(slot) * cd + c] = bf2f(kr[c]);
      scs[int64_t(slot) * cd + c] = __fadd_rn(bf2f(sr[c]), ape_row[c]);
    }
  }
  const bool emit = ((p + 1) % ratio) == 0;
  const int64_t out_row = int64_t(slot_offset) + p / ratio;
  const int cs_row = p + 1 - ratio;
  const bool in_range = out_row >= 0 && out_row < cache_rows && cs_row >= 0 && cs_row < n_pos;
  if (emitted && tid == 0) emitted[b] = emit ? (in_range ? 1 : -1) : 0;
  if (!emit || !in_range) return;
  __syncthreads();

  // ---- softmax over the slot axis of the (overlap) view, weighted sum
  float ss = 0.f;
  if (nslots == 8) ss = emit_columns<8>(kvs, scs, s_row, d, cd, ratio, overlap);
  else if (nslots == 4) ss = emit_columns<4>(kvs, scs, s_row, d, cd, ratio, overlap);
  else ss = emit_columns<0>(kvs, scs, s_row, d, cd, ratio, overlap, nslots);
  const float tot = block_sum(ss, s_red);
  const float rms = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(d)), eps)));

  // ---- RMSNorm * gamma
  for (int c = tid; c < d; c += blockDim.x) s_row[c] = __fmul_rn(gamma[c], __fmul_rn(s_row[c], rms));
  __syncthreads();

  // ---- interleaved rotary on the last rope_dim dims, angle row pos + 1 - r
  const int nope = d - rope_dim;
  const float* cr = cos_tab + int64_t(cs_row) * (rope_dim / 2);
  const float* sn = sin_tab + int64_t(cs_row) * (rope_dim / 2);
  for (int k = tid; k < rope_dim / 2; k += blockDim.x) {
    const float a = s_row[nope + 2 * k], bb = s_row[nope + 2 * k + 1];
    const float c = cr[k], s = sn[k];
    const float o0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(bb, s));
    const float o1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(bb, c));
    s_row[nope + 2 * k] = o0;
    s_row[nope + 2 * k + 1] = o1;
  }
  __syncthreads();

  // ---- optional orthonormal Walsh-Hadamard (indexer compressor, rotate=True)
  if (rotate) {
    for (int h = 1; h < d; h <<= 1) {
      for (int j = tid; j < d / 2; j += blockDim.x) {
        const int blk = j / h, off = j - blk * h;
        const int i0 = blk * 2 * h + off, i1 = i0 + h;
        const float a = s_row[i0], bb = s_row[i1];
        s_row[i0] = __fadd_rn(a, bb);
        s_row[i1] = __fsub_rn(a, bb);
      }
      __syncthreads();
    }
    for (int c = tid; c < d; c += blockDim.x) s_row[c] = __fmul_rn(s_row[c], had_scale);
    __syncthreads();
  }

  // ---- compressed row -> kv_cache[b, slot_offset + pos / r]
  __nv_bfloat16* dst = cache + int64_t(b) * cache_bstride + out_row * d;
  for (int c = tid; c < d; c += blockDim.x) dst[c] = f2bf(s_row[c]);

  // ---- slot shift (overlap): rows [0, r) <- rows [r, 2r), staged through
  // registers 8 elements per thread and array at a time so the loads of a
  // batch are all in flight before its stores
  if (overlap) {
    __syncthreads();
    constexpr int kBatch = 8;
    const int n = ratio * cd;
    for (int e0 = 0; e0 < n; e0 += kBatch * kCmpThreads) {
      float a[kBatch], c[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int e = e0 + j * kCmpThreads + tid;
        if (e < n) {
          a[j] = kvs[int64_t(ratio) * cd + e];
          c[j] = scs[int64_t(ratio) * cd + e];
        }
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int e = e0 + j * kCmpThreads + tid;
        if (e < n) {
          kvs[e] = a[j];
          scs[e] = c[j];
        }
      }
    }
  }
}

}  // namespace dsa
