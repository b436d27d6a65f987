// Row-wise stages either side of the path: per-head RMSNorm + interleaved
// rotary (attn.q, the indexer q, the inverse rotary on o), the fused
// kv_norm -> rotary -> act_quant -> window-ring write (the whole Lk-D1 zone
// plus attn.kv_update), and the fold of an additive validity mask into
// -1 index sentinels.
//
// References (zoecarver/tt-deepseek-v4):
//   RMSNorm                    inference.py:436-450 (fp32 math, result in
//                              the input dtype)
//   interleaved rotary         inference.py:4504-4553 (pairs x[2k], x[2k+1]
//                              times cos_k + i sin_k; inverse = conjugate)
//   q path                     inference.py:5982-5993 (rms_norm with weight
//                              softmax_scale per head, then rotary)
//   Lk-D1 + kv_update          inference.py:5997-6006, 6072-6079
//   index/mask split           inference.py:4444-4457
//
// All of these are a few KB per sequence: pure HBM/latency work with no
// reuse, so each row lives in registers (two bf16 per lane) and the only
// cross-lane traffic is the sum of squares.
#include "common.cuh"

namespace dsa {

constexpr int kRowWarps = 8;

// One warp per (b, h) row of Dh elements.  Norm (optional) then rotary
// (optional) on the last rope_dim dims; the normalised value is rounded to
// bf16 before the rotary, as the reference's RMSNorm returns the input dtype.
__global__ void __launch_bounds__(32 * kRowWarps) head_norm_rope_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ld_x, __nv_bfloat16* __restrict__ out, int64_t ld_out, int B,
    int H, int Dh, int rope_dim, const float* __restrict__ gamma, float weight, int do_norm, float eps,
    const float* __restrict__ cos_tab, const float* __restrict__ sin_tab, int n_pos,
    const int32_t* __restrict__ pos, int inverse, int32_t* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  pdl_wait();
  pdl_launch_dependents();
  if (row >= int64_t(B) * H) return;
  const int b = int(row / H), h = int(row - int64_t(b) * H);
  const __nv_bfloat162* src = reinterpret_cast<const __nv_bfloat162*>(x + int64_t(b) * ld_x + int64_t(h) * Dh);
  __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(out + int64_t(b) * ld_out + int64_t(h) * Dh);
  const int npair = Dh >> 1;
  float r = 1.f;
  if (do_norm) {
    float ss = 0.f;
    for (int j = lane; j < npair; j += 32) {
      const float2 v = __bfloat1622float2(src[j]);
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
    }
    ss = warp_sum(ss);
    r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(Dh)), eps)));
  }
  int p = 0;
  const int half = rope_dim >> 1;
  if (rope_dim > 0) {
    p = pos[b];
    if (p < 0 || p >= n_pos) {
      if (lane == 0 && status) atomicOr(status, 1);
      p = p < 0 ? 0 : n_pos - 1;
    }
  }
  const int nope_pairs = npair - half;
  const float* cr = cos_tab + int64_t(p) * half;
  const float* sr = sin_tab + int64_t(p) * half;
  for (int j = lane; j < npair; j += 32) {
    const float2 v = __bfloat1622float2(src[j]);
    float a = v.x, c = v.y;
    if (do_norm) {
      const float w0 = gamma ? gamma[2 * j] : weight, w1 = gamma ? gamma[2 * j + 1] : weight;
      a = bf2f(f2bf(__fmul_rn(w0, __fmul_rn(a, r))));
      c = bf2f(f2bf(__fmul_rn(w1, __fmul_rn(c, r))));
    }
    if (j >= nope_pairs) {
      const int k = j - nope_pairs;
      const float cs = cr[k], sn = inverse ? -sr[k] : sr[k];
      const float o0 = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(c, sn));
      const float o1 = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(c, cs));
      a = o0;
      c = o1;
    }
    dst[j] = __floats2bfloat162_rn(a, c);
  }
}

// One CTA per sequence, one warp per 64-element block of the D-wide row
// (lane owns elements 2*lane, 2*lane+1 of its block).  Blocks below
// D - rope_dim are act_quant'ed, the rest rotated; the finished row goes to
// ring slot pos % win and (optionally) to kv_out.
__global__ void __launch_bounds__(1024) kv_norm_rope_write_kernel(
    const __nv_bfloat16* __restrict__ kv, int64_t ld_kv, const float* __restrict__ gamma, float eps,
    const float* __restrict__ cos_tab, const float* __restrict__ sin_tab, int n_pos,
    const int32_t* __restrict__ pos, __nv_bfloat16* __restrict__ cache, int64_t cache_bstride, int win,
    __nv_bfloat16* __restrict__ kv_out, int64_t ld_out, float* __restrict__ scales, int D, int rope_dim,
    float fp8_max, float inv_max, float q_eps, int32_t* __restrict__ status) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  pdl_wait();
  pdl_launch_dependents();
  const int c0 = warp * 64 + 2 * lane;
  const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(kv + int64_t(b) * ld_kv + c0));
  float ss = fmaf(v.y, v.y, v.x * v.x);
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < nwarps; ++i) tot += red[i];  // same order in every thread
  const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(D)), eps)));
  float a = bf2f(f2bf(__fmul_rn(gamma[c0], __fmul_rn(v.x, r))));
  float c = bf2f(f2bf(__fmul_rn(gamma[c0 + 1], __fmul_rn(v.y, r))));
  const int nope = D - rope_dim;
  int p = pos[b];
  if (p < 0 || p >= n_pos) {
    if (threadIdx.x == 0 && status) atomicOr(status, 1);
    p = p < 0 ? 0 : n_pos - 1;
  }
  if (c0 < nope) {
    // act_quant_block on this 64-wide block (same arithmetic as act_quant.cu)
    float amax = warp_max(fmaxf(fabsf(a), fabsf(c)));
    const float s = __fmul_rn(fmaxf(amax, q_eps), inv_max);
    float y0 = fminf(fmaxf(__fdiv_rn(a, s), -fp8_max), fp8_max);
    float y1 = fminf(fmaxf(__fdiv_rn(c, s), -fp8_max), fp8_max);
    const __nv_fp8_storage_t q0 = __nv_cvt_float_to_fp8(y0, __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8_storage_t q1 = __nv_cvt_float_to_fp8(y1, __NV_SATFINITE, __NV_E4M3);
    a = __half2float(__half(__nv_cvt_fp8_to_halfraw(q0, __NV_E4M3))) * s;
    c = __half2float(__half(__nv_cvt_fp8_to_halfraw(q1, __NV_E4M3))) * s;
    if (scales && lane == 0) scales[int64_t(b) * (nope / 64) + warp] = s;
  } else {
    const int k = (c0 - nope) >> 1;
    const int half = rope_dim >> 1;
    const float cs = cos_tab[int64_t(p) * half + k], sn = sin_tab[int64_t(p) * half + k];
    const float o0 = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(c, sn));
    const float o1 = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(c, cs));
    a = o0;
    c = o1;
  }
  const __nv_bfloat162 o = __floats2bfloat162_rn(a, c);
  const int slot = ((p % win) + win) % win;
  *reinterpret_cast<__nv_bfloat162*>(cache + int64_t(b) * cache_bstride + int64_t(slot) * D + c0) = o;
  if (kv_out) *reinterpret_cast<__nv_bfloat162*>(kv_out + int64_t(b) * ld_out + c0) = o;
}

// out[i] = valid[i] is -inf (or any negative) ? -1 : idx[i]
__global__ void fold_index_mask_kernel(const int32_t* __restrict__ idx, const __nv_bfloat16* __restrict__ valid,
                                       int32_t* __restrict__ out, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    out[i] = bf2f(valid[i]) < 0.f ? -1 : idx[i];
}

}  // namespace dsa

using namespace dsa;

extern "C" int dsa_head_norm_rope(const void* x, int64_t ld_x, void* out, int64_t ld_out, int B, int H, int Dh,
                                  int rope_dim, const float* gamma, float weight, int do_norm, float eps,
                                  const float* cos_tab, const float* sin_tab, int n_pos, const int32_t* pos,
                                  int inverse, int32_t* status, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(x && out, "head_norm_rope: null x/out");
  DSA_CHECK_ARG(B >= 0 && H > 0 && Dh > 0 && Dh % 2 == 0, "head_norm_rope: bad B/H/Dh");
  DSA_CHECK_ARG(rope_dim >= 0 && rope_dim <= Dh && rope_dim % 2 == 0, "head_norm_rope: bad rope_dim %d", rope_dim);
  DSA_CHECK_ARG(ld_x >= int64_t(H) * Dh && ld_out >= int64_t(H) * Dh && ld_x % 2 == 0 && ld_out % 2 == 0,
                "head_norm_rope: row strides must cover H*Dh and be even");
  DSA_CHECK_ARG(aligned(x, 4) && aligned(out, 4), "head_norm_rope: x/out must be 4-byte aligned");
  DSA_CHECK_ARG(rope_dim == 0 || (cos_tab && sin_tab && pos && n_pos > 0),
                "head_norm_rope: rotary needs cos/sin tables and device positions");
  DSA_CHECK_ARG(!do_norm || eps > 0.f, "head_norm_rope: eps must be positive");
  if (B == 0) return DSA_OK;
  const int64_t rows = int64_t(B) * H;
  const int grid = int((rows + kRowWarps - 1) / kRowWarps);
  launch_pdl(head_norm_rope_kernel, dim3(grid), dim3(32 * kRowWarps), 0, reinterpret_cast<cudaStream_t>(stream),
             static_cast<const __nv_bfloat16*>(x), ld_x, static_cast<__nv_bfloat16*>(out), ld_out, B, H, Dh, rope_dim,
             gamma, weight, do_norm ? 1 : 0, eps, cos_tab, sin_tab, n_pos, pos, inverse ? 1 : 0, status);
  DSA_CHECK_LAUNCH("head_norm_rope");
  return DSA_OK;
}

extern "C" int dsa_kv_norm_rope_window_write(const void* kv, int64_t ld_kv, const float* gamma, float eps,
                                             const float* cos_tab, const float* sin_tab, int n_pos,
                                             const int32_t* pos, void* kv_cache, int64_t cache_bstride, int win,
                                             void* kv_out, int64_t ld_out, float* scales, int B, int D,
                                             int rope_dim, int32_t* status, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(kv && gamma && cos_tab && sin_tab && pos && kv_cache, "kv_norm_rope_window_write: null pointer");
  DSA_CHECK_ARG(B >= 0 && D > 0 && D % 64 == 0 && D / 64 <= 32,
                "kv_norm_rope_window_write: D=%d must be a multiple of 64 and <= 2048", D);
  DSA_CHECK_ARG(rope_dim >= 0 && rope_dim < D && rope_dim % 64 == 0,
                "kv_norm_rope_window_write: rope_dim %d must be a multiple of 64 below D", rope_dim);
  DSA_CHECK_ARG(n_pos > 0 && win > 0 && cache_bstride >= int64_t(win) * D, "kv_norm_rope_window_write: bad win/table");
  DSA_CHECK_ARG(ld_kv >= D && ld_kv % 2 == 0 && aligned(kv, 4) && aligned(kv_cache, 4) && cache_bstride % 2 == 0,
                "kv_norm_rope_window_write: kv/kv_cache must be 4-byte aligned with even strides");
  DSA_CHECK_ARG(!kv_out || (ld_out >= D && ld_out % 2 == 0 && aligned(kv_out, 4)),
                "kv_norm_rope_window_write: bad kv_out");
  DSA_CHECK_ARG(eps > 0.f, "kv_norm_rope_window_write: eps must be positive");
  if (B == 0) return DSA_OK;
  launch_pdl(kv_norm_rope_write_kernel, dim3(B), dim3((D / 64) * 32), 0, reinterpret_cast<cudaStream_t>(stream),
             static_cast<const __nv_bfloat16*>(kv), ld_kv, gamma, eps, cos_tab, sin_tab, n_pos, pos,
             static_cast<__nv_bfloat16*>(kv_cache), cache_bstride, win, static_cast<__nv_bfloat16*>(kv_out), ld_out,
             scales, D, rope_dim, 448.f, float(1.0 / 448.0), 1e-4f, status);
  DSA_CHECK_LAUNCH("kv_norm_rope_window_write");
  return DSA_OK;
}

extern "C" int dsa_fold_index_mask(const int32_t* idx, const void* valid, int64_t n, int32_t* out,
                                   dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(idx && valid && out && n >= 0, "fold_index_mask: bad arguments");
  if (n == 0) return DSA_OK;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, int64_t(num_sms()) * 8);
  fold_index_mask_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      idx, static_cast<const __nv_bfloat16*>(valid), out, n);
  DSA_CHECK_LAUNCH("fold_index_mask");
  return DSA_OK;
}
