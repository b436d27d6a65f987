// attn.compress: compressor state write + emit + slot shift in one kernel.
//
// Reference: DeviceCompressor.forward_device / _emit_body
// (inference.py:4938-5097), the fused softmax-sum-norm tt-lang kernel
// (3205-3364) and the in-place fanout slot shift (3101-3186).
//
// One CTA per sequence.  The emit decision ((pos + 1) % r == 0) is taken on
// the device from the per-sequence position, so one launch (and one CUDA
// graph) serves emit and non-emit steps alike - the reference needs two
// captured traces for that.  State is fp32 ([B, coff*r, coff*d], the CPU
// layout of inference.py:538-551) so the softmax/weighted sum is fp32 end to
// end; the emitted row is rounded to bf16 once.  The work is tiny (<= 32 KB
// of state per sequence), so the kernel is latency-bound by design; its job
// is to remove the reference's 16-24 dispatches per step.
#include "common.cuh"
#include "compressor_dev.cuh"

namespace dsa {

__global__ void __launch_bounds__(kCmpThreads) compressor_step_kernel(const CmpStep a) {
  __shared__ float s_row[kCmpMaxD];
  __shared__ float s_red[32];
  pdl_wait();
  pdl_launch_dependents();
  compressor_step_row(a, blockIdx.x, s_row, s_red);
}

}  // namespace dsa

using namespace dsa;

extern "C" int dsa_compressor_step(const void* kv_row, const void* score_row, int64_t ld_row, const float* ape,
                                   float* kv_state, float* score_state, const float* gamma,
                                   const float* cos_tab, const float* sin_tab, int n_pos, void* kv_cache,
                                   int64_t cache_bstride, int64_t cache_rows, int slot_offset,
                                   const int32_t* pos, int32_t* emitted, int B, int d, int rope_dim, int ratio,
                                   int overlap, int rotate, int write_state, float eps, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG((!write_state || (kv_row && score_row && ape)) && kv_state && score_state && gamma && cos_tab && sin_tab &&
                    kv_cache && pos,
                "compressor_step: null pointer");
  DSA_CHECK_ARG(B >= 0 && d > 0 && d <= kCmpMaxD && d % 2 == 0, "compressor_step: d=%d must be even and <= %d", d,
                kCmpMaxD);
  DSA_CHECK_ARG(rope_dim >= 0 && rope_dim <= d && rope_dim % 2 == 0, "compressor_step: bad rope_dim %d", rope_dim);
  DSA_CHECK_ARG(ratio > 0, "compressor_step: ratio must be positive");
  DSA_CHECK_ARG(!write_state || ld_row >= (overlap ? 2 : 1) * d, "compressor_step: ld_row too small");
  DSA_CHECK_ARG(cache_rows > 0 && cache_bstride >= cache_rows * d, "compressor_step: bad cache shape");
  DSA_CHECK_ARG(n_pos > 0, "compressor_step: empty rotary table");
  DSA_CHECK_ARG(!rotate || (d & (d - 1)) == 0, "compressor_step: Hadamard needs power-of-two d (got %d)", d);
  if (B == 0) return DSA_OK;
  const float had_scale = (float)(1.0 / sqrt((double)d));
  const CmpStep a{static_cast<const __nv_bfloat16*>(kv_row), static_cast<const __nv_bfloat16*>(score_row), ld_row,
                  ape, kv_state, score_state, gamma, cos_tab, sin_tab, n_pos, static_cast<__nv_bfloat16*>(kv_cache),
                  cache_bstride, cache_rows, slot_offset, pos, emitted, d, rope_dim, ratio, overlap ? 1 : 0,
                  rotate ? 1 : 0, write_state ? 1 : 0, had_scale, eps};
  launch_pdl(compressor_step_kernel, dim3(B), dim3(kCmpThreads), 0, reinterpret_cast<cudaStream_t>(stream), a);
  DSA_CHECK_LAUNCH("compressor_step");
  return DSA_OK;
}
