// attn.kv: block-wise FP8-E4M3 act_quant round trip, standalone and fused
// with the window-ring KV write.
//
// Semantics (reference inference.py:4578-4607 plus the e4m3 cast):
//   amax = max|x| over a block;  s = max(amax, eps) * (1 / fp8_max)
//        (the chain's multiply by the fp32 constant 1/fp8_max, 4602)
//   q = e4m3_rn_satfinite(clamp(x / s, +-fp8_max))            (IEEE div)
//   out = bf16_rn(float(q) * s)
// One warp owns one (row, block) pair; each lane holds block/32 contiguous
// elements in registers, so the max-abs is a 5-step shuffle reduction and
// nothing touches shared memory.  The op is a pure HBM stream (2 B in,
// 2 B out, 4 B per block of scale), so the grid is a grid-stride loop sized
// to the SM count.
#include "common.cuh"
#include "act_quant_dev.cuh"

namespace dsa {

template <int EPL>
__global__ void __launch_bounds__(256) act_quant_kernel(const __nv_bfloat16* __restrict__ x,
                                                        __nv_bfloat16* __restrict__ out,
                                                        float* __restrict__ scales,
                                                        uint8_t* __restrict__ codes, int64_t M,
                                                        int64_t N, int64_t ldx, int64_t ldo,
                                                        float fp8_max, float inv_max, float eps) {
  constexpr int BLOCK = EPL * 32;
  const int64_t nb = N / BLOCK;
  const int64_t total = M * nb;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t w = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total; w += nwarps) {
    const int64_t r = w / nb;
    const int64_t c0 = (w - r * nb) * BLOCK;
    quant_block_lane<EPL>(x + r * ldx + c0, out + r * ldo + c0, scales ? scales + w : nullptr,
                          codes ? codes + r * N + c0 : nullptr, lane, fp8_max, inv_max, eps);
  }
}

// One CTA per sequence (kv_window_write_row).
__global__ void __launch_bounds__(256) kv_window_write_kernel(
    const __nv_bfloat16* __restrict__ kv, __nv_bfloat16* __restrict__ cache,
    float* __restrict__ scales, const int32_t* __restrict__ pos, int D, int rope_dim,
    int64_t cache_bstride, int win, float fp8_max, float inv_max, float eps) {
  pdl_wait();
  pdl_launch_dependents();
  kv_window_write_row(kv, cache, scales, pos, D, rope_dim, cache_bstride, win, fp8_max, inv_max, eps, blockIdx.x);
}

}  // namespace dsa

using namespace dsa;

extern "C" int dsa_act_quant_block(const void* x, void* out, float* scales, uint8_t* codes, int64_t M,
                                   int64_t N, int64_t ld_x, int64_t ld_out, int block, float fp8_max,
                                   float eps, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(x && out, "act_quant_block: null x/out");
  DSA_CHECK_ARG(M >= 0 && N > 0 && ld_x >= N && ld_out >= N, "act_quant_block: bad M/N/ld");
  DSA_CHECK_ARG(block == 32 || block == 64 || block == 128 || block == 256,
                "act_quant_block: block must be 32, 64, 128 or 256 (got %d)", block);
  DSA_CHECK_ARG(N % block == 0, "act_quant_block: N=%lld not divisible by block=%d", (long long)N, block);
  DSA_CHECK_ARG(fp8_max > 0.f && eps > 0.f, "act_quant_block: fp8_max and eps must be positive");
  if (M == 0) return DSA_OK;
  // 1 / fp8_max rounded once to fp32, as the reference's Python constant is
  const float inv_max = float(1.0 / double(fp8_max));
  const int64_t total = M * (N / block);
  int grid = (int)std::min<int64_t>((total + 7) / 8, int64_t(num_sms()) * 16);
  auto* xp = static_cast<const __nv_bfloat16*>(x);
  auto* op = static_cast<__nv_bfloat16*>(out);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (block == 64) {
    DSA_CHECK_ARG(aligned(x, 4) && aligned(out, 4) && ld_x % 2 == 0 && ld_out % 2 == 0,
                  "act_quant_block: x/out must be 4-byte aligned with even strides");
    act_quant_kernel<2><<<grid, 256, 0, st>>>(xp, op, scales, codes, M, N, ld_x, ld_out, fp8_max, inv_max, eps);
  } else if (block == 32) {
    act_quant_kernel<1><<<grid, 256, 0, st>>>(xp, op, scales, codes, M, N, ld_x, ld_out, fp8_max, inv_max, eps);
  } else if (block == 128) {
    act_quant_kernel<4><<<grid, 256, 0, st>>>(xp, op, scales, codes, M, N, ld_x, ld_out, fp8_max, inv_max, eps);
  } else {
    act_quant_kernel<8><<<grid, 256, 0, st>>>(xp, op, scales, codes, M, N, ld_x, ld_out, fp8_max, inv_max, eps);
  }
  DSA_CHECK_LAUNCH("act_quant_block");
  return DSA_OK;
}

extern "C" int dsa_kv_window_write(const void* kv, void* kv_cache, float* scales, const int32_t* pos, int B,
                                   int D, int rope_dim, int64_t cache_bstride, int win, int block,
                                   dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(kv && kv_cache && pos, "kv_window_write: null pointer");
  DSA_CHECK_ARG(B >= 0 && D > 0 && rope_dim >= 0 && rope_dim < D, "kv_window_write: bad B/D/rope_dim");
  DSA_CHECK_ARG(block == 64, "kv_window_write: only block=64 is built (got %d)", block);
  DSA_CHECK_ARG((D - rope_dim) % 64 == 0, "kv_window_write: nope dims %d not divisible by 64", D - rope_dim);
  DSA_CHECK_ARG(win > 0 && cache_bstride >= int64_t(win) * D, "kv_window_write: bad win/cache stride");
  DSA_CHECK_ARG(aligned(kv, 4) && aligned(kv_cache, 4) && D % 2 == 0 && cache_bstride % 2 == 0,
                "kv_window_write: kv/kv_cache must be 4-byte aligned");
  if (B == 0) return DSA_OK;
  launch_pdl(kv_window_write_kernel, dim3(B), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
             static_cast<const __nv_bfloat16*>(kv), static_cast<__nv_bfloat16*>(kv_cache), scales, pos, D, rope_dim,
             cache_bstride, win, 448.f, float(1.0 / 448.0), 1e-4f);
  DSA_CHECK_LAUNCH("kv_window_write");
  return DSA_OK;
}
