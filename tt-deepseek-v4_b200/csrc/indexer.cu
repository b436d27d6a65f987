// attn.topk (indexer score): s[b, t] = sum_h w[b, h] * relu(q[b, h, :] . k[b, t, :])
//
// Reference: DeviceIndexer.forward_device_score score stage
// (inference.py:5260-5275: q @ kv_cache^T, relu * w, sum over heads) and the
// fused tt-lang version test_lk_d_idx_score.py:142-289.
//
// Layout / mapping.  Keys are the M dimension of the contraction
// (S^T = K . Q^T, M = keys, N = 64 heads, K = 128 dims) so that one row of the
// accumulator holds all 64 heads of one key and the relu * w head reduction is
// a register-local sum plus a 2-step quad shuffle - the [H, T] score matrix
// is never materialised.  Keys stream through a 4-stage cp.async ring of
// 64-key tiles (16 KB each, 16-byte XOR-swizzled rows so ldmatrix is
// conflict-free); q (16 KB) stays resident in shared memory.  The kernel is
// HBM-bound on the key stream: 256 B per key in, 4 B per key out.
#include "common.cuh"
#include "indexer_tc.cuh"
#include "indexer_prefill_tc.cuh"
#include <stdlib.h>

namespace dsa {

constexpr int kIdxH = 64;        // indexer heads
constexpr int kIdxD = 128;       // indexer head dim
constexpr int kIdxTile = 64;     // keys per pipeline stage
constexpr int kIdxStages = 4;
constexpr int kIdxThreads = 128; // 4 warps x 16 keys
constexpr int kIdxRowBytes = kIdxD * 2;  // 256 B per key / per head row

// byte offset of 16-byte chunk `c` (0..15) of row `r` in a swizzled [rows][256 B] tile
__device__ __forceinline__ uint32_t idx_swz(int r, int c) { return r * kIdxRowBytes + ((c ^ (r & 7)) << 4); }

__global__ void __launch_bounds__(kIdxThreads) indexer_score_mma_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const float* __restrict__ w,
    float* __restrict__ score, const int32_t* __restrict__ t_valid, int T, int64_t k_bstride, int64_t ld_score,
    int keys_per_cta) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;                                 // [64][256 B]
  uint8_t* sK = smem + kIdxH * kIdxRowBytes;          // [stages][64][256 B]
  const int b = blockIdx.y;
  const int t_begin = blockIdx.x * keys_per_cta;
  const int t_lim = t_valid ? min(T, max(0, t_valid[blockIdx.y])) : T;
  const int t_end = min(t_lim, t_begin + keys_per_cta);
  if (t_begin >= t_end) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16* qb = q + int64_t(b) * kIdxH * kIdxD;
  const __nv_bfloat16* kb = k + int64_t(b) * k_bstride;

  // q -> smem (16 KB = 1024 chunks, 8 per thread)
  for (int e = tid; e < kIdxH * 16; e += kIdxThreads) {
    const int r = e >> 4, c = e & 15;
    cp_async16(smem_u32(sQ + idx_swz(r, c)), qb + r * kIdxD + c * 8, 16);
  }
  const int ntiles = (t_end - t_begin + kIdxTile - 1) / kIdxTile;
  auto load_tile = [&](int tile, int stage) {
    const int t0 = t_begin + tile * kIdxTile;
    uint8_t* dst = sK + stage * (kIdxTile * kIdxRowBytes);
    for (int e = tid; e < kIdxTile * 16; e += kIdxThreads) {
      const int r = e >> 4, c = e & 15;
      const int t = t0 + r;
      const bool ok = t < t_end;
      cp_async16(smem_u32(dst + idx_swz(r, c)), kb + int64_t(ok ? t : t_begin) * kIdxD + c * 8, ok ? 16 : 0);
    }
  };
#pragma unroll
  for (int s = 0; s < kIdxStages - 1; ++s) {
    if (s < ntiles) load_tile(s, s);
    cp_async_commit();
  }

  // per-thread head weights for accumulator columns 8n + 2(lane%4) + {0,1}
  float wr[16];
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    wr[2 * n] = w[b * kIdxH + 8 * n + 2 * (lane & 3)];
    wr[2 * n + 1] = w[b * kIdxH + 8 * n + 2 * (lane & 3) + 1];
  }

  for (int tile = 0; tile < ntiles; ++tile) {
    const int pf = tile + kIdxStages - 1;
    if (pf < ntiles) load_tile(pf, pf % kIdxStages);
    cp_async_commit();
    cp_async_wait<kIdxStages - 1>();
    __syncthreads();
    const uint8_t* tK = sK + (tile % kIdxStages) * (kIdxTile * kIdxRowBytes);
    float acc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kIdxD / 16; ++ks) {
      uint32_t a[4];
      {
        const int r = warp * 16 + (lane & 15);
        const int c = 2 * ks + (lane >> 4);
        ldmatrix_x4(smem_u32(tK + idx_swz(r, c)), a[0], a[1], a[2], a[3]);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r0, r1, r2, r3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = 2 * ks + ((lane >> 3) & 1);
        ldmatrix_x4(smem_u32(sQ + idx_swz(r, c)), r0, r1, r2, r3);
        const uint32_t b0[2] = {r0, r1}, b1[2] = {r2, r3};
        mma_bf16_16816(acc[2 * np], a, b0);
        mma_bf16_16816(acc[2 * np + 1], a, b1);
      }
    }
    // epilogue: rows g = lane/4 and g+8 of this warp's 16 keys
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      s0 = fmaf(wr[2 * n], fmaxf(acc[n][0], 0.f), s0);
      s0 = fmaf(wr[2 * n + 1], fmaxf(acc[n][1], 0.f), s0);
      s1 = fmaf(wr[2 * n], fmaxf(acc[n][2], 0.f), s1);
      s1 = fmaf(wr[2 * n + 1], fmaxf(acc[n][3], 0.f), s1);
    }
    s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
    if ((lane & 3) == 0) {
      const int t0 = t_begin + tile * kIdxTile + warp * 16 + (lane >> 2);
      float* srow = score + int64_t(b) * ld_score;
      if (t0 < t_end) srow[t0] = s0;
      if (t0 + 8 < t_end) srow[t0 + 8] = s1;
    }
    __syncthreads();
  }
  cp_async_wait<0>();
}

}  // namespace dsa

using namespace dsa;

extern "C" int dsa_indexer_score(const void* q, const void* k, const float* w, float* score, const int32_t* t_valid,
                                 int B, int H, int Di, int T, int64_t k_bstride, int64_t ld_score,
                                 dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(q && k && w && score, "indexer_score: null pointer");
  DSA_CHECK_ARG(H == kIdxH && Di == kIdxD, "indexer_score: built for H=64, Di=128 (got H=%d Di=%d)", H, Di);
  DSA_CHECK_ARG(B >= 0 && T >= 0, "indexer_score: bad B/T");
  DSA_CHECK_ARG((k_bstride == 0 || k_bstride >= int64_t(T) * Di) && k_bstride % 8 == 0,
                "indexer_score: bad k batch stride (0 = one key cache shared by all rows)");
  DSA_CHECK_ARG(ld_score >= T, "indexer_score: ld_score < T");
  DSA_CHECK_ARG(aligned(q, 16) && aligned(k, 16), "indexer_score: q/k must be 16-byte aligned");
  if (B == 0 || T == 0) return DSA_OK;
  static int use_mma = -1;
  if (use_mma < 0) {
    const char* e = getenv("DSV4_INDEXER_MMA");
    use_mma = (e && e[0] == '1') ? 1 : 0;
  }
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = kIdxH * kIdxRowBytes + kIdxStages * kIdxTile * kIdxRowBytes;
  if (attr_dev != dev) {
    cudaFuncSetAttribute(indexer_score_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(idxtc::indexer_score_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         idxtc::kSmemBytes);
    attr_dev = dev;
  }
  const int nsm = num_sms();
  if (use_mma) {
    // enough CTAs to cover the SMs ~2x; each CTA streams a contiguous key range
    int per = (int)((int64_t(T) * B + 2LL * nsm - 1) / (2LL * nsm));
    per = std::max(kIdxTile * 2, ((per + kIdxTile - 1) / kIdxTile) * kIdxTile);
    dim3 grid((T + per - 1) / per, B);
    indexer_score_mma_kernel<<<grid, kIdxThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), w, score, t_valid, T, k_bstride,
        ld_score, per);
  } else if (k_bstride == 0 && B % idxpf::QG == 0) {
    // one key cache shared by all rows (a prefill chunk): 4 rows per MMA batch
    static int pf_attr_dev = -1;
    if (pf_attr_dev != dev) {
      cudaFuncSetAttribute(idxpf::indexer_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           idxpf::kSmemBytes);
      pf_attr_dev = dev;
    }
    DSA_CHECK_ARG(uint64_t(B) * kIdxH < (1ull << 31), "indexer_score: too many rows");
    CUtensorMap tm_k, tm_q;
    if (!tma::make_2d_bf16(&tm_k, k, kIdxD, uint64_t(T), kIdxD * 2, 64, idxpf::TILE) ||
        !tma::make_2d_bf16(&tm_q, q, kIdxD, uint64_t(B) * kIdxH, kIdxD * 2, 64, idxpf::N)) {
      set_error("indexer_score: cuTensorMapEncodeTiled failed");
      return DSA_ERR_CUDA;
    }
    idxpf::Args a{};
    a.w = w;
    a.score = score;
    a.t_valid = t_valid;
    a.status = nullptr;
    a.S = B;
    a.T = T;
    a.tiles = (T + idxpf::TILE - 1) / idxpf::TILE;
    const int total = (B / idxpf::QG) * a.tiles;
    a.items_per_cta = (total + nsm - 1) / nsm;
    a.ld_score = ld_score;
    const int grid = (total + a.items_per_cta - 1) / a.items_per_cta;
    idxpf::indexer_prefill_tc_kernel<<<grid, idxpf::THREADS, idxpf::kSmemBytes,
                                       reinterpret_cast<cudaStream_t>(stream)>>>(a, tm_k, tm_q);
  } else {
    DSA_CHECK_ARG(k_bstride % kIdxD == 0, "indexer_score: k batch stride must be a multiple of Di");
    const int64_t row_stride = k_bstride / kIdxD;
    const uint64_t k_rows = uint64_t(B - 1) * row_stride + uint64_t(T);
    DSA_CHECK_ARG(k_rows < (1ull << 31), "indexer_score: key cache has more than 2^31 rows");
    CUtensorMap tm_k, tm_q;
    if (!tma::make_2d_bf16(&tm_k, k, kIdxD, k_rows, kIdxD * 2, 64, idxtc::TILE) ||
        !tma::make_2d_bf16(&tm_q, q, kIdxD, uint64_t(B) * kIdxH, kIdxD * 2, 64, kIdxH)) {
      set_error("indexer_score: cuTensorMapEncodeTiled failed");
      return DSA_ERR_CUDA;
    }
    idxtc::Args a{};
    a.w = w;
    a.score = score;
    a.t_valid = t_valid;
    a.status = nullptr;
    a.B = B;
    a.T = T;
    a.tiles_per_seq = (T + idxtc::TILE - 1) / idxtc::TILE;
    const int total = B * a.tiles_per_seq;
    a.items_per_cta = (total + nsm - 1) / nsm;
    a.ld_score = ld_score;
    a.k_row_stride = row_stride;
    const int grid = (total + a.items_per_cta - 1) / a.items_per_cta;
    launch_pdl(idxtc::indexer_score_tc_kernel, dim3(grid), dim3(idxtc::THREADS), idxtc::kSmemBytes,
               reinterpret_cast<cudaStream_t>(stream), a, tm_k, tm_q);
  }
  DSA_CHECK_LAUNCH("indexer_score");
  return DSA_OK;
}
