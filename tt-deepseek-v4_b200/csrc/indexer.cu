// attn.topk (indexer score): s[b, t] = sum_h w[b, h] * relu(q[b, h, :] . k[b, t, :])
//
// Reference: DeviceIndexer.forward_device_score score stage
// (inference.py:5260-5275: q @ kv_cache^T, relu * w, sum over heads) and the
// fused tt-lang version test_lk_d_idx_score.py:142-289.
//
// Two tcgen05 kernels: indexer_tc.cuh for per-sequence keys (decode: one q
// of 64 heads per sequence, N = 64) and indexer_prefill_tc.cuh for one key
// cache shared by all rows (a prefill chunk: 4 tokens per MMA batch,
// N = 256).  Keys are the M dimension (S^T = K . Q^T) so one accumulator row
// holds all heads of one key and the relu * w head reduction stays in the
// epilogue's registers; the [H, T] score matrix is never materialised.
#include "common.cuh"
#include "indexer_tc.cuh"
#include "indexer_prefill_tc.cuh"
#include "indexer_row.cuh"

namespace dsa {

constexpr int kIdxH = 64;        // indexer heads
constexpr int kIdxD = 128;       // indexer head dim

// The score of each sequence's newest live key row, t = min(t_active[b], T)
// - 1, written into score[b, t].  A decode step scores the rows before it
// with the tensor-core kernel while the indexer compressor may still be
// writing that row; this kernel follows the compressor on its stream, so
// the top-k finds every live score in place.  indexer_row_score is the
// top-k's own recompute of the same row (dsa_indexer_topk_newest): the
// value is bit-identical to it.  One CTA of 8 warps per sequence.
__global__ void __launch_bounds__(256) indexer_score_newest_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, int64_t k_bstride,
    const float* __restrict__ w, const int32_t* __restrict__ t_active, float* __restrict__ score, int64_t ld_score,
    int T) {
  __shared__ float s_dot[kRowHeads];
  pdl_wait();
  pdl_launch_dependents();
  score_newest_row(q, k, k_bstride, w, t_active, score, ld_score, T, blockIdx.x, s_dot);
}

}  // namespace dsa

using namespace dsa;

static int indexer_score_run(const void* q, const void* k, const float* w, float* score, const int32_t* t_valid,
                             int B, int H, int Di, int T, int64_t k_bstride, int64_t ld_score, int flags,
                             dsa_stream_t stream, uint32_t* dyn = nullptr) {
  DSA_CHECK_ARG(q && k && w && score, "indexer_score: null pointer");
  DSA_CHECK_ARG(H == kIdxH && Di == kIdxD, "indexer_score: built for H=64, Di=128 (got H=%d Di=%d)", H, Di);
  DSA_CHECK_ARG(B >= 0 && T >= 0, "indexer_score: bad B/T");
  DSA_CHECK_ARG((k_bstride == 0 || k_bstride >= int64_t(T) * Di) && k_bstride % 8 == 0,
                "indexer_score: bad k batch stride (0 = one key cache shared by all rows)");
  DSA_CHECK_ARG(ld_score >= T, "indexer_score: ld_score < T");
  DSA_CHECK_ARG(aligned(q, 16) && aligned(k, 16), "indexer_score: q/k must be 16-byte aligned");
  if (B == 0 || T == 0) return DSA_OK;
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    cudaFuncSetAttribute(idxtc::indexer_score_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         idxtc::kSmemBytes);
    cudaFuncSetAttribute(idxtc::indexer_score_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         idxtc::kSmemBytes);
    attr_dev = dev;
  }
  const int nsm = num_sms();
  DSA_CHECK_ARG(!dyn || (k_bstride != 0 && B <= idxtc::kMaxSeqBalanced && aligned(dyn, 8)),
                "indexer_score: the dynamic split needs per-sequence keys, B <= %d and 8-byte aligned counters",
                idxtc::kMaxSeqBalanced);
  if (k_bstride == 0 && B % idxpf::QG == 0) {
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
    a.wait_limit = wait_limit_cycles();
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
    a.wait_limit = wait_limit_cycles();
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
    a.balanced = B <= idxtc::kMaxSeqBalanced ? 1 : 0;
    a.keys_ready = (flags & DSA_KEYS_READY) ? 1 : 0;
    const int grid = a.balanced ? std::min(nsm, total) : (total + a.items_per_cta - 1) / a.items_per_cta;
    a.dyn = dyn;
    if (dyn)
      launch_pdl(idxtc::indexer_score_tc_kernel<true>, dim3(grid), dim3(idxtc::THREADS), idxtc::kSmemBytes,
                 reinterpret_cast<cudaStream_t>(stream), a, tm_k, tm_q);
    else
      launch_pdl(idxtc::indexer_score_tc_kernel<false>, dim3(grid), dim3(idxtc::THREADS), idxtc::kSmemBytes,
                 reinterpret_cast<cudaStream_t>(stream), a, tm_k, tm_q);
  }
  DSA_CHECK_LAUNCH("indexer_score");
  return DSA_OK;
}

extern "C" int dsa_indexer_score(const void* q, const void* k, const float* w, float* score, const int32_t* t_valid,
                                 int B, int H, int Di, int T, int64_t k_bstride, int64_t ld_score,
                                 dsa_stream_t stream) {
  clear_error();
  return indexer_score_run(q, k, w, score, t_valid, B, H, Di, T, k_bstride, ld_score, 0, stream);
}

extern "C" int dsa_indexer_score_ex(const void* q, const void* k, const float* w, float* score,
                                    const int32_t* t_valid, int B, int H, int Di, int T, int64_t k_bstride,
                                    int64_t ld_score, int flags, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG((flags & ~DSA_KEYS_READY) == 0, "indexer_score: unknown flags 0x%x", flags);
  return indexer_score_run(q, k, w, score, t_valid, B, H, Di, T, k_bstride, ld_score, flags, stream);
}

extern "C" int dsa_indexer_score_newest(const void* q, const void* k, int64_t k_bstride, const float* w,
                                        const int32_t* t_active, float* score, int64_t ld_score, int B, int T,
                                        dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(q && k && w && t_active && score, "indexer_score_newest: null pointer");
  DSA_CHECK_ARG(B >= 0 && T > 0 && ld_score >= T && k_bstride >= int64_t(T) * kIdxD,
                "indexer_score_newest: need T > 0, ld_score >= T, k_bstride >= T * 128");
  DSA_CHECK_ARG(aligned(q, 8) && aligned(k, 8) && k_bstride % 4 == 0,
                "indexer_score_newest: q, k and the key row stride must be 8-byte aligned");
  if (B == 0) return DSA_OK;
  launch_pdl(indexer_score_newest_kernel, dim3(B), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
             static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), k_bstride, w, t_active,
             score, ld_score, T);
  DSA_CHECK_LAUNCH("indexer_score_newest");
  return DSA_OK;
}

extern "C" int dsa_indexer_score_dyn(const void* q, const void* k, const float* w, float* score,
                                     const int32_t* t_valid, int B, int H, int Di, int T, int64_t k_bstride,
                                     int64_t ld_score, int flags, uint32_t* counters, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG((flags & ~DSA_KEYS_READY) == 0, "indexer_score: unknown flags 0x%x", flags);
  DSA_CHECK_ARG(counters != nullptr, "indexer_score: null counters");
  return indexer_score_run(q, k, w, score, t_valid, B, H, Di, T, k_bstride, ld_score, flags, stream, counters);
}
