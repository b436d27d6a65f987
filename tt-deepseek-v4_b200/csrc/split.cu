// Index bookkeeping of the sequence split (one long context, compressed KV
// and indexer keys cut into contiguous shards, one shard per GPU).
//
// The split itself is planned in the reference's briefs
// (briefs/future_max_utilization.md:177-204) and is not implemented there;
// on one GPU it reduces to the unsplit path (inference.py:5823-5851 top-k,
// 4459-4501 attention).  These kernels only move int32 indices: a few KB per
// step, one launch each.
#include "common.cuh"

namespace dsa {

// t_local[b] = clamp(t_active[b] - lo, 0, n_local)
__global__ void shard_active_kernel(const int32_t* __restrict__ t_active, int32_t* __restrict__ t_local, int B,
                                    int lo, int n_local) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) t_local[b] = min(max(t_active[b] - lo, 0), n_local);
}

// One CTA per sequence.  out[b, j < W] = window slot + win_base (or -1 when
// this shard does not attend the window); out[b, W + j] = sel - lo +
// local_base for selected positions in [lo, hi), else -1.
__global__ void shard_local_indices_kernel(const int32_t* __restrict__ sel, int64_t ld_sel, int k,
                                           const int32_t* __restrict__ win_idx, int64_t ld_win, int W, int lo,
                                           int hi, int local_base, int win_base, int32_t* __restrict__ out,
                                           int64_t ld_out) {
  const int b = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  const int32_t* s = sel + int64_t(b) * ld_sel;
  int32_t* o = out + int64_t(b) * ld_out;
  for (int j = threadIdx.x; j < W; j += blockDim.x) {
    const int w = win_idx ? win_idx[int64_t(b) * ld_win + j] : -1;
    o[j] = w >= 0 ? w + win_base : -1;
  }
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const int p = s[j];
    o[W + j] = (p >= lo && p < hi) ? p - lo + local_base : -1;
  }
}

// Prefill chunk of S tokens at positions base .. base + S - 1: per query s
// the compressed entries it may see, t_active[s] = min(T, (p + 1) / ratio)
// (entry j holds tokens 4j .. 4j + 3, visible once all are <= p), and its
// causal window of W raw rows: the raw buffer holds the n_hist tokens before
// the chunk then the chunk, so position p - W + 1 + i sits in row
// s + i + n_hist - (W - 1) (-1 before the first held token).
__global__ void prefill_positions_kernel(int S, int base, int ratio, int T, int W, int n_hist,
                                         int32_t* __restrict__ t_active, int32_t* __restrict__ idx, int64_t ld_idx) {
  const int s = blockIdx.x;
  if (threadIdx.x == 0) t_active[s] = min(T, (base + s + 1) / ratio);
  for (int i = threadIdx.x; i < W; i += blockDim.x) {
    const int row = s + i + n_hist - (W - 1);
    idx[int64_t(s) * ld_idx + i] = row >= 0 ? row : -1;
  }
}

}  // namespace dsa

using namespace dsa;

extern "C" int dsa_prefill_positions(int S, int base, int ratio, int T, int W, int n_hist, int32_t* t_active,
                                     int32_t* idx, int64_t ld_idx, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(t_active && idx && S >= 0 && base >= 0 && ratio > 0 && T >= 0 && W > 0 && ld_idx >= W,
                "prefill_positions: bad arguments");
  DSA_CHECK_ARG(n_hist >= 0 && n_hist <= base, "prefill_positions: n_hist %d must be in [0, base]", n_hist);
  if (S == 0) return DSA_OK;
  prefill_positions_kernel<<<S, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(S, base, ratio, T, W, n_hist,
                                                                                 t_active, idx, ld_idx);
  DSA_CHECK_LAUNCH("prefill_positions");
  return DSA_OK;
}

extern "C" int dsa_shard_active(const int32_t* t_active, int32_t* t_local, int B, int lo, int n_local,
                                dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(t_active && t_local && B >= 0 && lo >= 0 && n_local >= 0, "shard_active: bad arguments");
  if (B == 0) return DSA_OK;
  launch_pdl(shard_active_kernel, dim3((B + 127) / 128), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream),
             t_active, t_local, B, lo, n_local);
  DSA_CHECK_LAUNCH("shard_active");
  return DSA_OK;
}

extern "C" int dsa_shard_local_indices(const int32_t* sel, int64_t ld_sel, int k, const int32_t* win_idx,
                                       int64_t ld_win, int W, int lo, int hi, int local_base, int win_base,
                                       int32_t* out, int64_t ld_out, int B, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(sel && out && B >= 0 && k >= 0 && W >= 0, "shard_local_indices: bad arguments");
  DSA_CHECK_ARG(ld_sel >= k && ld_out >= int64_t(W) + k && (!win_idx || ld_win >= W),
                "shard_local_indices: bad strides");
  DSA_CHECK_ARG(lo >= 0 && hi >= lo && local_base >= 0 && win_base >= 0, "shard_local_indices: bad shard range");
  if (B == 0) return DSA_OK;
  launch_pdl(shard_local_indices_kernel, dim3(B), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), sel, ld_sel, k,
             win_idx, ld_win, W, lo, hi, local_base, win_base, out, ld_out);
  DSA_CHECK_LAUNCH("shard_local_indices");
  return DSA_OK;
}
