// attn.topk: window indices, masked indexer top-k and candidate merge.
//
// Reference: DeviceAttention._indexer_topk_body (inference.py:5823-5851):
//   masked = score - 1e4 * (t >= T_active); ttnn.topk(masked, k, sorted);
//   out = idx + win where val >= -1000 else -1
// and the window table rows (479-506, picked at 6020-6026).
//
// Selection is an exact block-level radix select over order-preserving
// uint32 keys of the fp32 masked scores: four 8-bit digit passes over the
// candidates held in shared memory, each a warp-aggregated (match_any)
// histogram plus a one-warp suffix scan, find the k-th key; a final
// deterministic compaction emits every key above it and the lowest-index
// keys equal to it.  Rows longer than one CTA's shared-memory budget are cut
// into chunks whose local top-k lists are merged by the same select
// (dsa_topk_merge), which is also the cross-GPU merge of the sequence split.
#include "common.cuh"

namespace dsa {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMaxN = 16384;   // elements one CTA selects from (64 KB keys + 64 KB idx)
constexpr int kTopkMaxK = 4096;

struct SelectScratch {
  uint32_t hist[256];
  uint32_t prefix;
  uint32_t kgt;        // elements strictly above the threshold found so far
  uint32_t warp_cnt[2][32];
};

// Finds the threshold key of the k largest among keys[0, n) (k <= n).
// Returns (threshold, n_above) in s->prefix / s->kgt.
__device__ void radix_select(const uint32_t* keys, int n, int k, SelectScratch* s) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t prefix = 0, pmask = 0;
  int krem = k;
  int kgt = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += blockDim.x) s->hist[i] = 0;
    __syncthreads();
    for (int base = 0; base < n; base += blockDim.x) {
      const int i = base + tid;
      uint32_t bin = 256;
      if (i < n) {
        const uint32_t key = keys[i];
        if ((key & pmask) == prefix) bin = (key >> shift) & 255u;
      }
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (bin < 256 && lane == __ffs(peers) - 1) atomicAdd(&s->hist[bin], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins [8l, 8l+8); suffix counts from the top bin down
      uint32_t h[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        h[j] = s->hist[8 * lane + j];
        tot += h[j];
      }
      uint32_t incl = tot;  // inclusive suffix sum over lanes >= l
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_down_sync(0xffffffffu, incl, o);
        if (lane + o < 32) incl += v;
      }
      uint32_t run = incl - tot;  // count in bins above this lane's range
#pragma unroll
      for (int j = 7; j >= 0; --j) {
        if (run < (uint32_t)krem && run + h[j] >= (uint32_t)krem) {
          s->prefix = prefix | ((uint32_t)(8 * lane + j) << shift);
          s->kgt = run;
        }
        run += h[j];
      }
    }
    __syncthreads();
    prefix = s->prefix;
    pmask |= 0xffu << shift;
    krem -= (int)s->kgt;
    kgt += (int)s->kgt;
    __syncthreads();
  }
  if (tid == 0) s->kgt = (uint32_t)kgt;
  __syncthreads();
}

// Block exclusive scan of two counters (above, equal); returns offsets and
// writes the block totals to tot_a / tot_e.
__device__ void block_scan2(uint32_t a, uint32_t e, uint32_t& off_a, uint32_t& off_e, SelectScratch* s,
                            uint32_t& tot_a, uint32_t& tot_e) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint32_t ia = a, ie = e;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t va = __shfl_up_sync(0xffffffffu, ia, o), ve = __shfl_up_sync(0xffffffffu, ie, o);
    if (lane >= o) {
      ia += va;
      ie += ve;
    }
  }
  if (lane == 31) {
    s->warp_cnt[0][warp] = ia;
    s->warp_cnt[1][warp] = ie;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t wa = lane < nw ? s->warp_cnt[0][lane] : 0, we = lane < nw ? s->warp_cnt[1][lane] : 0;
    uint32_t xa = wa, xe = we;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t va = __shfl_up_sync(0xffffffffu, xa, o), ve = __shfl_up_sync(0xffffffffu, xe, o);
      if (lane >= o) {
        xa += va;
        xe += ve;
      }
    }
    if (lane < nw) {
      s->warp_cnt[0][lane] = xa - wa;
      s->warp_cnt[1][lane] = xe - we;
    }
    if (lane == 31) {
      s->hist[0] = xa;  // block totals (hist is free at this point)
      s->hist[1] = xe;
    }
  }
  __syncthreads();
  off_a = s->warp_cnt[0][warp] + ia - a;
  off_e = s->warp_cnt[1][warp] + ie - e;
  tot_a = s->hist[0];
  tot_e = s->hist[1];
  __syncthreads();
}

// Bitonic sort of n_pow2 (key, idx) pairs in shared memory: descending key,
// ascending idx among equal keys.
__device__ void bitonic_desc(uint64_t* v, int n_pow2) {
  for (int size = 2; size <= n_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n_pow2 / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const uint64_t a = v[lo], b = v[hi];
        if ((a < b) == desc) {
          v[lo] = b;
          v[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

// Selects the k best of (keys[i], ids[i]) for i < n and writes them out.
// mode_final: out index = id + win when the masked score >= -1000, else -1;
// otherwise the raw id is written (intermediate candidate lists).
__device__ void select_and_emit(uint32_t* keys, const int32_t* ids, int n, int k, bool sort_desc, bool mode_final,
                                int win, int32_t* out_idx, float* out_score, uint64_t* sort_buf,
                                SelectScratch* s) {
  radix_select(keys, n, k, s);
  const uint32_t thr = s->prefix;
  const int n_above = (int)s->kgt;
  const int n_eq_take = k - n_above;
  // contiguous per-thread ranges keep the output in ascending position order
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int i0 = threadIdx.x * per, i1 = min(n, i0 + per);
  uint32_t ca = 0, ce = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = keys[i];
    ca += key > thr;
    ce += key == thr;
  }
  uint32_t oa, oe, ta, te;
  block_scan2(ca, ce, oa, oe, s, ta, te);
  (void)ta;
  (void)te;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = keys[i];
    int slot = -1;
    if (key > thr) {
      slot = (int)oa++;
    } else if (key == thr) {
      if ((int)oe < n_eq_take) slot = n_above + (int)oe;
      ++oe;
    }
    if (slot >= 0) {
      const int32_t id = ids ? ids[i] : i;
      if (sort_desc) {
        sort_buf[slot] = ((uint64_t)key << 32) | (uint64_t)(0x7fffffffu - (uint32_t)id);
      } else {
        const float f = key_float(key);
        const bool ok = id >= 0 && f >= -1000.0f;
        out_idx[slot] = mode_final ? (ok ? id + win : -1) : id;
        if (out_score) out_score[slot] = f;
      }
    }
  }
  if (sort_desc) {
    __syncthreads();
    int np2 = 1;
    while (np2 < k) np2 <<= 1;
    for (int i = k + threadIdx.x; i < np2; i += blockDim.x) sort_buf[i] = 0;
    __syncthreads();
    bitonic_desc(sort_buf, np2);
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      const uint64_t v = sort_buf[i];
      const uint32_t key = (uint32_t)(v >> 32);
      const int32_t id = (int32_t)(0x7fffffffu - (uint32_t)(v & 0xffffffffu));
      const float f = key_float(key);
      const bool ok = id >= 0 && f >= -1000.0f;
      out_idx[i] = mode_final ? (ok ? id + win : -1) : id;
      if (out_score) out_score[i] = f;
    }
  }
}

// grid (n_chunks, B).  Chunk c of row b covers t in [c*chunk, min(T, (c+1)*chunk)).
// n_chunks == 1: final output.  Otherwise raw candidates at
// cand[(b*n_chunks + c)*k ...] (fewer than k real ones pad with key 0 / id -1).
__global__ void __launch_bounds__(kTopkThreads) topk_chunk_kernel(
    const float* __restrict__ score, int64_t ld_score, const int32_t* __restrict__ t_active, int T, int chunk, int k,
    int win, int sort_desc, int mask_mode, int32_t* __restrict__ out_idx, float* __restrict__ out_score, int64_t ld_out,
    uint32_t* __restrict__ cand_key, int32_t* __restrict__ cand_id) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ SelectScratch s;
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
  uint64_t* sort_buf = reinterpret_cast<uint64_t*>(smem + kTopkMaxN * 4);
  const int b = blockIdx.y, c = blockIdx.x, n_chunks = gridDim.x;
  const int t0 = c * chunk;
  const int n = min(T, t0 + chunk) - t0;
  const int ta = t_active[b];
  const float* row = score + int64_t(b) * ld_score + t0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float m;
    if (t0 + i < ta) m = row[i];
    else m = mask_mode ? -INFINITY : __fsub_rn(row[i], 1.0e4f);
    keys[i] = float_key(m);
  }
  __syncthreads();
  if (n_chunks == 1) {
    select_and_emit(keys, nullptr, n, k, sort_desc != 0, true, win, out_idx + int64_t(b) * ld_out,
                    out_score ? out_score + int64_t(b) * ld_out : nullptr, sort_buf, &s);
    return;
  }
  // intermediate: ids are global positions
  const int kk = min(k, n);
  int32_t* ids = reinterpret_cast<int32_t*>(smem + kTopkMaxN * 4);
  for (int i = threadIdx.x; i < n; i += blockDim.x) ids[i] = t0 + i;
  __syncthreads();
  const int64_t base = (int64_t(b) * n_chunks + c) * k;
  // write keys of the selected candidates: emit ids into cand_id, then keys
  select_and_emit(keys, ids, n, kk, false, false, 0, cand_id + base, nullptr, nullptr, &s);
  __syncthreads();
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    if (i < kk) {
      const int32_t id = cand_id[base + i];
      cand_key[base + i] = keys[id - t0];
    } else {
      cand_key[base + i] = 0u;
      cand_id[base + i] = -1;
    }
  }
}

// grid (B).  Selects the k best of n_cand candidates per row.  keys_in: either
// ordered-uint keys (cand_key) or fp32 masked scores (cand_score).
__global__ void __launch_bounds__(kTopkThreads) topk_merge_kernel(
    const uint32_t* __restrict__ cand_key, const float* __restrict__ cand_score, const int32_t* __restrict__ cand_id,
    int n_cand, int k, int win, int sort_desc, int final_mode, int32_t* __restrict__ out_idx,
    float* __restrict__ out_score, int64_t ld_out) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ SelectScratch s;
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
  int32_t* ids = reinterpret_cast<int32_t*>(smem + kTopkMaxN * 4);
  uint64_t* sort_buf = reinterpret_cast<uint64_t*>(smem + kTopkMaxN * 8);
  const int b = blockIdx.x;
  for (int i = threadIdx.x; i < n_cand; i += blockDim.x) {
    const int32_t id = cand_id[int64_t(b) * n_cand + i];
    uint32_t key;
    if (cand_key) key = cand_key[int64_t(b) * n_cand + i];
    else key = float_key(cand_score[int64_t(b) * n_cand + i]);
    ids[i] = id;
    keys[i] = (id < 0) ? 0u : key;
  }
  __syncthreads();
  select_and_emit(keys, ids, n_cand, k, sort_desc != 0, final_mode != 0, win, out_idx + int64_t(b) * ld_out,
                  out_score ? out_score + int64_t(b) * ld_out : nullptr, sort_buf, &s);
}

__global__ void window_indices_kernel(const int32_t* __restrict__ pos, int32_t* __restrict__ idx, int64_t ld,
                                      int B, int win) {
  const int b = blockIdx.x;
  const int p = pos[b];
  for (int i = threadIdx.x; i < win; i += blockDim.x) {
    int v;
    if (p < win) v = (i <= p) ? i : -1;
    else v = (p % win + 1 + i) % win;
    idx[int64_t(b) * ld + i] = v;
  }
}

}  // namespace dsa

using namespace dsa;

namespace {
int chunk_smem() { return kTopkMaxN * 4 + std::max(kTopkMaxN * 4, kTopkMaxK * 8); }
int merge_smem() { return kTopkMaxN * 8 + kTopkMaxK * 8; }
}  // namespace

extern "C" int dsa_window_indices(const int32_t* pos, int32_t* idx, int64_t ld_idx, int B, int win,
                                  dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(pos && idx, "window_indices: null pointer");
  DSA_CHECK_ARG(B >= 0 && win > 0 && ld_idx >= win, "window_indices: bad B/win/ld");
  if (B == 0) return DSA_OK;
  window_indices_kernel<<<B, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(pos, idx, ld_idx, B, win);
  DSA_CHECK_LAUNCH("window_indices");
  return DSA_OK;
}

// Rows longer than kTopkMaxN are selected in two levels; the per-chunk
// candidate lists go to caller-owned workspace (no allocation here).
extern "C" size_t dsa_indexer_topk_workspace_size(int B, int T, int k) {
  if (T <= kTopkMaxN) return 0;
  const int n_chunks = (T + kTopkMaxN - 1) / kTopkMaxN;
  return size_t(B) * n_chunks * k * 8;
}

static int topk_launch(const float* score, int64_t ld_score, const int32_t* t_active, int32_t* out_idx,
                       float* out_score, int64_t ld_out, int B, int T, int k, int win, int sort_desc, int mask_mode,
                       void* ws, size_t ws_bytes, cudaStream_t st) {
  DSA_CHECK_ARG(score && t_active && out_idx, "indexer_topk: null pointer");
  DSA_CHECK_ARG(B >= 0 && T > 0 && k > 0 && k <= T, "indexer_topk: need 0 < k <= T (k=%d T=%d)", k, T);
  DSA_CHECK_ARG(k <= kTopkMaxK, "indexer_topk: k=%d above the built maximum %d", k, kTopkMaxK);
  DSA_CHECK_ARG(ld_score >= T && ld_out >= k, "indexer_topk: bad strides");
  if (B == 0) return DSA_OK;
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    cudaFuncSetAttribute(topk_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, chunk_smem());
    cudaFuncSetAttribute(topk_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, merge_smem());
    attr_dev = dev;
  }
  if (T <= kTopkMaxN) {
    topk_chunk_kernel<<<dim3(1, B), kTopkThreads, chunk_smem(), st>>>(score, ld_score, t_active, T, T, k, win,
                                                                     sort_desc, mask_mode, out_idx, out_score,
                                                                     ld_out, nullptr, nullptr);
    DSA_CHECK_LAUNCH("indexer_topk");
    return DSA_OK;
  }
  const int n_chunks = (T + kTopkMaxN - 1) / kTopkMaxN;
  const size_t need = size_t(B) * n_chunks * k * 8;
  if (ws_bytes < need || ws == nullptr) {
    set_error("indexer_topk: T=%d needs %zu bytes of workspace (got %zu)", T, need, ws_bytes);
    return DSA_ERR_WORKSPACE;
  }
  DSA_CHECK_ARG(int64_t(n_chunks) * k <= kTopkMaxN, "indexer_topk: T=%d k=%d exceeds the two-level merge", T, k);
  uint32_t* ck = static_cast<uint32_t*>(ws);
  int32_t* ci = reinterpret_cast<int32_t*>(ck + size_t(B) * n_chunks * k);
  topk_chunk_kernel<<<dim3(n_chunks, B), kTopkThreads, chunk_smem(), st>>>(
      score, ld_score, t_active, T, kTopkMaxN, k, win, 0, mask_mode, nullptr, nullptr, 0, ck, ci);
  DSA_CHECK_LAUNCH("indexer_topk(chunks)");
  topk_merge_kernel<<<B, kTopkThreads, merge_smem(), st>>>(ck, nullptr, ci, n_chunks * k, k, win, sort_desc, 1,
                                                            out_idx, out_score, ld_out);
  DSA_CHECK_LAUNCH("indexer_topk(merge)");
  return DSA_OK;
}

extern "C" int dsa_indexer_topk(const float* score, int64_t ld_score, const int32_t* t_active, int32_t* out_idx,
                                float* out_score, int64_t ld_out, int B, int T, int k, int win, int sort_desc,
                                int mask_mode, dsa_stream_t stream) {
  clear_error();
  return topk_launch(score, ld_score, t_active, out_idx, out_score, ld_out, B, T, k, win, sort_desc, mask_mode,
                     nullptr, 0, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dsa_indexer_topk_ws(const float* score, int64_t ld_score, const int32_t* t_active, int32_t* out_idx,
                                   float* out_score, int64_t ld_out, int B, int T, int k, int win, int sort_desc,
                                   int mask_mode, void* workspace, size_t workspace_bytes, dsa_stream_t stream) {
  clear_error();
  return topk_launch(score, ld_score, t_active, out_idx, out_score, ld_out, B, T, k, win, sort_desc, mask_mode,
                     workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

__global__ void advance_positions_kernel(int32_t* pos, int32_t* t_active, int B, int ratio, int step) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    const int p = pos[b] + step;
    pos[b] = p;
    if (t_active) t_active[b] = (p + 1) / ratio;
  }
}

extern "C" int dsa_advance_positions(int32_t* pos, int32_t* t_active, int B, int ratio, int step,
                                     dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(pos && B >= 0 && ratio > 0, "advance_positions: bad arguments");
  if (B == 0) return DSA_OK;
  advance_positions_kernel<<<(B + 127) / 128, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(pos, t_active, B,
                                                                                               ratio, step);
  DSA_CHECK_LAUNCH("advance_positions");
  return DSA_OK;
}

extern "C" int dsa_topk_merge(const float* cand_score, const int32_t* cand_idx, int n_cand, int32_t* out_idx,
                              float* out_score, int64_t ld_out, int B, int k, int win, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(cand_score && cand_idx && out_idx, "topk_merge: null pointer");
  DSA_CHECK_ARG(B >= 0 && n_cand > 0 && n_cand <= kTopkMaxN, "topk_merge: n_cand=%d outside (0, %d]", n_cand,
                kTopkMaxN);
  DSA_CHECK_ARG(k > 0 && k <= n_cand && k <= kTopkMaxK, "topk_merge: bad k=%d", k);
  DSA_CHECK_ARG(ld_out >= k, "topk_merge: ld_out < k");
  if (B == 0) return DSA_OK;
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    cudaFuncSetAttribute(topk_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, merge_smem());
    attr_dev = dev;
  }
  topk_merge_kernel<<<B, kTopkThreads, merge_smem(), reinterpret_cast<cudaStream_t>(stream)>>>(
      nullptr, cand_score, cand_idx, n_cand, k, win, 1, 1, out_idx, out_score, ld_out);
  DSA_CHECK_LAUNCH("topk_merge");
  return DSA_OK;
}
