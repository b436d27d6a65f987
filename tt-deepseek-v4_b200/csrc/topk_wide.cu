// Top-k of a few long rows across many CTAs (the single long context of the
// sequence split: 1 row of 65536 scores on one GPU, 8192 per shard, 16384
// merge candidates).  The per-row kernels of topk.cu give one CTA per row,
// which leaves 147 of 148 SMs idle on such a row.
//
// Same selection and output contract as dsa_indexer_topk (inference.py:
// 5823-5851): masked = s - 1e4 [t >= t_active] (mask_mode 0) or -inf there
// without reading (mask_mode 1); the k largest masked values, ties towards
// the lower position; out = t + win (or ids[t] + win) where masked >= -1000,
// else -1.  Output order: ascending position.
//
// One cooperative launch, grid (cpr, B): each CTA owns a contiguous slice of
// its row, keys (order-preserving uint32 of the masked value) in registers.
// An MSD radix select over 12 + 12 + 8 bits finds the k-th largest key: per
// level every CTA histograms its live keys into a global per-row histogram,
// a grid barrier, then every CTA scans the histogram to the bin holding the
// k-th key.  A last barrier exchanges per-CTA counts of keys above / equal
// to the threshold, which gives each CTA its output offset, so the result
// is written in position order with no atomics on the output.  Grid
// barriers are an arrival count plus a generation word with a clock-bounded
// spin; a wait that runs out sets *status and the CTA returns.  The
// histograms are zeroed again at the end of the launch, so the workspace must be zeroed once
// before its first use (and again after a timeout).
#include "common.cuh"

namespace dsa {
namespace wide {

constexpr int kThreads = 512;
constexpr int kBins = 4096;
constexpr int kLevels = 3;
constexpr int kMaxPerThread = 8;
constexpr long long kSpinCycles = 2000000000ll;  // ~1 s at 1.9 GHz
constexpr int kStatusTimeout = 2;

struct RowWs {
  uint32_t hist[kLevels][kBins];
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier over all nctas CTAs of the launch (sense by generation:
// the last CTA to arrive resets the count, then bumps the generation), so
// launches of any grid size can share one workspace.  False on timeout.
__device__ bool grid_barrier(uint32_t* bar, unsigned nctas, int32_t* status, volatile int* s_ok) {
  uint32_t* count = bar;
  uint32_t* gen = bar + 1;
  __threadfence();  // this thread's histogram / count writes before the arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t g = ld_acquire_u32(gen);
    __threadfence();
    const uint32_t old = atomicAdd(count, 1u);
    int ok = 1;
    if (old == nctas - 1) {
      atomicExch(count, 0u);
      __threadfence();
      atomicAdd(gen, 1u);
    } else {
      const long long t0 = clock64();
      while (ld_acquire_u32(gen) == g) {
        if (clock64() - t0 > kSpinCycles) {
          ok = 0;
          if (status) atomicOr(status, kStatusTimeout);
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

// Block-wide: find the bin d (scanning from the top) where the running count
// of higher bins first reaches `need`.  Returns d and sets *above to the
// count in bins above d.
__device__ int find_bin(const uint32_t* hist, uint32_t need, uint32_t* above, uint32_t* s_part, int* s_res,
                        uint32_t* s_above) {
  constexpr int kPer = kBins / kThreads;  // 8 bins per thread, thread 0 the top bins
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t h[kPer], tot = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    h[i] = __ldcg(hist + (kBins - 1 - (tid * kPer + i)));
    tot += h[i];
  }
  // exclusive scan of tot over threads (descending bin order)
  uint32_t incl = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_part[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < kThreads / 32 ? s_part[lane] : 0;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += v;
    }
    if (lane < kThreads / 32) s_part[lane] = wi - w;  // exclusive warp offsets
  }
  __syncthreads();
  uint32_t run = s_part[warp] + incl - tot;  // count in bins above this thread's first bin
  if (run < need && run + tot >= need) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      if (run < need && run + h[i] >= need) {
        *s_res = kBins - 1 - (tid * kPer + i);
        *s_above = run;
      }
      run += h[i];
    }
  }
  __syncthreads();
  *above = *s_above;
  const int d = *s_res;
  __syncthreads();
  return d;
}

__global__ void __launch_bounds__(kThreads, 1) topk_wide_kernel(
    const float* __restrict__ score, int64_t ld_score, const int32_t* __restrict__ ids, int64_t ld_ids,
    const int32_t* __restrict__ t_active, int T, int k, int win, int mask_mode, int per_cta,
    int32_t* __restrict__ out_idx, float* __restrict__ out_score, int64_t ld_out, RowWs* __restrict__ rows,
    uint32_t* __restrict__ counts, uint32_t* __restrict__ bar, int32_t* __restrict__ status) {
  __shared__ uint32_t s_hist[kBins];
  __shared__ uint32_t s_part[kThreads / 32];
  __shared__ int s_res;
  __shared__ uint32_t s_above;
  __shared__ int s_ok;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.y, c = blockIdx.x, cpr = gridDim.x;
  const unsigned nctas = gridDim.x * gridDim.y;
  const int s0 = c * per_cta;
  const int s1 = min(T, s0 + per_cta);
  const int ept = (per_cta + kThreads - 1) / kThreads;  // elements per thread (<= kMaxPerThread)
  const int e0 = s0 + tid * ept;
  const int ta = t_active ? t_active[b] : T;
  const float* srow = score + int64_t(b) * ld_score;
  const int32_t* irow = ids ? ids + int64_t(b) * ld_ids : nullptr;

  uint32_t key[kMaxPerThread];
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i) {
    const int t = e0 + i;
    key[i] = 0u;  // below every real key: padding
    if (i < ept && t < s1) {
      float v;
      if (irow && irow[t] < 0) {
        v = -INFINITY;
      } else if (t >= ta) {
        v = mask_mode == 1 ? -INFINITY : __fsub_rn(srow[t], 1e4f);
      } else {
        v = srow[t];
      }
      key[i] = float_key(v);
    }
  }

  RowWs* rw = rows + b;
  uint32_t prefix = 0, pmask = 0, need = uint32_t(k);
#pragma unroll 1
  for (int level = 0; level < kLevels; ++level) {
    const int shift = level == 0 ? 20 : (level == 1 ? 8 : 0);
    const uint32_t dmask = level == 2 ? 0xffu : 0xfffu;
    for (int i = tid; i < kBins; i += kThreads) s_hist[i] = 0;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxPerThread; ++i)
      if (i < ept && e0 + i < s1 && (key[i] & pmask) == prefix) atomicAdd(&s_hist[(key[i] >> shift) & dmask], 1u);
    __syncthreads();
    for (int i = tid; i < kBins; i += kThreads)
      if (s_hist[i]) atomicAdd(&rw->hist[level][i], s_hist[i]);
    if (!grid_barrier(bar, nctas, status, &s_ok)) return;
    uint32_t above;
    const int d = find_bin(rw->hist[level], need, &above, s_part, &s_res, &s_above);
    need -= above;
    prefix |= uint32_t(d) << shift;
    pmask |= dmask << shift;
  }
  const uint32_t thr = prefix;  // the k-th largest key; `need` of the keys equal to it are taken

  // per-thread counts above / equal, then per-CTA totals to the global table
  uint32_t n_gt = 0, n_eq = 0;
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i) {
    if (i < ept && e0 + i < s1) {
      n_gt += key[i] > thr;
      n_eq += key[i] == thr;
    }
  }
  // block exclusive scans of n_gt and n_eq (thread order = position order)
  uint32_t ig = n_gt, ie = n_eq;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t vg = __shfl_up_sync(0xffffffffu, ig, o), ve = __shfl_up_sync(0xffffffffu, ie, o);
    if (lane >= o) {
      ig += vg;
      ie += ve;
    }
  }
  __shared__ uint32_t s_wg[kThreads / 32], s_we[kThreads / 32], s_tot[2];
  if (lane == 31) {
    s_wg[warp] = ig;
    s_we[warp] = ie;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t g = lane < kThreads / 32 ? s_wg[lane] : 0, e = lane < kThreads / 32 ? s_we[lane] : 0;
    uint32_t gi = g, ei = e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t vg = __shfl_up_sync(0xffffffffu, gi, o), ve = __shfl_up_sync(0xffffffffu, ei, o);
      if (lane >= o) {
        gi += vg;
        ei += ve;
      }
    }
    if (lane < kThreads / 32) {
      s_wg[lane] = gi - g;
      s_we[lane] = ei - e;
    }
    if (lane == kThreads / 32 - 1) {
      s_tot[0] = gi;
      s_tot[1] = ei;
    }
  }
  __syncthreads();
  const uint32_t thr_gt = s_wg[warp] + ig - n_gt, thr_eq = s_we[warp] + ie - n_eq;
  uint32_t* crow = counts + int64_t(b) * cpr * 2;
  if (tid == 0) {
    crow[2 * c] = s_tot[0];
    crow[2 * c + 1] = s_tot[1];
  }
  if (!grid_barrier(bar, nctas, status, &s_ok)) return;
  // offsets of this CTA: selected elements of the CTAs before it
  uint32_t cg = 0, ce = 0;
  for (int j = tid; j < c; j += kThreads) {
    cg += __ldcg(crow + 2 * j);
    ce += __ldcg(crow + 2 * j + 1);
  }
  cg = __reduce_add_sync(0xffffffffu, cg);
  ce = __reduce_add_sync(0xffffffffu, ce);
  if (lane == 0) {
    s_wg[warp] = cg;
    s_we[warp] = ce;
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t a = 0, e = 0;
    for (int w = 0; w < kThreads / 32; ++w) {
      a += s_wg[w];
      e += s_we[w];
    }
    s_tot[0] = a;
    s_tot[1] = e;
  }
  __syncthreads();
  const uint32_t cta_gt = s_tot[0], cta_eq = s_tot[1];
  // selected before this thread = gt before it + min(eq before it, need)
  uint32_t eq_before = cta_eq + thr_eq;
  uint32_t out_pos = cta_gt + thr_gt + min(eq_before, need);
  int32_t* orow = out_idx + int64_t(b) * ld_out;
  float* osrow = out_score ? out_score + int64_t(b) * ld_out : nullptr;
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i) {
    const int t = e0 + i;
    if (i < ept && t < s1) {
      bool take = key[i] > thr;
      if (key[i] == thr) {
        take = eq_before < need;
        ++eq_before;
      }
      if (take && out_pos < uint32_t(k)) {  // bound holds unless the histograms were not zeroed
        const float v = key_float(key[i]);
        const int id = irow ? irow[t] : t;
        orow[out_pos] = (v >= -1000.f && id >= 0) ? id + win : -1;
        if (osrow) osrow[out_pos] = v;
        ++out_pos;
      }
    }
  }
  // every CTA has read the histograms (before the count barrier): clear them
  // for the next launch
  for (int i = c * kThreads + tid; i < kLevels * kBins; i += cpr * kThreads)
    (&rw->hist[0][0])[i] = 0u;
}

}  // namespace wide
}  // namespace dsa

using namespace dsa;

namespace {
int wide_ctas_per_row(int B, int T) {
  const int by_size = (T + wide::kThreads - 1) / wide::kThreads;
  const int by_sms = std::max(1, num_sms() / std::max(1, B));
  int cpr = std::max(1, std::min(by_size, by_sms));
  // every thread holds at most kMaxPerThread keys
  const int min_cpr = (T + wide::kThreads * wide::kMaxPerThread - 1) / (wide::kThreads * wide::kMaxPerThread);
  return std::max(cpr, min_cpr);
}
}  // namespace

extern "C" size_t dsa_topk_wide_workspace_size(int B, int T) {
  if (B <= 0 || T <= 0) return 0;
  const int cpr = wide_ctas_per_row(B, T);
  return 64 + size_t(B) * sizeof(wide::RowWs) + size_t(B) * cpr * 2 * sizeof(uint32_t);
}

extern "C" int dsa_topk_wide(const float* score, int64_t ld_score, const int32_t* ids, int64_t ld_ids,
                             const int32_t* t_active, int32_t* out_idx, float* out_score, int64_t ld_out, int B, int T,
                             int k, int win, int mask_mode, void* workspace, size_t workspace_bytes, int32_t* status,
                             dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(score && out_idx && workspace, "topk_wide: null pointer");
  DSA_CHECK_ARG(B >= 0 && T > 0 && k > 0 && k <= T, "topk_wide: need 0 < k <= T (k=%d, T=%d)", k, T);
  DSA_CHECK_ARG(ld_score >= T && ld_out >= k && (!ids || ld_ids >= T), "topk_wide: bad strides");
  DSA_CHECK_ARG(mask_mode == 0 || mask_mode == 1, "topk_wide: mask_mode must be 0 or 1");
  DSA_CHECK_ARG(aligned(workspace, 16), "topk_wide: workspace must be 16-byte aligned");
  if (B == 0) return DSA_OK;
  if (workspace_bytes < dsa_topk_wide_workspace_size(B, T)) {
    set_error("topk_wide: workspace %zu bytes < %zu", workspace_bytes, dsa_topk_wide_workspace_size(B, T));
    return DSA_ERR_WORKSPACE;
  }
  const int cpr = wide_ctas_per_row(B, T);
  if (int64_t(cpr) * B > num_sms()) {
    set_error("topk_wide: %d rows x %d CTAs exceed one CTA per SM (%d SMs); use dsa_indexer_topk", B, cpr,
              num_sms());
    return DSA_ERR_UNSUPPORTED;
  }
  const int per_cta = (T + cpr - 1) / cpr;
  auto* base = static_cast<uint8_t*>(workspace);
  auto* bar = reinterpret_cast<uint32_t*>(base);
  auto* rows = reinterpret_cast<wide::RowWs*>(base + 64);
  auto* counts = reinterpret_cast<uint32_t*>(base + 64 + size_t(B) * sizeof(wide::RowWs));

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cpr, B);
  cfg.blockDim = dim3(wide::kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, wide::topk_wide_kernel, score, ld_score, ids, ld_ids, t_active, T, k, win,
                                     mask_mode, per_cta, out_idx, out_score, ld_out, rows, counts, bar, status);
  if (e != cudaSuccess) {
    set_error("topk_wide: launch failed: %s", cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}
