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
// MSD radix select: every CTA histograms the top 12 bits of its keys into a
// global per-row histogram; after a grid barrier every CTA scans it to the
// bin holding the k-th key.  Each CTA then publishes its count of keys above
// that bin and its keys in it (at most kCap, in position order); after a
// second barrier every CTA loads all published bin keys (a few hundred for
// continuous scores) and finishes the select on their low 20 bits in shared
// memory.  The per-CTA counts give each CTA its output offset, so the result
// is written in position order with no atomics on the output.  A crowded bin
// (some CTA holding more than kCap of its keys: ties, quantised scores) takes
// two more grid-wide 12/8-bit levels and a count exchange instead.  Grid
// barriers are an arrival count plus a generation word with a clock-bounded
// spin; a wait that runs out sets *status and the CTA returns.  The
// histograms are zeroed again at the end of the launch, so the workspace must be zeroed once
// before its first use (and again after a timeout).  Workspace layout: a
// 64-byte header, the per-launch count and candidate slots of up to
// kScratchCtas CTAs at fixed offsets, then one histogram block per row; the
// slots are rewritten by every launch and never overlap a histogram block,
// so one workspace serves launches of any row count.
#include "common.cuh"

namespace dsa {
namespace wide {

constexpr int kThreads = 512;
constexpr int kBins = 4096;
constexpr int kLevels = 3;
constexpr int kMaxPerThread = 8;
constexpr int kStatusTimeout = 2;
constexpr int kCap = 24;                 // level-0 bin keys one CTA may publish
constexpr int kMaxCtasPerRow = 148;
constexpr int kCandSmem = kCap * kMaxCtasPerRow;
constexpr int kScratchCtas = 1024;       // CTAs of one launch the count / candidate slots hold

struct RowWs {
  uint32_t hist[kLevels][kBins];
  uint32_t bar[4];  // this row's grid barrier: arrival count, generation
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Barrier over the nctas CTAs of one row (sense by generation:
// the last CTA to arrive resets the count, then bumps the generation), so
// launches of any grid size can share one workspace.  Thread 0 arrives with
// release semantics after the CTA's __syncthreads, which orders the whole
// CTA's prior writes; waiters poll the generation with acquire loads.
// False on timeout.
__device__ bool grid_barrier(uint32_t* bar, unsigned nctas, int32_t* status, volatile int* s_ok, long long spin) {
  uint32_t* count = bar;
  uint32_t* gen = bar + 1;
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t g = ld_acquire_u32(gen);
    const uint32_t old = atom_add_acq_rel(count, 1u);
    int ok = 1;
    if (old == nctas - 1) {
      atomicExch(count, 0u);
      atom_add_acq_rel(gen, 1u);
    } else {
      const long long t0 = clock64();
      int polls = 0;
      while (ld_acquire_u32(gen) == g) {
        if (++polls > 256) __nanosleep(32);
        if (clock64() - t0 > spin) {
          ok = 0;
          if (status) atomicOr(status, kStatusTimeout);
          break;
        }
      }
    }
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

// Block-wide exclusive scan of one value per thread (thread order); returns
// the exclusive prefix and writes the block total to *total.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* s_w, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) s_w[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = lane < nw ? s_w[lane] : 0;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < nw) s_w[lane] = wi - w;
    if (lane == nw - 1) s_w[32] = wi;
  }
  __syncthreads();
  const uint32_t r = s_w[warp] + inc - v;
  *total = s_w[32];
  __syncthreads();
  return r;
}

// Block-wide: find the bin d (scanning from the top of nbins) where the
// running count of higher bins first reaches `need`; *above = the count in
// bins above d.  hist is global (L2) or shared memory.
template <int kPer, bool kGlobal>
__device__ int find_bin(const uint32_t* hist, int nbins, uint32_t need, uint32_t* above, uint32_t* s_w,
                        int* s_res, uint32_t* s_above) {
  const int tid = threadIdx.x;
  uint32_t h[kPer], tot = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int bin = nbins - 1 - (tid * kPer + i);
    h[i] = bin >= 0 ? (kGlobal ? __ldcg(hist + bin) : hist[bin]) : 0u;
    tot += h[i];
  }
  uint32_t all;
  uint32_t run = block_excl_scan(tot, s_w, &all);
  if (run < need && run + tot >= need) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      if (run < need && run + h[i] >= need) {
        *s_res = nbins - 1 - (tid * kPer + i);
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

// per-row counters: [0] keys above the level-0 bin, [1] keys in it, [2] keys
// above the final threshold, [3] keys equal to it (overflow path)
constexpr int kCountWords = 4;

__global__ void __launch_bounds__(kThreads, 1) topk_wide_kernel(
    const float* __restrict__ score, int64_t ld_score, const int32_t* __restrict__ ids, int64_t ld_ids,
    const int32_t* __restrict__ t_active, int T, int k, int win, int mask_mode, int per_cta, int seg_len,
    int64_t seg_stride,
    int32_t* __restrict__ out_idx, float* __restrict__ out_score, int64_t ld_out, RowWs* __restrict__ rows,
    uint32_t* __restrict__ counts, unsigned long long* __restrict__ cands, int32_t* __restrict__ status,
    long long spin) {
  __shared__ uint32_t s_hist[kBins];
  __shared__ unsigned long long s_cand[kCandSmem];
  __shared__ uint32_t s_w[33];
  __shared__ uint32_t s_coff[kMaxCtasPerRow + 1];
  __shared__ int s_res;
  __shared__ uint32_t s_above;
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  const int b = blockIdx.y, c = blockIdx.x, cpr = gridDim.x;
  const int s0 = c * per_cta;
  const int s1 = min(T, s0 + per_cta);
  const int ept = (per_cta + kThreads - 1) / kThreads;  // elements per thread (<= kMaxPerThread)
  const int e0 = s0 + tid * ept;
  const int ta = t_active ? t_active[b] : T;
  const float* srow = score + int64_t(b) * ld_score;
  const int32_t* irow = ids ? ids + int64_t(b) * ld_ids : nullptr;
  RowWs* rw = rows + b;
  uint32_t* bar = rw->bar;  // rows are independent: each synchronises only its own CTAs
  const unsigned nctas = cpr;
  uint32_t* crow = counts + int64_t(b) * cpr * kCountWords;
  unsigned long long* cand_row = cands + int64_t(b) * cpr * kCap;

  uint32_t key[kMaxPerThread];
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i) {
    const int t = e0 + i;
    key[i] = 0u;  // below every real key: padding
    if (i < ept && t < s1) {
      // a segmented row (the gathered candidate lists) lives in pieces of
      // seg_len elements seg_stride apart
      const int64_t at = seg_len > 0 ? int64_t(t / seg_len) * seg_stride + t % seg_len : int64_t(t);
      float v;
      if (irow && irow[at] < 0) {
        v = -INFINITY;
      } else if (t >= ta) {
        v = mask_mode == 1 ? -INFINITY : __fsub_rn(srow[at], 1e4f);
      } else {
        v = srow[at];
      }
      key[i] = float_key(v);
    }
  }
  auto live = [&](int i) { return i < ept && e0 + i < s1; };

  // ---- level 0: top 12 bits over the whole row
  for (int i = tid; i < kBins; i += kThreads) s_hist[i] = 0;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i)
    if (live(i)) atomicAdd(&s_hist[key[i] >> 20], 1u);
  __syncthreads();
  for (int i = tid; i < kBins; i += kThreads)
    if (s_hist[i]) atomicAdd(&rw->hist[0][i], s_hist[i]);
  if (!grid_barrier(bar, nctas, status, &s_ok, spin)) return;
  uint32_t above;
  const uint32_t d0 = find_bin<kBins / kThreads, true>(rw->hist[0], kBins, uint32_t(k), &above, s_w, &s_res,
                                                       &s_above);
  uint32_t need = uint32_t(k) - above;  // keys still to take from bin d0

  // ---- exchange: per CTA the keys above bin d0, and the keys in it
  uint32_t n_gt = 0, n_in = 0;
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i) {
    if (live(i)) {
      n_gt += (key[i] >> 20) > d0;
      n_in += (key[i] >> 20) == d0;
    }
  }
  uint32_t cta_gt, cta_in;
  (void)block_excl_scan(n_gt, s_w, &cta_gt);
  const uint32_t in_base = block_excl_scan(n_in, s_w, &cta_in);  // this thread's first in-bin slot
  if (tid == 0) {
    crow[kCountWords * c + 0] = cta_gt;
    crow[kCountWords * c + 1] = cta_in;
  }
  if (cta_in <= uint32_t(kCap)) {
    uint32_t slot = in_base;
#pragma unroll
    for (int i = 0; i < kMaxPerThread; ++i) {
      if (live(i) && (key[i] >> 20) == d0) {
        cand_row[int64_t(c) * kCap + slot] = (uint64_t(key[i]) << 32) | uint32_t(e0 + i - s0);
        ++slot;
      }
    }
  }
  if (!grid_barrier(bar, nctas, status, &s_ok, spin)) return;
  // level-0 histogram: every CTA read it before the barrier above
  for (int i = c * kThreads + tid; i < kBins; i += cpr * kThreads) rw->hist[0][i] = 0u;

  // the row's per-CTA counts: offsets of this CTA and the overflow test
  uint32_t my_gt = 0, my_in = 0, over = 0;
  if (tid < cpr) {
    my_gt = __ldcg(crow + kCountWords * tid + 0);
    my_in = __ldcg(crow + kCountWords * tid + 1);
    over = my_in > uint32_t(kCap);
  }
  over = __syncthreads_or(over);
  uint32_t tot_in;
  const uint32_t in_off = block_excl_scan(tid < cpr ? my_in : 0u, s_w, &tot_in);  // candidates before CTA tid
  if (tid < cpr) s_coff[tid] = in_off;
  if (tid == 0) s_coff[cpr] = tot_in;
  uint32_t gt_all;
  const uint32_t gt_off = block_excl_scan(tid < cpr ? my_gt : 0u, s_w, &gt_all);
  if (tid == c) s_above = gt_off;
  __syncthreads();
  const uint32_t gt_before = s_above;  // keys above bin d0 in the CTAs before this one

  int32_t* orow = out_idx + int64_t(b) * ld_out;
  float* osrow = out_score ? out_score + int64_t(b) * ld_out : nullptr;
  auto emit = [&](uint32_t out_pos, uint32_t kk, int t) {
    if (out_pos < uint32_t(k)) {  // holds unless the histograms were not zeroed
      const float v = key_float(kk);
      const int64_t at = seg_len > 0 ? int64_t(t / seg_len) * seg_stride + t % seg_len : int64_t(t);
      const int id = irow ? irow[at] : t;
      orow[out_pos] = (v >= -1000.f && id >= 0) ? id + win : -1;
      if (osrow) osrow[out_pos] = v;
    }
  };

  if (!over && tot_in <= uint32_t(kCandSmem)) {
    // ---- fast path: select `need` of the tot_in bin-d0 keys in every CTA
    for (int j = tid; j < cpr; j += kThreads) {
      const uint32_t o = s_coff[j], n = s_coff[j + 1] - o;
      for (uint32_t q = 0; q < n; ++q) s_cand[o + q] = __ldcg(cand_row + int64_t(j) * kCap + q);
    }
    __syncthreads();
    // two 10-bit passes over the low 20 bits, in shared memory
    uint32_t prefix = d0 << 20, pmask = 0xfff00000u;
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
      const int shift = pass == 0 ? 10 : 0;
      for (int i = tid; i < 1024; i += kThreads) s_hist[i] = 0;
      __syncthreads();
      for (uint32_t j = tid; j < tot_in; j += kThreads) {
        const uint32_t kk = uint32_t(s_cand[j] >> 32);
        if ((kk & pmask) == prefix) atomicAdd(&s_hist[(kk >> shift) & 0x3ffu], 1u);
      }
      __syncthreads();
      uint32_t ab;
      const uint32_t dd = find_bin<2, false>(s_hist, 1024, need, &ab, s_w, &s_res, &s_above);
      need -= ab;
      prefix |= dd << shift;
      pmask |= 0x3ffu << shift;
    }
    const uint32_t thr = prefix;  // the k-th largest key; `need` keys equal to it are taken
    // selection flags of the candidates, in position order: > thr, or the
    // first `need` equal to thr; count the selected ones before this CTA
    const uint32_t per = (tot_in + kThreads - 1) / kThreads;
    const uint32_t j0 = tid * per, j1 = min(tot_in, j0 + per);
    uint32_t n_eq = 0;
    for (uint32_t j = j0; j < j1; ++j) n_eq += uint32_t(s_cand[j] >> 32) == thr;
    uint32_t eq_tot;
    uint32_t eq_before = block_excl_scan(n_eq, s_w, &eq_tot);
    const uint32_t my0 = s_coff[c];
    uint32_t sel_before = 0;  // selected candidates before this CTA's own
    for (uint32_t j = j0; j < j1; ++j) {
      const uint32_t kk = uint32_t(s_cand[j] >> 32);
      bool sel = kk > thr;
      if (kk == thr) {
        sel = eq_before < need;
        ++eq_before;
      }
      // mark the selection in bit 31 of the entry's position word (positions are < 2^13)
      if (sel) s_cand[j] |= 0x80000000ull;
      if (sel && j < my0) ++sel_before;
    }
    uint32_t sel_tot;  // selected candidates before this CTA's own (summed over threads)
    (void)block_excl_scan(sel_before, s_w, &sel_tot);
    const uint32_t cta_base = gt_before + sel_tot;
    // this thread's outputs in position order
    uint32_t n_sel = 0;
    uint32_t slot = my0 + in_base;
#pragma unroll
    for (int i = 0; i < kMaxPerThread; ++i) {
      if (live(i)) {
        const uint32_t dg = key[i] >> 20;
        if (dg > d0) {
          ++n_sel;
        } else if (dg == d0) {
          n_sel += (s_cand[slot] & 0x80000000ull) ? 1u : 0u;
          ++slot;
        }
      }
    }
    uint32_t cta_sel;
    uint32_t out_pos = cta_base + block_excl_scan(n_sel, s_w, &cta_sel);
    slot = my0 + in_base;
#pragma unroll
    for (int i = 0; i < kMaxPerThread; ++i) {
      if (live(i)) {
        const uint32_t dg = key[i] >> 20;
        bool take = dg > d0;
        if (dg == d0) {
          take = (s_cand[slot] & 0x80000000ull) != 0;
          ++slot;
        }
        if (take) emit(out_pos++, key[i], e0 + i);
      }
    }
    return;
  }

  // ---- overflow path (a crowded level-0 bin): two more levels grid-wide
  uint32_t prefix = d0 << 20, pmask = 0xfff00000u;
#pragma unroll 1
  for (int level = 1; level < kLevels; ++level) {
    const int shift = level == 1 ? 8 : 0;
    const uint32_t dmask = level == 1 ? 0xfffu : 0xffu;
    for (int i = tid; i < kBins; i += kThreads) s_hist[i] = 0;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxPerThread; ++i)
      if (live(i) && (key[i] & pmask) == prefix) atomicAdd(&s_hist[(key[i] >> shift) & dmask], 1u);
    __syncthreads();
    for (int i = tid; i < kBins; i += kThreads)
      if (s_hist[i]) atomicAdd(&rw->hist[level][i], s_hist[i]);
    if (!grid_barrier(bar, nctas, status, &s_ok, spin)) return;
    uint32_t ab;
    const uint32_t dd = find_bin<kBins / kThreads, true>(rw->hist[level], kBins, need, &ab, s_w, &s_res, &s_above);
    need -= ab;
    prefix |= dd << shift;
    pmask |= dmask << shift;
  }
  const uint32_t thr = prefix;
  uint32_t g2 = 0, q2 = 0;
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i) {
    if (live(i)) {
      g2 += key[i] > thr;
      q2 += key[i] == thr;
    }
  }
  uint32_t cg2, cq2;
  const uint32_t tg = block_excl_scan(g2, s_w, &cg2);
  const uint32_t tq = block_excl_scan(q2, s_w, &cq2);
  if (tid == 0) {
    crow[kCountWords * c + 2] = cg2;
    crow[kCountWords * c + 3] = cq2;
  }
  if (!grid_barrier(bar, nctas, status, &s_ok, spin)) return;
  for (int i = c * kThreads + tid; i < (kLevels - 1) * kBins; i += cpr * kThreads) (&rw->hist[1][0])[i] = 0u;
  uint32_t pg = 0, pq = 0;
  if (tid < c) {
    pg = __ldcg(crow + kCountWords * tid + 2);
    pq = __ldcg(crow + kCountWords * tid + 3);
  }
  uint32_t before_g, before_q;
  (void)block_excl_scan(pg, s_w, &before_g);
  (void)block_excl_scan(pq, s_w, &before_q);
  uint32_t eq_before = before_q + tq;
  uint32_t out_pos = before_g + tg + min(eq_before, need);
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i) {
    if (live(i)) {
      bool take = key[i] > thr;
      if (key[i] == thr) {
        take = eq_before < need;
        ++eq_before;
      }
      if (take) emit(out_pos++, key[i], e0 + i);
    }
  }
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

namespace {
constexpr size_t kWideCountBytes = size_t(wide::kScratchCtas) * wide::kCountWords * sizeof(uint32_t);
constexpr size_t kWideCandBytes = size_t(wide::kScratchCtas) * wide::kCap * sizeof(unsigned long long);
constexpr size_t kWideRowsOffset = 64 + kWideCountBytes + kWideCandBytes;
}  // namespace

extern "C" size_t dsa_topk_wide_workspace_size(int B, int T) {
  if (B <= 0 || T <= 0) return 0;
  return kWideRowsOffset + size_t(B) * sizeof(wide::RowWs);
}

extern "C" int dsa_topk_wide(const float* score, int64_t ld_score, const int32_t* ids, int64_t ld_ids,
                             const int32_t* t_active, int32_t* out_idx, float* out_score, int64_t ld_out, int B, int T,
                             int k, int win, int mask_mode, int seg_len, int64_t seg_stride, void* workspace,
                             size_t workspace_bytes, int32_t* status, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(score && out_idx && workspace, "topk_wide: null pointer");
  DSA_CHECK_ARG(B >= 0 && T > 0 && k > 0 && k <= T, "topk_wide: need 0 < k <= T (k=%d, T=%d)", k, T);
  DSA_CHECK_ARG(seg_len >= 0 && (seg_len == 0 || (T % seg_len == 0 && seg_stride >= seg_len)),
                "topk_wide: T must be a whole number of segments of seg_len <= seg_stride");
  // contiguous rows: ld >= T; segmented rows: the B rows' pieces of one
  // segment, ld apart, fit in seg_stride
  auto ld_ok = [&](int64_t ld) {
    return seg_len > 0 ? (ld >= seg_len && int64_t(B - 1) * ld + seg_len <= seg_stride) : ld >= T;
  };
  DSA_CHECK_ARG(ld_ok(ld_score) && ld_out >= k && (!ids || ld_ok(ld_ids)), "topk_wide: bad strides");
  DSA_CHECK_ARG(mask_mode == 0 || mask_mode == 1, "topk_wide: mask_mode must be 0 or 1");
  DSA_CHECK_ARG(aligned(workspace, 16), "topk_wide: workspace must be 16-byte aligned");
  if (B == 0) return DSA_OK;
  if (workspace_bytes < dsa_topk_wide_workspace_size(B, T)) {
    set_error("topk_wide: workspace %zu bytes < %zu", workspace_bytes, dsa_topk_wide_workspace_size(B, T));
    return DSA_ERR_WORKSPACE;
  }
  const int cpr = wide_ctas_per_row(B, T);
  if (int64_t(cpr) * B > num_sms() || cpr > wide::kMaxCtasPerRow) {
    set_error("topk_wide: %d rows x %d CTAs exceed one CTA per SM (%d SMs); use dsa_indexer_topk", B, cpr,
              num_sms());
    return DSA_ERR_UNSUPPORTED;
  }
  DSA_CHECK_ARG(int64_t(cpr) * B <= wide::kScratchCtas, "topk_wide: %d CTAs exceed the %d workspace slots",
                cpr * B, wide::kScratchCtas);
  const int per_cta = (T + cpr - 1) / cpr;
  auto* base = static_cast<uint8_t*>(workspace);
  auto* counts = reinterpret_cast<uint32_t*>(base + 64);
  auto* cands = reinterpret_cast<unsigned long long*>(base + 64 + kWideCountBytes);
  auto* rows = reinterpret_cast<wide::RowWs*>(base + kWideRowsOffset);

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
                                     mask_mode, per_cta, seg_len, seg_stride, out_idx, out_score, ld_out, rows,
                                     counts, cands, status, wait_limit_cycles());
  if (e != cudaSuccess) {
    set_error("topk_wide: launch failed: %s", cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}
