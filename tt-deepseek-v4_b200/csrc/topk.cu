// attn.topk: window indices, masked indexer top-k and candidate merge.
//
// Reference: DeviceAttention._indexer_topk_body (inference.py:5823-5851):
//   masked = score - 1e4 * (t >= T_active); ttnn.topk(masked, k, sorted);
//   out = idx + win where val >= -1000 else -1
// and the window table rows (479-506, picked at 6020-6026).
//
// Selection is exact and deterministic.  Each thread keeps its keys (the
// order-preserving uint32 of the masked fp32 scores) in registers.  The first
// level histograms the live scores linearly in value between their min and
// max into 256 bins (a monotone map, so exact; masked -inf positions are left
// out when at least k keys lie above them), a one-warp suffix scan finds the
// bin holding the k-th largest, and only that bin's keys are kept.  When at
// most 256 are, each is ranked directly (one thread per candidate counts the
// candidates above it).  Heavily clustered rows go through further levels
// that bin the survivors' keys over their own range (each narrows it by
// 2^8), or, with at most 512 left, one warp bisects over their key bits with
// ballot counts.  A deterministic compaction (ballot ranks inside each warp,
// one scan over the warp counts) then emits every key above the threshold
// and the lowest-index keys equal to it, in position order.  Rows longer than one CTA's shared-memory budget are cut
// into chunks whose local top-k lists are merged by the same select
// (dsa_topk_merge), which is also the cross-GPU merge of the sequence split.
#include "common.cuh"
#include "indexer_row.cuh"
#include "window_rows.cuh"

namespace dsa {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMaxN = 16384;   // elements one CTA selects from (64 KB keys + 64 KB idx)
constexpr int kTopkMaxK = 4096;
constexpr int kKeysPerThread = kTopkMaxN / kTopkThreads;  // 16
// per-CTA scratch after keys and ids: the survivors of a level during the
// select, then the (key, id) pairs of the optional descending sort
constexpr int kScratchBytes = (kTopkMaxN * 4 > kTopkMaxK * 8) ? kTopkMaxN * 4 : kTopkMaxK * 8;
constexpr uint32_t kNoBin = 0xffffffffu;

struct SelectScratch {
  uint32_t hist[256];
  uint32_t prefix;
  uint32_t kgt;        // keys in bins above the chosen one
  uint32_t ncand;
  uint32_t warp_cnt[2][32];
  uint32_t part[32][4];
  float fix_dot[64];  // per-head dots of the recomputed newest entry
};

// Block-wide min / max / sum of one value each per thread; every thread
// receives the results.
__device__ __forceinline__ void block_minmax_sum(uint32_t lo, uint32_t hi, uint32_t cnt, SelectScratch* s,
                                                 uint32_t& mn, uint32_t& mx, uint32_t& sum) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  lo = __reduce_min_sync(0xffffffffu, lo);
  hi = __reduce_max_sync(0xffffffffu, hi);
  cnt = __reduce_add_sync(0xffffffffu, cnt);
  if (lane == 0) {
    s->part[warp][0] = lo;
    s->part[warp][1] = hi;
    s->part[warp][2] = cnt;
  }
  __syncthreads();
  mn = __reduce_min_sync(0xffffffffu, lane < nw ? s->part[lane][0] : 0xffffffffu);
  mx = __reduce_max_sync(0xffffffffu, lane < nw ? s->part[lane][1] : 0u);
  sum = __reduce_add_sync(0xffffffffu, lane < nw ? s->part[lane][2] : 0u);
  __syncthreads();
}

// The bin of s->hist holding the kl-th largest key: s->prefix = bin, s->kgt
// = keys in the bins above it.  Warp 0 scans; ends with a block barrier.
__device__ __forceinline__ void pick_bin(int kl, SelectScratch* s);

// Histogram of the live keys (bin_of(key) != kNoBin for index < nl) and the
// bin holding the kl-th largest: s->prefix = bin, s->kgt = keys above it.
// Lanes sharing lane 0's bin add with one atomic (clustered scores would
// otherwise serialise on a few bins).
template <class BinOf>
__device__ __forceinline__ void hist_pick(const uint32_t (&r)[kKeysPerThread], int nj, int nl, int kl, BinOf bin_of,
                                          SelectScratch* s) {
  const int tid = threadIdx.x, lane = tid & 31;
  for (int i = tid; i < 256; i += blockDim.x) s->hist[i] = 0;
  if (tid == 0) s->ncand = 0;
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    if (j >= nj) break;  // uniform across the block
    const uint32_t bin = tid + j * kTopkThreads < nl ? bin_of(r[j]) : kNoBin;
    const uint32_t lead = __shfl_sync(0xffffffffu, bin, 0);
    const unsigned same = __ballot_sync(0xffffffffu, bin == lead);
    if (bin == lead) {
      if (lane == __ffs(same) - 1 && lead != kNoBin) atomicAdd(&s->hist[lead], (uint32_t)__popc(same));
    } else if (bin != kNoBin) {
      atomicAdd(&s->hist[bin], 1u);
    }
  }
  __syncthreads();
  pick_bin(kl, s);
}

__device__ __forceinline__ void pick_bin(int kl, SelectScratch* s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == 0) {
    // lane l owns bins [8l, 8l+8); find the bin of the kl-th largest from the top
    uint32_t h[8], tot = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      h[j] = s->hist[8 * lane + j];
      tot += h[j];
    }
    uint32_t incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_down_sync(0xffffffffu, incl, o);
      if (lane + o < 32) incl += v;
    }
    uint32_t run = incl - tot;
#pragma unroll
    for (int j = 7; j >= 0; --j) {
      if (run < (uint32_t)kl && run + h[j] >= (uint32_t)kl) {
        s->prefix = (uint32_t)(8 * lane + j);
        s->kgt = run;
      }
      run += h[j];
    }
  }
  __syncthreads();
}

// Copies the live keys of bin `bin` to cand (one atomic per warp and key slot;
// their order is irrelevant, only the threshold value is sought) and returns
// how many there are.
template <class BinOf>
__device__ __forceinline__ int gather_bin(const uint32_t (&r)[kKeysPerThread], int nj, int nl, uint32_t bin,
                                          BinOf bin_of, uint32_t* cand, SelectScratch* s) {
  const int tid = threadIdx.x, lane = tid & 31;
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    if (j >= nj) break;
    const bool hit = tid + j * kTopkThreads < nl && bin_of(r[j]) == bin;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (m) {
      uint32_t o = 0;
      if (lane == 0) o = atomicAdd(&s->ncand, (uint32_t)__popc(m));
      o = __shfl_sync(0xffffffffu, o, 0);
      if (hit) cand[o + __popc(m & ((1u << lane) - 1u))] = r[j];
    }
  }
  __syncthreads();
  return (int)s->ncand;
}

// Candidates of a bin few enough for a direct rank: thread t takes candidate
// t and counts the candidates above it and at or above it.
constexpr int kRankMax = 256;

// Finds the k-th largest of the n keys (1 <= k <= n <= kTopkMaxN, blockDim.x
// == kTopkThreads) held in registers, r[j] = key tid + j * kTopkThreads (0
// past n), and in shared memory (keys[i]), and leaves it in s->prefix; r is
// clobbered.  `cand` holds up to n keys.
__device__ void kth_key_select(uint32_t (&r)[kKeysPerThread], const uint32_t* keys, int n, int k, SelectScratch* s,
                               uint32_t* cand) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int nj = (n + kTopkThreads - 1) / kTopkThreads;
  // level 0 over the keys above the floor (the key of -inf: masked positions
  // and padding sit at or below it), binned by score value
  const uint32_t kfloor = float_key(-INFINITY);
  uint32_t lo = 0xffffffffu, hi = 0u, cnt = 0;
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    if (j >= nj) break;
    if (tid + j * kTopkThreads < n && r[j] > kfloor) {
      ++cnt;
      lo = min(lo, r[j]);
      hi = max(hi, r[j]);
    }
  }
  uint32_t mn, mx, n_live;
  block_minmax_sum(lo, hi, cnt, s, mn, mx, n_live);
  int nl = n, kl = k, nc = -1;
  uint32_t thr = 0;
  bool done = false;
  if (n_live >= (uint32_t)k) {
    const float vmin = key_float(mn), vmax = key_float(mx);
    if (mx == mn) {
      thr = mn;  // every live key is equal
      done = true;
    } else if (isfinite(vmin) && isfinite(vmax)) {
      const float scale = 255.99f / (vmax - vmin);
      auto vbin = [&](uint32_t key) -> uint32_t {
        if (key <= kfloor) return kNoBin;
        return min((uint32_t)((key_float(key) - vmin) * scale), 255u);
      };
      hist_pick(r, nj, nl, kl, vbin, s);
      const uint32_t bin = s->prefix;
      kl -= (int)s->kgt;
      nc = gather_bin(r, nj, nl, bin, vbin, cand, s);
    }
  }
  // otherwise (threshold at or below the floor, or non-finite scores) the
  // key levels below start from all keys
  for (int level = 0; level < 6 && !done; ++level) {
    if (nc >= 0 && nc <= kRankMax) {
      // the kl-th largest of the nc candidates: the value c with fewer than
      // kl candidates above it and at least kl at or above it (every thread
      // holding that value writes the same word)
      if (tid < nc) {
        const uint32_t c = cand[tid];
        uint32_t gt = 0, ge = 0;
        const int n4 = nc & ~3;
        for (int u = 0; u < n4; u += 4) {
          const uint4 v = *reinterpret_cast<const uint4*>(cand + u);
          gt += (v.x > c) + (v.y > c) + (v.z > c) + (v.w > c);
          ge += (v.x >= c) + (v.y >= c) + (v.z >= c) + (v.w >= c);
        }
        for (int u = n4; u < nc; ++u) {
          gt += cand[u] > c;
          ge += cand[u] >= c;
        }
        if (gt < (uint32_t)kl && (uint32_t)kl <= ge) s->prefix = c;
      }
      __syncthreads();
      thr = s->prefix;
      break;
    }
    if (nc >= 0) {
#pragma unroll
      for (int j = 0; j < kKeysPerThread; ++j) {
        const int i = tid + j * kTopkThreads;
        r[j] = i < nc ? cand[i] : 0u;
      }
      nl = nc;
      nj = (nc + kTopkThreads - 1) / kTopkThreads;
    }
    lo = 0xffffffffu;
    hi = 0u;
#pragma unroll
    for (int j = 0; j < kKeysPerThread; ++j) {
      if (j >= nj) break;
      if (tid + j * kTopkThreads < nl) {
        lo = min(lo, r[j]);
        hi = max(hi, r[j]);
      }
    }
    block_minmax_sum(lo, hi, 0u, s, mn, mx, cnt);  // also orders the reload before cand is rewritten
    const uint32_t range = mx - mn;
    if (range == 0) {
      thr = mn;
      break;
    }
    if (nl <= 32 * kKeysPerThread) {
      // few keys left: warp 0 bisects over their offsets above mn, two bits
      // per pass, counting with ballots (no block barrier per pass)
      if (warp == 0) {
        uint32_t c[kKeysPerThread];
#pragma unroll
        for (int j = 0; j < kKeysPerThread; ++j) {
          const int i = lane + 32 * j;
          c[j] = i < nl ? (nc >= 0 ? cand[i] : keys[i]) - mn : 0u;
        }
        const int ncj = (nl + 31) / 32;
        uint32_t pre = 0;
        for (int b2 = (32 - __clz(range) + 1) & ~1; b2 > 0; b2 -= 2) {
          const int sh = b2 - 2;
          const uint32_t p1 = pre | (1u << sh), p2 = pre | (2u << sh), p3 = pre | (3u << sh);
          uint32_t t1 = 0, t2 = 0, t3 = 0;
#pragma unroll
          for (int j = 0; j < kKeysPerThread; ++j) {
            if (j >= ncj) break;
            const bool ok = lane + 32 * j < nl;
            t1 += __popc(__ballot_sync(0xffffffffu, ok && c[j] >= p1));
            t2 += __popc(__ballot_sync(0xffffffffu, ok && c[j] >= p2));
            t3 += __popc(__ballot_sync(0xffffffffu, ok && c[j] >= p3));
          }
          pre = t3 >= (uint32_t)kl ? p3 : t2 >= (uint32_t)kl ? p2 : t1 >= (uint32_t)kl ? p1 : pre;
        }
        if (lane == 0) s->prefix = mn + pre;
      }
      __syncthreads();
      thr = s->prefix;
      break;
    }
    // key level: 256 bins over [mn, mx], each narrowing the range by 2^8
    const int shift = range < 256u ? 0 : 32 - __clz(range) - 8;
    const uint32_t mn0 = mn;
    auto kbin = [&](uint32_t key) -> uint32_t { return (key - mn0) >> shift; };
    hist_pick(r, nj, nl, kl, kbin, s);
    const uint32_t bin = s->prefix;
    kl -= (int)s->kgt;
    if (shift == 0) {
      thr = mn0 + bin;
      break;
    }
    nc = gather_bin(r, nj, nl, bin, kbin, cand, s);
  }
  __syncthreads();
  if (tid == 0) s->prefix = thr;
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

// Selects the k best of (keys[i], ids[i]) for i < n and writes them out, in
// ascending position order.  r holds the keys in registers (r[j] = key
// tid + j * kTopkThreads, 0 past n) for the select; keys[] holds them in
// shared memory for the compaction.
// mode_final: out index = id + win when the masked score >= -1000, else -1;
// otherwise the raw id is written (intermediate candidate lists).
// `scratch` (kScratchBytes) holds a level's survivors during the select and the
// (key, id) pairs of the optional descending sort afterwards.
__device__ void select_and_emit(uint32_t (&r)[kKeysPerThread], const uint32_t* keys, const int32_t* ids, int n,
                                int k, bool sort_desc, bool mode_final, int win, int32_t* out_idx, float* out_score,
                                uint8_t* scratch, SelectScratch* s) {
  kth_key_select(r, keys, n, k, s, reinterpret_cast<uint32_t*>(scratch));
  uint64_t* sort_buf = reinterpret_cast<uint64_t*>(scratch);
  const uint32_t thr = s->prefix;
  // Compaction: warp w walks positions [w * 32 * per, (w + 1) * 32 * per),
  // 32 consecutive ones per step (conflict-free shared reads); ballots give
  // each key's rank inside its warp, one scan over the 32 warp counts the
  // warps' offsets.  Keys above the threshold, then the lowest-position
  // keys equal to it, land in ascending position order.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int base = warp * 32 * per;
  uint32_t ca = 0, ce = 0;
#pragma unroll 4
  for (int j = 0; j < per; ++j) {
    const int i = base + 32 * j + lane;
    const uint32_t key = i < n ? keys[i] : 0u;
    ca += __popc(__ballot_sync(0xffffffffu, i < n && key > thr));
    ce += __popc(__ballot_sync(0xffffffffu, i < n && key == thr));
  }
  if (lane == 0) {
    s->warp_cnt[0][warp] = ca;
    s->warp_cnt[1][warp] = ce;
  }
  __syncthreads();
  if (warp == 0) {
    const uint32_t wa = lane < nw ? s->warp_cnt[0][lane] : 0, we = lane < nw ? s->warp_cnt[1][lane] : 0;
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
    if (lane == 31) s->kgt = xa;  // keys above the threshold, all warps
  }
  __syncthreads();
  uint32_t oa = s->warp_cnt[0][warp], oe = s->warp_cnt[1][warp];
  const int n_above = (int)s->kgt;  // < k by the choice of thr
  const int n_eq_take = k - n_above;
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll 4
  for (int j = 0; j < per; ++j) {
    const int i = base + 32 * j + lane;
    const uint32_t key = i < n ? keys[i] : 0u;
    const bool above = i < n && key > thr, eq = i < n && key == thr;
    const uint32_t ma = __ballot_sync(0xffffffffu, above), me = __ballot_sync(0xffffffffu, eq);
    int slot = -1;
    if (above) {
      slot = (int)(oa + __popc(ma & lt));
    } else if (eq) {
      const int re = (int)(oe + __popc(me & lt));
      if (re < n_eq_take) slot = n_above + re;
    }
    oa += __popc(ma);
    oe += __popc(me);
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
// With fq != null the score of each row's newest live entry, t = t_active - 1,
// is recomputed from the indexer inputs (fq [B, 64, 128], key rows fk + b *
// fk_bstride + t * 128, fw [B, 64]) instead of read from `score`: the key row
// may have been written after the score matrix was computed.
__global__ void __launch_bounds__(kTopkThreads) topk_chunk_kernel(
    const float* __restrict__ score, int64_t ld_score, const int32_t* __restrict__ t_active, int T, int chunk, int k,
    int win, int sort_desc, int mask_mode, int32_t* __restrict__ out_idx, float* __restrict__ out_score, int64_t ld_out,
    uint32_t* __restrict__ cand_key, int32_t* __restrict__ cand_id, const __nv_bfloat16* __restrict__ fq,
    const __nv_bfloat16* __restrict__ fk, int64_t fk_bstride, const float* __restrict__ fw) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ SelectScratch s;
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
  int32_t* ids = reinterpret_cast<int32_t*>(smem + kTopkMaxN * 4);
  uint8_t* scratch = smem + kTopkMaxN * 8;
  const int b = blockIdx.y, c = blockIdx.x, n_chunks = gridDim.x;
  const int t0 = c * chunk;
  const int n = min(T, t0 + chunk) - t0;
  pdl_wait();
  pdl_launch_dependents();
  const int ta = t_active[b];
  const float* row = score + int64_t(b) * ld_score + t0;
  const int tf = min(ta, T) - 1;  // the newest live entry
  const bool fix = fq != nullptr && tf >= t0 && tf < t0 + n;  // uniform across the CTA
  // every load of a thread in flight before any use (n <= 16 x 1024); the
  // keys stay in registers for the select and go to shared memory for the
  // compaction
  uint32_t r[kKeysPerThread];
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    const int i = threadIdx.x + j * kTopkThreads;
    r[j] = i < n ? __float_as_uint(__ldg(row + i)) : 0u;
  }
  float fix_score = 0.f;
  if (fix) {
    fix_score = indexer_row_score(fq + int64_t(b) * kRowHeads * kRowDim, fk + int64_t(b) * fk_bstride +
                                  int64_t(tf) * kRowDim, fw + int64_t(b) * kRowHeads, s.fix_dot);
  }
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    const int i = threadIdx.x + j * kTopkThreads;
    if (i < n) {
      const float v = (fix && t0 + i == tf) ? fix_score : __uint_as_float(r[j]);
      r[j] = float_key((t0 + i < ta) ? v : (mask_mode ? -INFINITY : __fsub_rn(v, 1.0e4f)));
      keys[i] = r[j];
    } else {
      r[j] = 0u;
    }
  }
  __syncthreads();
  if (n_chunks == 1) {
    select_and_emit(r, keys, nullptr, n, k, sort_desc != 0, true, win, out_idx + int64_t(b) * ld_out,
                    out_score ? out_score + int64_t(b) * ld_out : nullptr, scratch, &s);
    return;
  }
  // intermediate: ids are global positions
  const int kk = min(k, n);
  for (int i = threadIdx.x; i < n; i += blockDim.x) ids[i] = t0 + i;
  __syncthreads();
  const int64_t base = (int64_t(b) * n_chunks + c) * k;
  // write keys of the selected candidates: emit ids into cand_id, then keys
  select_and_emit(r, keys, ids, n, kk, false, false, 0, cand_id + base, nullptr, scratch, &s);
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
  uint8_t* scratch = smem + kTopkMaxN * 8;
  const int b = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  uint32_t r[kKeysPerThread];
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    const int i = threadIdx.x + j * kTopkThreads;
    r[j] = 0u;
    if (i < n_cand) {
      const int32_t id = cand_id[int64_t(b) * n_cand + i];
      uint32_t key;
      if (cand_key) key = cand_key[int64_t(b) * n_cand + i];
      else key = float_key(cand_score[int64_t(b) * n_cand + i]);
      ids[i] = id;
      r[j] = (id < 0) ? 0u : key;
      keys[i] = r[j];
    }
  }
  __syncthreads();
  select_and_emit(r, keys, ids, n_cand, k, sort_desc != 0, final_mode != 0, win, out_idx + int64_t(b) * ld_out,
                  out_score ? out_score + int64_t(b) * ld_out : nullptr, scratch, &s);
}

// One row per CTA with the final indices in position order (the decode
// step's case: T <= kTopkMaxN, no sort).  The same selection as
// topk_chunk_kernel with one chunk -- the threshold is the k-th largest key,
// ties go to the lowest positions -- in far fewer instructions (the select
// is issue-bound at one CTA per row):
//  * warp w holds positions [w * 32 * per, (w + 1) * 32 * per) in registers,
//    32 consecutive ones per register (coalesced loads; the compaction counts
//    and emits from registers);
//  * the first level's value bins (0..254 over [min, max] of the live keys)
//    are computed once, by a round-to-integer FMA (x + 1.5 * 2^23 holds
//    round(x) in its low mantissa bits; monotone in x, so the map stays
//    exact), and kept in shared memory for the gather;
//  * the candidates of the chosen bin are ranked by four threads each.
// Rows the first level cannot settle (fewer than k live keys, equal or
// non-finite extremes, more than kRankMax keys in the bin) take the general
// select.
constexpr uint32_t kRowNoBin = 255;         // masked keys: in no bin
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

__global__ void __launch_bounds__(kTopkThreads) topk_row_kernel(
    const float* __restrict__ score, int64_t ld_score, const int32_t* __restrict__ t_active, int n, int k, int win,
    int mask_mode, int32_t* __restrict__ out_idx, float* __restrict__ out_score, int64_t ld_out,
    const __nv_bfloat16* __restrict__ fq, const __nv_bfloat16* __restrict__ fk, int64_t fk_bstride,
    const float* __restrict__ fw) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ SelectScratch s;
  __shared__ uint32_t rank_gt[kRankMax], rank_ge[kRankMax];
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
  uint8_t* bins = smem + kTopkMaxN * 4;
  uint32_t* cand = reinterpret_cast<uint32_t*>(smem + kTopkMaxN * 8);
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + kTopkThreads - 1) / kTopkThreads;
  const int base = warp * 32 * per + lane;  // r[j] holds position base + 32 j
  if (tid < 256) s.hist[tid] = 0;
  if (tid < kRankMax) {
    rank_gt[tid] = 0;
    rank_ge[tid] = 0;
  }
  if (tid == 0) s.ncand = 0;
  pdl_wait();
  pdl_launch_dependents();
  const int ta = t_active[b];
  const float* row = score + int64_t(b) * ld_score;
  const int tf = min(ta, n) - 1;  // the newest live entry
  const bool fix = fq != nullptr && tf >= 0;
  uint32_t r[kKeysPerThread];
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    const int i = base + 32 * j;
    r[j] = (j < per && i < n) ? __float_as_uint(__ldg(row + i)) : 0u;
  }
  float fix_score = 0.f;
  if (fix) {
    fix_score = indexer_row_score(fq + int64_t(b) * kRowHeads * kRowDim, fk + int64_t(b) * fk_bstride +
                                  int64_t(tf) * kRowDim, fw + int64_t(b) * kRowHeads, s.fix_dot);
  }
  const uint32_t kfloor = float_key(-INFINITY);
  uint32_t lo = 0xffffffffu, hi = 0u, cnt = 0;
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    if (j >= per) break;
    const int i = base + 32 * j;
    if (i < n) {
      const float v = (fix && i == tf) ? fix_score : __uint_as_float(r[j]);
      const uint32_t key = float_key(i < ta ? v : (mask_mode ? -INFINITY : __fsub_rn(v, 1.0e4f)));
      r[j] = key;
      keys[i] = key;
      if (key > kfloor) {
        ++cnt;
        lo = min(lo, key);
        hi = max(hi, key);
      }
    }
  }
  uint32_t mn, mx, n_live;
  block_minmax_sum(lo, hi, cnt, &s, mn, mx, n_live);
  const float vmin = key_float(mn), vmax = key_float(mx);
  const float scale = 254.99f / (vmax - vmin);
  // uniform across the block: mn, mx, n_live and later s.ncand are shared
  bool fast = n_live >= uint32_t(k) && mx != mn && isfinite(vmin) && isfinite(vmax) && isfinite(scale) &&
              scale > 0.f;
  uint32_t thr = 0;
  if (fast) {
#pragma unroll
    for (int j = 0; j < kKeysPerThread; ++j) {
      if (j >= per) break;
      const int i = base + 32 * j;
      uint32_t bin = kRowNoBin;
      if (i < n && r[j] > kfloor) {
        const float d = key_float(r[j]) - vmin;
        bin = min(__float_as_uint(fmaf(d, scale, kRoundMagic)) - __float_as_uint(kRoundMagic), 254u);
      }
      if (i < n) bins[i] = uint8_t(bin);
      const uint32_t lead = __shfl_sync(0xffffffffu, bin, 0);
      const unsigned same = __ballot_sync(0xffffffffu, bin == lead);
      if (bin == lead) {
        if (lane == __ffs(same) - 1 && lead != kRowNoBin) atomicAdd(&s.hist[lead], uint32_t(__popc(same)));
      } else if (bin != kRowNoBin) {
        atomicAdd(&s.hist[bin], 1u);
      }
    }
    __syncthreads();
    pick_bin(k, &s);
    const uint32_t bin = s.prefix;
    const uint32_t kl = uint32_t(k) - s.kgt;
#pragma unroll
    for (int j = 0; j < kKeysPerThread; ++j) {
      if (j >= per) break;
      const int i = base + 32 * j;
      const bool hit = i < n && bins[i] == bin;
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      if (m) {
        uint32_t o = 0;
        if (lane == 0) o = atomicAdd(&s.ncand, uint32_t(__popc(m)));
        o = __shfl_sync(0xffffffffu, o, 0);
        if (hit) cand[o + __popc(m & ((1u << lane) - 1u))] = r[j];
      }
    }
    __syncthreads();
    const int nc = int(s.ncand);
    if (nc <= kRankMax) {
      // the kl-th largest candidate c: fewer than kl candidates above it and
      // at least kl at or above it; thread t counts candidate t % 256 against
      // a quarter of the list
      const int ci = tid & (kRankMax - 1), qt = tid >> 8;
      if (ci < nc) {
        const uint32_t c = cand[ci];
        const int u0 = (nc * qt) >> 2, u1 = (nc * (qt + 1)) >> 2;
        uint32_t gt = 0, ge = 0;
        for (int u = u0; u < u1; ++u) {
          const uint32_t x = cand[u];
          gt += x > c;
          ge += x >= c;
        }
        if (u1 > u0) {
          atomicAdd(&rank_gt[ci], gt);
          atomicAdd(&rank_ge[ci], ge);
        }
      }
      __syncthreads();
      if (tid < nc && rank_gt[tid] < kl && kl <= rank_ge[tid]) s.prefix = cand[tid];
      __syncthreads();
      thr = s.prefix;
    } else {
      fast = false;
    }
  }
  if (!fast) {
    // the general select, over the strided register layout it expects
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kKeysPerThread; ++j) {
      const int i = tid + j * kTopkThreads;
      r[j] = i < n ? keys[i] : 0u;
    }
    kth_key_select(r, keys, n, k, &s, cand);
    thr = s.prefix;
#pragma unroll
    for (int j = 0; j < kKeysPerThread; ++j) {
      const int i = base + 32 * j;
      r[j] = (j < per && i < n) ? keys[i] : 0u;
    }
  }
  // compaction: keys above thr, then the lowest-position keys equal to it,
  // in position order (ballot ranks inside each warp, one scan over the
  // warps' counts)
  uint32_t ca = 0, ce = 0;
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    if (j >= per) break;
    const bool valid = base + 32 * j < n;
    ca += __popc(__ballot_sync(0xffffffffu, valid && r[j] > thr));
    ce += __popc(__ballot_sync(0xffffffffu, valid && r[j] == thr));
  }
  if (lane == 0) {
    s.warp_cnt[0][warp] = ca;
    s.warp_cnt[1][warp] = ce;
  }
  __syncthreads();
  if (warp == 0) {
    const uint32_t wa = s.warp_cnt[0][lane], we = s.warp_cnt[1][lane];
    uint32_t xa = wa, xe = we;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t va = __shfl_up_sync(0xffffffffu, xa, o), ve = __shfl_up_sync(0xffffffffu, xe, o);
      if (lane >= o) {
        xa += va;
        xe += ve;
      }
    }
    s.warp_cnt[0][lane] = xa - wa;
    s.warp_cnt[1][lane] = xe - we;
    if (lane == 31) s.kgt = xa;  // keys above the threshold, all warps
  }
  __syncthreads();
  uint32_t oa = s.warp_cnt[0][warp], oe = s.warp_cnt[1][warp];
  const int n_above = int(s.kgt);  // < k by the choice of thr
  const int n_eq_take = k - n_above;
  const uint32_t lt = (1u << lane) - 1u;
  int32_t* orow = out_idx + int64_t(b) * ld_out;
  float* srow = out_score ? out_score + int64_t(b) * ld_out : nullptr;
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    if (j >= per) break;
    const int i = base + 32 * j;
    const bool valid = i < n;
    const bool above = valid && r[j] > thr, eq = valid && r[j] == thr;
    const uint32_t ma = __ballot_sync(0xffffffffu, above), me = __ballot_sync(0xffffffffu, eq);
    int slot = -1;
    if (above) {
      slot = int(oa + __popc(ma & lt));
    } else if (eq) {
      const int re = int(oe + __popc(me & lt));
      if (re < n_eq_take) slot = n_above + re;
    }
    oa += __popc(ma);
    oe += __popc(me);
    if (slot >= 0) {
      const float f = key_float(r[j]);
      orow[slot] = f >= -1000.0f ? i + win : -1;
      if (srow) srow[slot] = f;
    }
  }
}

// ---------------------------------------------------------------------------
// One row per 2-CTA cluster (the decode step's case with few rows: 2 B CTAs
// fit the SMs).  CTA c of the pair takes positions [c * half, ...) of the
// row, in the warp-contiguous register layout of topk_row_kernel, so each
// CTA bins, gathers and emits half the keys; the two exchange only small
// values through distributed shared memory: (min, max, live count), the
// first level's 255-bin histogram, the threshold bin's keys (at most
// kRankMax in all) and, for the compaction, their counts of keys above and
// equal to the threshold.  Both CTAs then hold the same histogram and the
// same survivors, find the same threshold, and write their own keys'
// slots - the lower half's first: the same output as topk_row_kernel.
// Rows the first level cannot settle take the general select over the whole
// row in both CTAs.
struct PairExchange {
  uint64_t bar[4];             // arrivals of the peer's values: mm, hist, cand + ncand, tot
  uint32_t mm[3];              // the peer's (min, max, live count)
  uint32_t ncand;              // the peer's keys in the threshold bin
  uint32_t tot[2];             // the peer's keys above / equal to the threshold
  uint32_t hist[256];          // the peer's first-level histogram
  uint32_t cand[kRankMax];     // the peer's keys in the threshold bin
};

__device__ __forceinline__ void cl_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cl_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// One value into the peer CTA's copy of `field`, counted on the peer's copy
// of mbarrier `bar` (st.async ... complete_tx): the receiver waits for
// exactly the bytes it expects, and neither side stops at a cluster-wide
// barrier, whose release fence stalled every exchange (ncu: membar 1.5
// stall cycles per issued instruction with four cluster barriers).
__device__ __forceinline__ void px_send(const void* field, uint32_t rank, uint32_t v, const uint64_t* bar) {
  uint32_t dst, rbar;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst) : "r"(smem_u32(field)), "r"(rank));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(smem_u32(bar)), "r"(rank));
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(dst), "r"(v),
               "r"(rbar)
               : "memory");
}
// bounded wait for the peer's values (phase 0: each barrier is used once);
// past about a second it gives up rather than hang
__device__ __forceinline__ void px_wait(const uint64_t* bar) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  uint32_t ok = 0;
  do {
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(a)
        : "memory");
  } while (!ok && clock64() - t0 < 2000000000LL);
}

__global__ void __launch_bounds__(kTopkThreads) topk_pair_kernel(
    const float* __restrict__ score, int64_t ld_score, const int32_t* __restrict__ t_active, int n, int k, int win,
    int mask_mode, int32_t* __restrict__ out_idx, float* __restrict__ out_score, int64_t ld_out) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ SelectScratch s;
  __shared__ PairExchange px;
  __shared__ uint32_t rank_gt[kRankMax], rank_ge[kRankMax];
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem);  // this CTA's keys by local position; the whole row on fallback
  uint8_t* bins = smem + kTopkMaxN * 4;
  uint32_t* cand = reinterpret_cast<uint32_t*>(smem + kTopkMaxN * 8);
  const int c = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t peer = uint32_t(c ^ 1);
  const int half = min(n, (((n + 1) >> 1) + 31) & ~31);
  const int p0 = c ? half : 0, cnt_pos = c ? n - half : half;  // this CTA's positions [p0, p0 + cnt_pos)
  const int per = (cnt_pos + kTopkThreads - 1) / kTopkThreads;
  const int base = warp * 32 * per + lane;  // local position of r[j]: base + 32 j
  if (tid < 256) s.hist[tid] = 0;
  if (tid < kRankMax) {
    rank_gt[tid] = 0;
    rank_ge[tid] = 0;
  }
  if (tid == 0) {
    s.ncand = 0;
    const uint32_t bytes[4] = {3 * 4, 256 * 4, 4 + kRankMax * 4, 2 * 4};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&px.bar[i])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i)
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&px.bar[i])), "r"(bytes[i])
                   : "memory");
  }
  // both CTAs have started (and set up their barriers) before either
  // writes the other's shared memory
  cl_arrive();
  pdl_wait();
  pdl_launch_dependents();
  const int ta = t_active[b];
  const float* row = score + int64_t(b) * ld_score;
  uint32_t r[kKeysPerThread];
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    const int i = base + 32 * j;
    r[j] = (j < per && i < cnt_pos) ? __float_as_uint(__ldg(row + p0 + i)) : 0u;
  }
  const uint32_t kfloor = float_key(-INFINITY);
  auto mask_key = [&](int pos, float v) {
    return float_key(pos < ta ? v : (mask_mode ? -INFINITY : __fsub_rn(v, 1.0e4f)));
  };
  uint32_t lo = 0xffffffffu, hi = 0u, cnt = 0;
#pragma unroll
  for (int j = 0; j < kKeysPerThread; ++j) {
    if (j >= per) break;
    const int i = base + 32 * j;
    if (i < cnt_pos) {
      const uint32_t key = mask_key(p0 + i, __uint_as_float(r[j]));
      r[j] = key;
      keys[i] = key;
      if (key > kfloor) {
        ++cnt;
        lo = min(lo, key);
        hi = max(hi, key);
      }
    }
  }
  uint32_t mn, mx, n_live;
  block_minmax_sum(lo, hi, cnt, &s, mn, mx, n_live);
  cl_wait();
  if (tid == 0) {
    px_send(&px.mm[0], peer, mn, &px.bar[0]);
    px_send(&px.mm[1], peer, mx, &px.bar[0]);
    px_send(&px.mm[2], peer, n_live, &px.bar[0]);
  }
  px_wait(&px.bar[0]);
  mn = min(mn, px.mm[0]);
  mx = max(mx, px.mm[1]);
  n_live += px.mm[2];
  const float vmin = key_float(mn), vmax = key_float(mx);
  const float scale = 254.99f / (vmax - vmin);
  // uniform across both CTAs: every input to it was exchanged
  bool fast = n_live >= uint32_t(k) && mx != mn && isfinite(vmin) && isfinite(vmax) && isfinite(scale) &&
              scale > 0.f;
  uint32_t thr = 0;
  // After the loads, the per-key loops are not unrolled and read the keys
  // back from shared memory: in the decode step this kernel starts on SMs
  // whose instruction cache holds the indexer's code, and unrolled copies
  // cost more in instruction fetch than they save in issue (same box, A/B:
  // 75.8 against 77.5 us per layer, although the kernel timed back to back
  // with itself, warm, runs 10.7 against 9.5 us).
  if (fast) {
#pragma unroll 1
    for (int j = 0; j < per; ++j) {
      const int i = base + 32 * j;
      uint32_t bin = kRowNoBin;
      const uint32_t x = i < cnt_pos ? keys[i] : 0u;
      if (i < cnt_pos && x > kfloor) {
        const float d = key_float(x) - vmin;
        bin = min(__float_as_uint(fmaf(d, scale, kRoundMagic)) - __float_as_uint(kRoundMagic), 254u);
      }
      if (i < cnt_pos) bins[i] = uint8_t(bin);
      const uint32_t lead = __shfl_sync(0xffffffffu, bin, 0);
      const unsigned same = __ballot_sync(0xffffffffu, bin == lead);
      if (bin == lead) {
        if (lane == __ffs(same) - 1 && lead != kRowNoBin) atomicAdd(&s.hist[lead], uint32_t(__popc(same)));
      } else if (bin != kRowNoBin) {
        atomicAdd(&s.hist[bin], 1u);
      }
    }
    __syncthreads();
    if (tid < 256) px_send(&px.hist[tid], peer, s.hist[tid], &px.bar[1]);
    px_wait(&px.bar[1]);
    if (tid < 256) s.hist[tid] += px.hist[tid];
    __syncthreads();
    pick_bin(k, &s);
    const uint32_t bin = s.prefix;
    const uint32_t kl = uint32_t(k) - s.kgt;
#pragma unroll 1
    for (int j = 0; j < per; ++j) {
      const int i = base + 32 * j;
      const bool hit = i < cnt_pos && bins[i] == bin;
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      if (m) {
        uint32_t o = 0;
        if (lane == 0) o = atomicAdd(&s.ncand, uint32_t(__popc(m)));
        o = __shfl_sync(0xffffffffu, o, 0);
        if (hit) cand[o + __popc(m & ((1u << lane) - 1u))] = keys[i];
      }
    }
    __syncthreads();
    const int nc_own = int(s.ncand);
    if (tid == 0) px_send(&px.ncand, peer, uint32_t(nc_own), &px.bar[2]);
    // a fixed kRankMax entries (the receiver's byte count); those past the
    // count are not read
    if (tid < kRankMax) px_send(&px.cand[tid], peer, cand[tid], &px.bar[2]);
    px_wait(&px.bar[2]);
    __syncthreads();  // every thread has sent its cand entry before any is overwritten below
    const int nc_peer = int(px.ncand);
    const int nc = nc_own + nc_peer;
    if (nc_own <= kRankMax && nc_peer <= kRankMax && nc <= kRankMax) {
      // the union of both halves' survivors (same multiset on both CTAs)
      if (tid < nc_peer) cand[nc_own + tid] = px.cand[tid];
      __syncthreads();
      const int ci = tid & (kRankMax - 1), qt = tid / kRankMax;
      constexpr int kParts = kTopkThreads / kRankMax;
      if (ci < nc) {
        const uint32_t cv = cand[ci];
        const int u0 = (nc * qt) / kParts, u1 = (nc * (qt + 1)) / kParts;
        uint32_t gt = 0, ge = 0;
        for (int u = u0; u < u1; ++u) {
          const uint32_t x = cand[u];
          gt += x > cv;
          ge += x >= cv;
        }
        if (u1 > u0) {
          atomicAdd(&rank_gt[ci], gt);
          atomicAdd(&rank_ge[ci], ge);
        }
      }
      __syncthreads();
      if (tid < nc && rank_gt[tid] < kl && kl <= rank_ge[tid]) s.prefix = cand[tid];
      __syncthreads();
      thr = s.prefix;
    } else {
      fast = false;
    }
  }
  if (!fast) {
    // the general select over the whole row, in both CTAs
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kKeysPerThread; ++j) {
      const int i = tid + j * kTopkThreads;
      r[j] = i < n ? mask_key(i, __ldg(row + i)) : 0u;
      if (i < n) keys[i] = r[j];
    }
    __syncthreads();
    kth_key_select(r, keys, n, k, &s, cand);
    thr = s.prefix;
  }
  // compaction: this CTA's keys above thr, then the lowest-position keys
  // equal to it; the lower half's counts come first
  uint32_t ca = 0, ce = 0;
  // this CTA's keys by local position (the general select left the whole
  // row in shared memory)
  const uint32_t* lkeys = keys + (fast ? 0 : p0);
#pragma unroll 1
  for (int j = 0; j < per; ++j) {
    const bool valid = base + 32 * j < cnt_pos;
    const uint32_t x = valid ? lkeys[base + 32 * j] : 0u;
    ca += __popc(__ballot_sync(0xffffffffu, valid && x > thr));
    ce += __popc(__ballot_sync(0xffffffffu, valid && x == thr));
  }
  if (lane == 0) {
    s.warp_cnt[0][warp] = ca;
    s.warp_cnt[1][warp] = ce;
  }
  __syncthreads();
  if (warp == 0) {
    const uint32_t wa = s.warp_cnt[0][lane], we = s.warp_cnt[1][lane];
    uint32_t xa = wa, xe = we;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t va = __shfl_up_sync(0xffffffffu, xa, o), ve = __shfl_up_sync(0xffffffffu, xe, o);
      if (lane >= o) {
        xa += va;
        xe += ve;
      }
    }
    s.warp_cnt[0][lane] = xa - wa;
    s.warp_cnt[1][lane] = xe - we;
    if (lane == 31) {
      px_send(&px.tot[0], peer, xa, &px.bar[3]);
      px_send(&px.tot[1], peer, xe, &px.bar[3]);
      s.part[0][0] = xa;
      s.part[0][1] = xe;
    }
  }
  __syncthreads();
  px_wait(&px.bar[3]);
  const uint32_t a0 = c ? px.tot[0] : s.part[0][0], a1 = c ? s.part[0][0] : px.tot[0];
  const uint32_t e0 = c ? px.tot[1] : 0u;
  const int n_above = int(a0 + a1);  // < k by the choice of thr
  const int n_eq_take = k - n_above;
  uint32_t oa = s.warp_cnt[0][warp] + (c ? a0 : 0u), oe = s.warp_cnt[1][warp] + e0;
  const uint32_t lt = (1u << lane) - 1u;
  int32_t* orow = out_idx + int64_t(b) * ld_out;
  float* srow = out_score ? out_score + int64_t(b) * ld_out : nullptr;
#pragma unroll 1
  for (int j = 0; j < per; ++j) {
    const int i = base + 32 * j;
    const bool valid = i < cnt_pos;
    const uint32_t x = valid ? lkeys[i] : 0u;
    const bool above = valid && x > thr, eq = valid && x == thr;
    const uint32_t ma = __ballot_sync(0xffffffffu, above), me = __ballot_sync(0xffffffffu, eq);
    int slot = -1;
    if (above) {
      slot = int(oa + __popc(ma & lt));
    } else if (eq) {
      const int re = int(oe + __popc(me & lt));
      if (re < n_eq_take) slot = n_above + re;
    }
    oa += __popc(ma);
    oe += __popc(me);
    if (slot >= 0) {
      const float f = key_float(x);
      orow[slot] = f >= -1000.0f ? p0 + i + win : -1;
      if (srow) srow[slot] = f;
    }
  }
  // neither CTA exits while a value it sent may still be in flight to the
  // other (no data: a relaxed arrive)
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  cl_wait();
}

__global__ void window_indices_kernel(const int32_t* __restrict__ pos, int32_t* __restrict__ idx, int64_t ld,
                                      int B, int win) {
  pdl_wait();
  pdl_launch_dependents();
  window_indices_row(pos, idx, ld, win, blockIdx.x);
}

}  // namespace dsa

using namespace dsa;

namespace {
// keys | ids | scratch
int chunk_smem() { return kTopkMaxN * 8 + kScratchBytes; }
int merge_smem() { return kTopkMaxN * 8 + kScratchBytes; }
}  // namespace

extern "C" int dsa_window_indices(const int32_t* pos, int32_t* idx, int64_t ld_idx, int B, int win,
                                  dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(pos && idx, "window_indices: null pointer");
  DSA_CHECK_ARG(B >= 0 && win > 0 && ld_idx >= win, "window_indices: bad B/win/ld");
  if (B == 0) return DSA_OK;
  launch_pdl(window_indices_kernel, dim3(B), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream), pos, idx, ld_idx,
             B, win);
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
                       void* ws, size_t ws_bytes, cudaStream_t st, const __nv_bfloat16* fq = nullptr,
                       const __nv_bfloat16* fk = nullptr, int64_t fk_bstride = 0, const float* fw = nullptr) {
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
    cudaFuncSetAttribute(topk_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, chunk_smem());
    cudaFuncSetAttribute(topk_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, chunk_smem());
    attr_dev = dev;
  }
  if (T <= kTopkMaxN && !sort_desc && fq == nullptr && 2 * B <= num_sms()) {
    // few rows: two CTAs per row (a cluster pair)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, B);
    cfg.blockDim = dim3(kTopkThreads);
    cfg.dynamicSmemBytes = chunk_smem();
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, topk_pair_kernel, score, ld_score, t_active, T, k, win, mask_mode, out_idx, out_score,
                       ld_out);
    DSA_CHECK_LAUNCH("indexer_topk");
    return DSA_OK;
  }
  if (T <= kTopkMaxN && !sort_desc) {
    launch_pdl(topk_row_kernel, dim3(B), dim3(kTopkThreads), chunk_smem(), st, score, ld_score, t_active, T, k, win,
               mask_mode, out_idx, out_score, ld_out, fq, fk, fk_bstride, fw);
    DSA_CHECK_LAUNCH("indexer_topk");
    return DSA_OK;
  }
  if (T <= kTopkMaxN) {
    launch_pdl(topk_chunk_kernel, dim3(1, B), dim3(kTopkThreads), chunk_smem(), st, score, ld_score, t_active, T, T,
               k, win, sort_desc, mask_mode, out_idx, out_score, ld_out, (uint32_t*)nullptr, (int32_t*)nullptr, fq, fk,
               fk_bstride, fw);
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
  launch_pdl(topk_chunk_kernel, dim3(n_chunks, B), dim3(kTopkThreads), chunk_smem(), st, score, ld_score, t_active, T,
             (int)kTopkMaxN, k, win, 0, mask_mode, (int32_t*)nullptr, (float*)nullptr, (int64_t)0, ck, ci, fq, fk,
             fk_bstride, fw);
  DSA_CHECK_LAUNCH("indexer_topk(chunks)");
  launch_pdl(topk_merge_kernel, dim3(B), dim3(kTopkThreads), merge_smem(), st, (const uint32_t*)ck,
             (const float*)nullptr, (const int32_t*)ci, n_chunks * k, k, win, sort_desc, 1, out_idx, out_score, ld_out);
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

extern "C" int dsa_indexer_topk_newest(const float* score, int64_t ld_score, const int32_t* t_active,
                                       int32_t* out_idx, float* out_score, int64_t ld_out, int B, int T, int k,
                                       int win, int sort_desc, int mask_mode, const void* q, const void* k_cache,
                                       int64_t k_bstride, const float* w, void* workspace, size_t workspace_bytes,
                                       dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(q && k_cache && w, "indexer_topk_newest: null q / k_cache / w");
  DSA_CHECK_ARG(aligned(q, 16) && aligned(k_cache, 16) && k_bstride % 8 == 0 && k_bstride >= int64_t(T) * kRowDim,
                "indexer_topk_newest: q / k_cache must be 16-byte aligned and k_bstride >= T * 128, a multiple of 8");
  return topk_launch(score, ld_score, t_active, out_idx, out_score, ld_out, B, T, k, win, sort_desc, mask_mode,
                     workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream),
                     static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k_cache), k_bstride, w);
}

extern "C" int dsa_indexer_topk_ws(const float* score, int64_t ld_score, const int32_t* t_active, int32_t* out_idx,
                                   float* out_score, int64_t ld_out, int B, int T, int k, int win, int sort_desc,
                                   int mask_mode, void* workspace, size_t workspace_bytes, dsa_stream_t stream) {
  clear_error();
  return topk_launch(score, ld_score, t_active, out_idx, out_score, ld_out, B, T, k, win, sort_desc, mask_mode,
                     workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

__global__ void advance_positions_kernel(int32_t* pos, int32_t* t_active, int B, int ratio, int step) {
  pdl_wait();
  pdl_launch_dependents();
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
  launch_pdl(advance_positions_kernel, dim3((B + 127) / 128), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream),
             pos, t_active, B, ratio, step);
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
