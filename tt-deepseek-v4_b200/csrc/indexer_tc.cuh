// attn.topk indexer score on the tcgen05 tensor cores.
//
// s[b, t] = sum_h w[b, h] * relu(q[b, h, :] . k[b, t, :])   (H = 64, Di = 128)
//
// Persistent kernel: one CTA per SM walks a contiguous range of the live
// (sequence, 128-key tile) work items -- tiles below the sequence's t_valid;
// each CTA first builds the per-sequence prefix of live tiles in shared
// memory and takes an equal share of them (a split over all allocated tiles
// left CTAs whose range missed the dead tails with ~12 % more work at
// t_valid = 8192 of T = 9216).  Roles:
//   warp 0      TMA producer: per item a [128 keys x 128] tile of the key
//               cache and the sequence's [64 x 128] q (two 128-B-swizzled
//               k-blocks each) into a 4-stage ring (48 KB per stage).
//   warp 1      MMA issuer: S^T = K_tile . Q^T, M = 128 keys, N = 64 heads,
//               K = 128 (8 x K16), into one of two TMEM accumulators.
//   warps 2-5   epilogue: thread = key row (TMEM lane), 64 head scores in
//               registers -> sum_h w_h relu(s_h) -> one fp32 score, coalesced.
// Dynamic split (kDyn, a caller's counters): each CTA keeps a contiguous
// four fifths of an even share (its first items still requested before the
// dependency wait when keys_ready) and then claims items one at a time from
// a global counter, one claim in flight ahead, so CTAs that start late -- on
// SMs the previous kernel still held -- take fewer and the CTAs finish
// together (79.1 against 80.5 us per decode layer at config 2, A/B; claiming
// all but the first NS items lost 2.6 us: claim latency on the item path and
// the epilogue reloading a sequence's head weights at almost every item).  The producer publishes every item it takes
// (sequence and first key, or an end marker) in an 8-entry ring guarded by
// mbarriers, which the MMA and epilogue warps follow; at most 6 items are in
// flight between the producer and the epilogue, so 8 entries never wrap onto
// an unread one.  The last CTA to finish claiming resets the counters.
// The [H, T] score matrix never exists; HBM traffic is the key stream
// (256 B per key) plus 4 B of score per key.
#pragma once

#include "common.cuh"
#include "tc05.cuh"
#include "tma.cuh"

namespace dsa {
namespace idxtc {

constexpr int H = 64;
constexpr int DI = 128;
constexpr int TILE = 128;         // keys per work item
constexpr int NS = 4;
constexpr int THREADS = 192;
constexpr int kKeyBytes = TILE * DI * 2;   // 32 KB: 2 k-blocks of [128 rows x 128 B]
constexpr int kQBytes = H * DI * 2;        // 16 KB: 2 k-blocks of [64 rows x 128 B]
constexpr int kStageBytes = kKeyBytes + kQBytes;
constexpr int kOffAux = NS * kStageBytes;
constexpr int kMaxSeqBalanced = 4096;      // sequences the live-tile prefix holds
constexpr int kAuxBytes = 512;
constexpr int kOffPre = kOffAux + kAuxBytes;
constexpr int kInfo = 8;                   // dynamic split: published items ring
constexpr int kSmemBytes = kOffPre + (kMaxSeqBalanced + 1) * 4 + 1024;
constexpr uint32_t kTmemCols = 128;        // 2 accumulators x 64 columns
constexpr uint32_t kIdesc = tc::idesc_bf16(128, 64, false, false);

struct Aux {
  uint64_t full[NS];
  uint64_t empty[NS];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t info_full[kInfo];
  int info_b[kInfo], info_t0[kInfo];  // sequence (-1: no more items) and first key
  uint32_t tmem_base;
  int wsum[THREADS / 32];
};
static_assert(sizeof(Aux) <= kAuxBytes, "aux block");

struct Args {
  const float* w;
  float* score;
  const int32_t* t_valid;
  int32_t* status;
  long long wait_limit;   // spin budget of every bounded wait, SM cycles
  int B, T, tiles_per_seq, items_per_cta;
  int balanced;           // B <= kMaxSeqBalanced: split the live tiles evenly (items_per_cta unused)
  // The key cache and t_valid were complete before the previous kernel on
  // the stream started (keys of earlier decode steps): the first NS key
  // tiles are requested before the programmatic-dependent-launch wait, so
  // their latency overlaps the previous kernel's tail; q and w are read
  // after the wait.
  int keys_ready;
  int64_t ld_score;
  int64_t k_row_stride;   // rows between consecutive sequences in the key map
  uint32_t* dyn;          // dynamic split: [claimed items, CTAs done], zero on entry and on exit
};

__device__ __forceinline__ int seq_limit(const Args& a, int b) {
  return a.t_valid ? min(a.T, max(0, a.t_valid[b])) : a.T;
}

__device__ __forceinline__ bool item_live(const Args& a, int item, int& b, int& t0, int& t_lim) {
  b = item / a.tiles_per_seq;
  t0 = (item - b * a.tiles_per_seq) * TILE;
  t_lim = seq_limit(a, b);
  return t0 < t_lim;
}

// This CTA's work items in order.  Balanced: live items [l, l_end) of the
// live-tile prefix pre[] (pre[b] = live tiles of the sequences before b);
// otherwise the item range [item, i_end), dead items skipped.
struct ItemWalk {
  const Args* a;
  const int* pre;
  int l, l_end, b, tile;
  int item, i_end;
  __device__ bool next(int& b_, int& t0, int& t_lim) {
    if (pre) {
      if (l >= l_end) return false;
      b_ = b;
      t0 = tile * TILE;
      t_lim = seq_limit(*a, b);
      ++l;
      if (++tile >= pre[b + 1] - pre[b]) {
        tile = 0;
        do {
          ++b;
        } while (b < a->B && pre[b + 1] == pre[b]);
      }
      return true;
    }
    while (item < i_end) {
      if (item_live(*a, item++, b_, t0, t_lim)) return true;
    }
    return false;
  }
};

template <bool kDyn>
__global__ void __launch_bounds__(THREADS, 1) indexer_score_tc_kernel(const Args a,
                                                                      const __grid_constant__ CUtensorMap tm_k,
                                                                      const __grid_constant__ CUtensorMap tm_q) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Aux* aux = reinterpret_cast<Aux*>(smem + kOffAux);
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 1) {
    tc::tmem_alloc(smem_u32(&aux->tmem_base), kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(smem_u32(&aux->full[s]), 1);
      tc::mbar_init(smem_u32(&aux->empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(smem_u32(&aux->acc_full[s]), 1);
      tc::mbar_init(smem_u32(&aux->acc_empty[s]), 4);
    }
    for (int s = 0; s < kInfo; ++s) tc::mbar_init(smem_u32(&aux->info_full[s]), 1);
    tc::mbar_fence_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = aux->tmem_base;

  ItemWalk walk{};
  walk.a = &a;
  int total_live = 0;
  auto build_walk = [&]() {
    if (a.balanced) {
      // live tiles per sequence -> exclusive prefix (one block scan)
      int* pre = reinterpret_cast<int*>(smem + kOffPre);
      auto live = [&](int b) { return (seq_limit(a, b) + TILE - 1) / TILE; };
      const int per = (a.B + THREADS - 1) / THREADS;
      const int b0 = min(a.B, tid * per), b1 = min(a.B, b0 + per);
      int loc = 0;
      for (int b = b0; b < b1; ++b) loc += live(b);
      int inc = loc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
      }
      if (lane == 31) aux->wsum[warp] = inc;
      __syncthreads();
      int run = inc - loc;
      for (int w = 0; w < warp; ++w) run += aux->wsum[w];
      for (int b = b0; b < b1; ++b) {
        pre[b] = run;
        run += live(b);
      }
      if (tid == THREADS - 1) pre[a.B] = run;
      __syncthreads();
      total_live = pre[a.B];
      // dynamic split: about four fifths of an even share are each CTA's
      // own (contiguous, so the epilogue's head weights change rarely); the
      // rest is claimed
      const int even = (total_live + gridDim.x - 1) / gridDim.x;
      const int share = kDyn ? max(NS, even * 4 / 5) : even;
      walk.pre = pre;
      walk.l = min(total_live, int(blockIdx.x) * share);
      walk.l_end = min(total_live, walk.l + share);
      if (walk.l < walk.l_end) {
        // the sequence holding live item l: the last b with pre[b] <= l
        int lo = 0, hi = a.B - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (pre[mid] <= walk.l) lo = mid;
          else hi = mid - 1;
        }
        walk.b = lo;
        walk.tile = walk.l - pre[lo];
      }
    } else {
      walk.i_end = min(a.B * a.tiles_per_seq, int(blockIdx.x + 1) * a.items_per_cta);
      walk.item = int(blockIdx.x) * a.items_per_cta;
    }
  };

  // keys_ready: the work split (from t_valid) and the first NS key tiles
  // before the wait; each stage's q follows after it on the same barrier
  int npre = 0;
  int qb[NS], qt0[NS];
  if (a.keys_ready) {
    build_walk();
    if (warp == 0 && lane == 0) {
      tma::prefetch_map(&tm_k);
      int b, t0, t_lim;
      while (npre < NS && walk.next(b, t0, t_lim)) {
        const uint32_t st = sbase + npre * kStageBytes;
        const uint32_t fb = smem_u32(&aux->full[npre]);
        tma::mbar_arrive_expect_tx(fb, kStageBytes);
        const int krow = int(int64_t(b) * a.k_row_stride + t0);
        tma::load_2d(st, &tm_k, 0, krow, fb);
        tma::load_2d(st + kKeyBytes / 2, &tm_k, 64, krow, fb);
        qt0[npre] = t0;
        qb[npre++] = b;
      }
    }
  }
  // otherwise the set-up above touches no global memory; keys, q, w and
  // t_valid may be the previous kernels' outputs
  pdl_wait();
  pdl_launch_dependents();
  if (!a.keys_ready) build_walk();

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      tma::prefetch_map(&tm_k);
      tma::prefetch_map(&tm_q);
      for (int i = 0; i < npre; ++i) {
        const uint32_t st = sbase + i * kStageBytes;
        const uint32_t fb = smem_u32(&aux->full[i]);
        tma::load_2d(st + kKeyBytes, &tm_q, 0, qb[i] * H, fb);
        tma::load_2d(st + kKeyBytes + kQBytes / 2, &tm_q, 64, qb[i] * H, fb);
      }
      int it = npre;
      int b, t0, t_lim;
      auto issue = [&](int b_, int t0_) {
        const int s = it % NS;
        if (it >= NS) tc::mbar_wait(smem_u32(&aux->empty[s]), ((it / NS) - 1) & 1, a.status, 2, a.wait_limit);
        const uint32_t st = sbase + s * kStageBytes;
        const uint32_t fb = smem_u32(&aux->full[s]);
        tma::mbar_arrive_expect_tx(fb, kStageBytes);
        const int krow = int(int64_t(b_) * a.k_row_stride + t0_);
        tma::load_2d(st, &tm_k, 0, krow, fb);
        tma::load_2d(st + kKeyBytes / 2, &tm_k, 64, krow, fb);
        tma::load_2d(st + kKeyBytes, &tm_q, 0, b_ * H, fb);
        tma::load_2d(st + kKeyBytes + kQBytes / 2, &tm_q, 64, b_ * H, fb);
      };
      if constexpr (kDyn) {
        // every item taken is published for the MMA and epilogue warps
        auto publish = [&](int i, int b_, int t0_) {
          aux->info_b[i % kInfo] = b_;
          aux->info_t0[i % kInfo] = t0_;
          tc::mbar_arrive(smem_u32(&aux->info_full[i % kInfo]));
        };
        for (int i = 0; i < npre; ++i) publish(i, qb[i], qt0[i]);
        while (walk.next(b, t0, t_lim)) {
          issue(b, t0);
          publish(it, b, t0);
          ++it;
        }
        const int* pre = reinterpret_cast<const int*>(smem + kOffPre);
        const int even = (total_live + gridDim.x - 1) / gridDim.x;
        const int first = int(gridDim.x) * max(NS, even * 4 / 5);
        // one claim in flight ahead of the item being issued
        int next = int(atomicAdd(a.dyn, 1u));
        for (;;) {
          const int l = first + next;
          if (l >= total_live) break;
          next = int(atomicAdd(a.dyn, 1u));
          // the sequence holding live item l: the last b with pre[b] <= l
          int lo = 0, hi = a.B - 1;
          while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (pre[mid] <= l) lo = mid;
            else hi = mid - 1;
          }
          t0 = (l - pre[lo]) * TILE;
          issue(lo, t0);
          publish(it, lo, t0);
          ++it;
        }
        publish(it, -1, 0);
        // every CTA has made its last claim once all have counted themselves
        // here: the last one resets the counters for the next call
        if (atomicAdd(a.dyn + 1, 1u) == gridDim.x - 1) {
          atomicExch(a.dyn, 0u);
          atomicExch(a.dyn + 1, 0u);
        }
      } else {
        while (walk.next(b, t0, t_lim)) {
          issue(b, t0);
          ++it;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0;
      int b, t0, t_lim;
      auto next_item = [&]() -> bool {
        if constexpr (kDyn) {
          if (!tc::mbar_wait(smem_u32(&aux->info_full[it % kInfo]), (it / kInfo) & 1, a.status, 2, a.wait_limit))
            return false;
          return aux->info_b[it % kInfo] >= 0;
        } else {
          return walk.next(b, t0, t_lim);
        }
      };
      while (next_item()) {
        const int s = it % NS, acc = it & 1;
        tc::mbar_wait(smem_u32(&aux->full[s]), (it / NS) & 1, a.status, 2, a.wait_limit);
        if (it >= 2) tc::mbar_wait(smem_u32(&aux->acc_empty[acc]), ((it - 2) >> 1) & 1, a.status, 2, a.wait_limit);
        tc::fence_after_sync();
        const uint32_t st = sbase + s * kStageBytes;
#pragma unroll
        for (int ks = 0; ks < DI / 16; ++ks) {
          const uint64_t ad = tc::smem_desc(st + (ks >> 2) * (kKeyBytes / 2) + (ks & 3) * 32, 16, 1024,
                                            tc::kLayoutSw128);
          const uint64_t bd = tc::smem_desc(st + kKeyBytes + (ks >> 2) * (kQBytes / 2) + (ks & 3) * 32, 16, 1024,
                                            tc::kLayoutSw128);
          tc::mma_bf16(tmem + 64 * acc, ad, bd, kIdesc, ks > 0 ? 1u : 0u);
        }
        tc::mma_commit(smem_u32(&aux->acc_full[acc]));
        tc::mma_commit(smem_u32(&aux->empty[s]));
        ++it;
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    int it = 0;
    int cur_b = -1;
    float wv[H];
    int b, t0, t_lim;
    auto next_item = [&]() -> bool {
      if constexpr (kDyn) {
        if (!tc::mbar_wait(smem_u32(&aux->info_full[it % kInfo]), (it / kInfo) & 1, a.status, 2, a.wait_limit))
          return false;
        b = aux->info_b[it % kInfo];
        t0 = aux->info_t0[it % kInfo];
        if (b < 0) return false;
        t_lim = seq_limit(a, b);
        return true;
      } else {
        return walk.next(b, t0, t_lim);
      }
    };
    while (next_item()) {
      const int acc = it & 1;
      if (b != cur_b) {
#pragma unroll
        for (int h = 0; h < H; ++h) wv[h] = __ldg(a.w + int64_t(b) * H + h);
        cur_b = b;
      }
      tc::mbar_wait(smem_u32(&aux->acc_full[acc]), (it >> 1) & 1, a.status, 2, a.wait_limit);
      tc::fence_after_sync();
      float v0[32], v1[32];
      tc::tmem_ld32(trow + 64 * acc, v0);
      tc::tmem_ld32(trow + 64 * acc + 32, v1);
      tc::tmem_wait_ld();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(smem_u32(&aux->acc_empty[acc]));
      float s = 0.f;
#pragma unroll
      for (int h = 0; h < 32; ++h) s = fmaf(wv[h], fmaxf(v0[h], 0.f), s);
#pragma unroll
      for (int h = 0; h < 32; ++h) s = fmaf(wv[32 + h], fmaxf(v1[h], 0.f), s);
      const int t = t0 + quarter * 32 + lane;
      if (t < t_lim) a.score[int64_t(b) * a.ld_score + t] = s;
      ++it;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace idxtc
}  // namespace dsa
