// Indexer scores of a prefill chunk on the tcgen05 tensor cores: the dense
// [S*64 x 128] x [128 x T] contraction with the relu * w head reduction in
// the epilogue (inference.py:5260-5275 per token; CPU formula
// indexer.py:10-23), one key cache shared by all S tokens.
//
// s[q, t] = sum_h w[q, h] * relu(iq[q, h, :] . k[t, :])   for t < t_valid[q]
//
// A work item is (group of 4 tokens, 128-key tile): one MMA batch of
// M = 128 keys x N = 256 (4 tokens x 64 heads) x K = 128, so each key tile
// read from L2 feeds four tokens (the decode kernel, N = 64, re-reads the
// tile for every token).  Persistent CTAs walk a contiguous item range in
// (group, tile) order, so a group's 64 KB of q stays in shared memory across
// its tiles and is reloaded only when the group changes.  Roles:
//   warp 0      TMA producer: q of the group (once per group, single buffer
//               guarded by q_full / q_empty) and key tiles into a 4-stage ring
//   warp 1      MMA issuer: 8 x (M128 N256 K16) per item into one of two
//               256-column TMEM accumulators (all 512 columns)
//   warps 2-5   epilogue: thread = key (TMEM lane); per token 64 relu * w
//               terms from 2 x 32-column TMEM loads, the group's w staged in
//               shared memory by these warps at each group switch
// Tiles at or past the group's largest t_valid are skipped; scores at or past
// a token's own t_valid are not written.
#pragma once

#include "common.cuh"
#include "tc05.cuh"
#include "tma.cuh"

namespace dsa {
namespace idxpf {

constexpr int H = 64;
constexpr int DI = 128;
constexpr int QG = 4;                      // tokens per group
constexpr int N = QG * H;                  // 256 MMA columns
constexpr int TILE = 128;                  // keys per item
constexpr int NS = 4;
constexpr int THREADS = 192;
constexpr int kKeyBytes = TILE * DI * 2;   // 32 KB: 2 k-blocks of [128 rows x 128 B]
constexpr int kQBytes = N * DI * 2;        // 64 KB: 2 k-blocks of [256 rows x 128 B]
constexpr int kOffQ = NS * kKeyBytes;      // ring first, then q
constexpr int kOffW = kOffQ + kQBytes;     // w of the group [4 x 64] fp32
constexpr int kOffAux = kOffW + QG * H * 4;
constexpr int kSmemBytes = kOffAux + 256 + 1024;  // Aux (< 192 B), the group's t_valid at +192
constexpr uint32_t kTmemCols = 512;        // 2 accumulators x 256 columns
constexpr uint32_t kIdesc = tc::idesc_bf16(128, N, false, false);

struct Aux {
  uint64_t full[NS];
  uint64_t empty[NS];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t q_full;
  uint64_t q_empty;
  uint64_t w_full;   // the MMA warp's final drain
  uint32_t tmem_base;
};

struct Args {
  const float* w;         // [S, 64]
  float* score;           // [S, ld_score]
  const int32_t* t_valid; // [S] or null
  int32_t* status;
  long long wait_limit;   // spin budget of every bounded wait, SM cycles
  int S, T, tiles, items_per_cta;
  int64_t ld_score;
};

// the group's scoring limit: the largest t_valid of its tokens
__device__ __forceinline__ int group_limit(const Args& a, int g) {
  if (!a.t_valid) return a.T;
  int m = 0;
#pragma unroll
  for (int j = 0; j < QG; ++j) m = max(m, min(a.T, a.t_valid[g * QG + j]));
  return m;
}

__global__ void __launch_bounds__(THREADS, 1) indexer_prefill_tc_kernel(const Args a,
                                                                        const __grid_constant__ CUtensorMap tm_k,
                                                                        const __grid_constant__ CUtensorMap tm_q) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Aux* aux = reinterpret_cast<Aux*>(smem + kOffAux);
  float* sw = reinterpret_cast<float*>(smem + kOffW);
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = (a.S / QG) * a.tiles;
  const int i_begin = blockIdx.x * a.items_per_cta;
  const int i_end = min(total, i_begin + a.items_per_cta);

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
    tc::mbar_init(smem_u32(&aux->q_full), 1);
    tc::mbar_init(smem_u32(&aux->q_empty), 1);
    tc::mbar_init(smem_u32(&aux->w_full), 1);
    tc::mbar_fence_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = aux->tmem_base;

  // the live items (tiles below their group's limit) in order; every role
  // walks the same sequence, noting group switches
  auto next_live = [&](int& item, int& g, int& t0, int& lim, int& cur_g) -> bool {
    for (; item < i_end; ++item) {
      g = item / a.tiles;
      t0 = (item - g * a.tiles) * TILE;
      if (g != cur_g) {
        lim = group_limit(a, g);
        cur_g = g;
      }
      if (t0 < lim) return true;
    }
    return false;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      tma::prefetch_map(&tm_k);
      tma::prefetch_map(&tm_q);
      int it = 0, gi = 0, qg = -1;
      int item = i_begin, g = 0, t0 = 0, lim = 0, cur_g = -1;
      for (; next_live(item, g, t0, lim, cur_g); ++item) {
        if (g != qg) {
          // q of a new group: the previous group's MMAs must have finished
          if (gi > 0) tc::mbar_wait(smem_u32(&aux->q_empty), (gi - 1) & 1, a.status, 2, a.wait_limit);
          const uint32_t qb = smem_u32(&aux->q_full);
          tma::mbar_arrive_expect_tx(qb, kQBytes);
          tma::load_2d(sbase + kOffQ, &tm_q, 0, g * N, qb);
          tma::load_2d(sbase + kOffQ + kQBytes / 2, &tm_q, 64, g * N, qb);
          qg = g;
          ++gi;
        }
        const int s = it % NS;
        if (it >= NS) tc::mbar_wait(smem_u32(&aux->empty[s]), ((it / NS) - 1) & 1, a.status, 2, a.wait_limit);
        const uint32_t st = sbase + s * kKeyBytes;
        const uint32_t fb = smem_u32(&aux->full[s]);
        tma::mbar_arrive_expect_tx(fb, kKeyBytes);
        tma::load_2d(st, &tm_k, 0, t0, fb);
        tma::load_2d(st + kKeyBytes / 2, &tm_k, 64, t0, fb);
        ++it;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0, gi = 0, qg = -1;
      int item = i_begin, g = 0, t0 = 0, lim = 0, cur_g = -1;
      for (; next_live(item, g, t0, lim, cur_g); ++item) {
        if (g != qg) {
          if (gi > 0) tc::mma_commit(smem_u32(&aux->q_empty));  // after every MMA of the previous group
          tc::mbar_wait(smem_u32(&aux->q_full), gi & 1, a.status, 2, a.wait_limit);
          qg = g;
          ++gi;
        }
        const int s = it % NS, acc = it & 1;
        tc::mbar_wait(smem_u32(&aux->full[s]), (it / NS) & 1, a.status, 2, a.wait_limit);
        if (it >= 2) tc::mbar_wait(smem_u32(&aux->acc_empty[acc]), ((it - 2) >> 1) & 1, a.status, 2, a.wait_limit);
        tc::fence_after_sync();
        const uint32_t st = sbase + s * kKeyBytes;
#pragma unroll
        for (int ks = 0; ks < DI / 16; ++ks) {
          const uint64_t ad = tc::smem_desc(st + (ks >> 2) * (kKeyBytes / 2) + (ks & 3) * 32, 16, 1024,
                                            tc::kLayoutSw128);
          const uint64_t bd = tc::smem_desc(sbase + kOffQ + (ks >> 2) * (kQBytes / 2) + (ks & 3) * 32, 16, 1024,
                                            tc::kLayoutSw128);
          tc::mma_bf16(tmem + N * acc, ad, bd, kIdesc, ks > 0 ? 1u : 0u);
        }
        tc::mma_commit(smem_u32(&aux->acc_full[acc]));
        tc::mma_commit(smem_u32(&aux->empty[s]));
        ++it;
      }
      // drain: every MMA has completed before TMEM is released
      tc::mma_commit(smem_u32(&aux->w_full));
      tc::mbar_wait(smem_u32(&aux->w_full), 0, a.status, 2, a.wait_limit);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const int etid = tid - 64;     // 0..127
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    int it = 0, qg = -1;
    int* s_tv = reinterpret_cast<int*>(smem + kOffAux + 192);  // the group's t_valid, after Aux
    int item = i_begin, g = 0, t0 = 0, lim = 0, cur_g = -1;
    for (; next_live(item, g, t0, lim, cur_g); ++item) {
      if (g != qg) {
        // w of the new group into shared memory, once the 4 warps are done with the old one
        tc::named_bar_sync(2, 128);
        for (int e = etid; e < QG * H; e += 128) sw[e] = __ldg(a.w + int64_t(g) * QG * H + e);
        if (etid < QG) s_tv[etid] = a.t_valid ? min(a.T, a.t_valid[g * QG + etid]) : a.T;
        tc::named_bar_sync(2, 128);
        qg = g;
      }
      const int acc = it & 1;
      tc::mbar_wait(smem_u32(&aux->acc_full[acc]), (it >> 1) & 1, a.status, 2, a.wait_limit);
      tc::fence_after_sync();
      const int t = t0 + quarter * 32 + lane;
#pragma unroll 1
      for (int j = 0; j < QG; ++j) {
        float v0[32], v1[32];
        tc::tmem_ld32(trow + N * acc + H * j, v0);
        tc::tmem_ld32(trow + N * acc + H * j + 32, v1);
        tc::tmem_wait_ld();
        if (j == QG - 1) {
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(smem_u32(&aux->acc_empty[acc]));
        }
        const float4* wj = reinterpret_cast<const float4*>(sw + H * j);
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int h4 = 0; h4 < 8; ++h4) {
          const float4 wa = wj[h4], wb = wj[8 + h4];
          s0 = fmaf(wa.x, fmaxf(v0[4 * h4 + 0], 0.f), s0);
          s0 = fmaf(wa.y, fmaxf(v0[4 * h4 + 1], 0.f), s0);
          s0 = fmaf(wa.z, fmaxf(v0[4 * h4 + 2], 0.f), s0);
          s0 = fmaf(wa.w, fmaxf(v0[4 * h4 + 3], 0.f), s0);
          s1 = fmaf(wb.x, fmaxf(v1[4 * h4 + 0], 0.f), s1);
          s1 = fmaf(wb.y, fmaxf(v1[4 * h4 + 1], 0.f), s1);
          s1 = fmaf(wb.z, fmaxf(v1[4 * h4 + 2], 0.f), s1);
          s1 = fmaf(wb.w, fmaxf(v1[4 * h4 + 3], 0.f), s1);
        }
        if (t < s_tv[j]) a.score[int64_t(g * QG + j) * a.ld_score + t] = s0 + s1;
      }
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

}  // namespace idxpf
}  // namespace dsa
