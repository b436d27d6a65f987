// attn.sparse on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA per (query row, key split); 6 warps with fixed roles:
//   warps 5-8   gather producers: 16-byte cp.async of the selected kv rows
//               (each warp owns 8 rows of every 32-row tile) into a 4-stage
//               ring (128-B swizzled, K-major), plus L2 prefetches of the rows
//               a few tiles ahead.  Many LSU-issuing warps are what saturates
//               HBM for random 1 KB rows on B200 (a single TMA gather4 issuer
//               tops out near 1.8 TB/s); the query's 64 x 512 Q block comes
//               in once by 2-D TMA.
//   warp 4      MMA issuer (one thread): S(t) = Q K_t^T  (M=64 heads, N=32
//               keys, K=512) into a double-buffered TMEM slot, then
//               O^T += V_t^T P(t-1)^T  (M=128 dims x4, N=64 heads, K=32 keys)
//               into a TMEM accumulator that lives for the whole split.
//   warps 0-3   softmax: lane l < 16 of warp w owns head 16w+l (the M=64
//               accumulator layout puts row 16w+l in TMEM lane 32w+l); online
//               softmax with lazy rescaling (the running max only moves when a
//               tile beats it by 2^8, so P <= 256 and O^T is rarely touched);
//               writes P as bf16 8x16-B core matrices; epilogue reads O^T back
//               (TMEM lane = output dim, column = head) and stores coalesced.
// The same shared-memory kv tile is the K-major B operand of Q K^T and the
// MN-major A operand of V^T P^T, so each gathered row is read from HBM once
// and from shared memory twice by the tensor cores.
#pragma once

#include "common.cuh"
#include "tc05.cuh"
#include "tma.cuh"

namespace dsa {
namespace satc {

constexpr int H = 64;
constexpr int D = 512;
constexpr int kProducerWarps = 4;
constexpr int THREADS = 32 * (5 + kProducerWarps);
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kQBytes = H * D * 2;          // 64 KB, 8 k-blocks of [64 rows x 128 B]
constexpr int kKBlockQ = H * 128;           // 8 KB
constexpr int kAuxBytes = 2048;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0;     // O^T: 4 blocks x 64 columns
constexpr uint32_t kColS = 256;   // S: 2 buffers x TK columns
constexpr uint32_t kIdescPV = tc::idesc_bf16(128, 64, true, false);
constexpr int kL2Ahead = 4;       // tiles prefetched into L2 beyond the ones being loaded

// Tile geometry: TK keys per tile, NS ring stages.
template <int TK_, int NS_>
struct Cfg {
  static constexpr int TK = TK_;
  static constexpr int NS = NS_;
  static constexpr int kTileBytes = TK * D * 2;      // 8 k-blocks of [TK rows x 128 B]
  static constexpr int kKBlockT = TK * 128;
  static constexpr int kPBytes = H * TK * 2;         // per buffer, 8x16-B core matrices
  static constexpr int kPSbo = TK * 16;              // stride between 8-head groups of P
  static constexpr int kIdxCap = 2048;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;
  static constexpr int kOffP = kOffK + NS * kTileBytes;
  static constexpr int kOffAux = kOffP + 2 * kPBytes;
  static constexpr int kOffIdx = kOffAux + kAuxBytes;
  static constexpr int kSmemBytes = kOffIdx + kIdxCap * 4 + 1024;
  static constexpr uint32_t kIdescS = tc::idesc_bf16(64, TK, false, false);
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(TK == 64, "the softmax fragment mapping is written for 64-key tiles");
  static_assert(kColS + 2 * TK <= kTmemCols, "TMEM columns");
};

enum : int { kStatusBadIndex = 1, kStatusTimeout = 2 };

struct Args {
  const __nv_bfloat16* q;
  const __nv_bfloat16* kv;
  int64_t kv_bstride;
  int64_t kv_rows;
  const int32_t* idx;
  int64_t ld_idx;
  const float* sink;
  __nv_bfloat16* out;
  float* lse;
  float* part_ml;
  float* part_o;
  int32_t* status;
  int S, M, K, tiles_per_split;
  float scale_log2;
  int final_mode;
  long long* trace;  // optional: per-tile clock64 stamps of CTA (0, 0), see kTr*
};

// trace slots (each kTrTiles long): producer issued / producer signalled /
// MMA got tile / MMA issued S / MMA issued PV / softmax got S / softmax done P
enum : int { kTrTiles = 256, kTrIssue = 0, kTrFull = 1, kTrMmaGot = 2, kTrS = 3, kTrPV = 4, kTrSGot = 5, kTrPDone = 6,
             kTrMisc = 7 };
#define SA_TRACE(slot, t)                                                                         \
  do {                                                                                            \
    if (tr && (t) < kTrTiles) tr[(slot) * kTrTiles + (t)] = clock64();                            \
  } while (0)

struct Aux {
  uint64_t q_full;
  uint64_t full[4];
  uint64_t empty[4];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t o_done[2];
  uint32_t tmem_base;
  int any[4];
  float alpha[H];
  float m[H];
  float l[H];
  float f[H];
};

// byte offset of 16-B chunk c (0..63, 8 dims each) of row r in a [rows x 512]
// bf16 tile stored as 8 k-blocks of [rows x 128 B] with the 128-B swizzle
__device__ __forceinline__ uint32_t sw128_off(int r, int c, int kblock_bytes) {
  return (c >> 3) * kblock_bytes + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

template <class C>
__global__ void __launch_bounds__(THREADS, 1) sparse_attn_tc_kernel(const Args a,
                                                                    const __grid_constant__ CUtensorMap tm_kv,
                                                                    const __grid_constant__ CUtensorMap tm_q,
                                                                    int64_t kv_row_base_stride) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int TK = C::TK, NS = C::NS, kTileBytes = C::kTileBytes, kKBlockT = C::kKBlockT, kPBytes = C::kPBytes;
  Aux* aux = reinterpret_cast<Aux*>(smem + C::kOffAux);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase + C::kOffQ, sK = sbase + C::kOffK, sP = sbase + C::kOffP;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = blockIdx.y, split = blockIdx.x;
  const int b = m / a.S;
  const int j_begin = split * a.tiles_per_split * TK;
  const int j_end = min(a.K, j_begin + a.tiles_per_split * TK);
  const int n = j_end > j_begin ? (j_end - j_begin + TK - 1) / TK : 0;
  const int32_t* idxr = a.idx + int64_t(m) * a.ld_idx;
  int32_t* s_idx = reinterpret_cast<int32_t*>(smem + C::kOffIdx);
  long long* tr = (a.trace && blockIdx.x == 0 && blockIdx.y == 0) ? a.trace : nullptr;
  if (tid == 0) SA_TRACE(kTrMisc, 0);

  // The split's index list, staged once: -1 for masked / padding slots,
  // out-of-range rows clamped (and reported through status).
  for (int e = tid; e < n * TK; e += THREADS) {
    const int j = j_begin + e;
    int id = (j < j_end) ? idxr[j] : -1;
    if (id >= a.kv_rows) {
      if (a.status) atomicOr(a.status, kStatusBadIndex);
      id = int(a.kv_rows - 1);
    }
    s_idx[e] = id;
  }

  if (warp == 0) {
    tc::tmem_alloc(smem_u32(&aux->tmem_base), kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 32) {
    tc::mbar_init(smem_u32(&aux->q_full), 1);
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(smem_u32(&aux->full[s]), 32 * kProducerWarps);  // one cp.async arrival per producer lane
      tc::mbar_init(smem_u32(&aux->empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(smem_u32(&aux->s_full[s]), 1);
      tc::mbar_init(smem_u32(&aux->s_free[s]), 4);
    }
    tc::mbar_init(smem_u32(&aux->p_full[0]), 1);
    tc::mbar_init(smem_u32(&aux->p_full[1]), 1);
    tc::mbar_init(smem_u32(&aux->o_done[0]), 1);
    tc::mbar_init(smem_u32(&aux->o_done[1]), 1);
    tc::mbar_fence_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = aux->tmem_base;

  if (warp >= 5) {
    // ------------------------------------------------------------ producers (warps 5..)
    const int pw = warp - 5;  // rows [8 pw, 8 pw + 8) of every tile
    if (pw == 0 && lane == 0 && n > 0) {
      tma::prefetch_map(&tm_q);
      tma::mbar_arrive_expect_tx(smem_u32(&aux->q_full), kQBytes);
#pragma unroll
      for (int kb = 0; kb < 8; ++kb)
        tma::load_2d(sQ + kb * kKBlockQ, &tm_q, kb * 64, m * H, smem_u32(&aux->q_full));
    }
    const __nv_bfloat16* kvb = a.kv + int64_t(b) * kv_row_base_stride * D;
    constexpr int kRowsPerWarp = TK / kProducerWarps;      // 8
    const int rr = lane >> 3, cc = lane & 7;
    // L2 prefetch of this warp's rows of tile u: 8 rows x 8 lines of 128 B
    auto prefetch_tile = [&](int u) {
#pragma unroll
      for (int i = 0; i < kRowsPerWarp * 8 / 32; ++i) {
        const int e = i * 32 + lane, r = e >> 3, line = e & 7;
        const int id = s_idx[u * TK + pw * kRowsPerWarp + r];
        if (id >= 0) asm volatile("prefetch.global.L2 [%0];" ::"l"(kvb + int64_t(id) * D + line * 64));
      }
    };
    for (int u = 0; u < min(n, NS + kL2Ahead); ++u) prefetch_tile(u);
    for (int t = 0; t < n; ++t) {
      const int stage = t % NS;
      if (t + NS + kL2Ahead < n) prefetch_tile(t + NS + kL2Ahead);
      if (t >= NS) tc::mbar_wait(smem_u32(&aux->empty[stage]), ((t / NS) - 1) & 1, a.status, kStatusTimeout);
      const uint32_t dst = sK + stage * kTileBytes;
#pragma unroll
      for (int rg = 0; rg < kRowsPerWarp / 4; ++rg) {
        const int r = pw * kRowsPerWarp + rg * 4 + rr;
        const int id = s_idx[t * TK + r];
        const bool ok = id >= 0;
        const __nv_bfloat16* src = kvb + int64_t(ok ? id : 0) * D + cc * 8;
#pragma unroll
        for (int kb = 0; kb < 8; ++kb)
          cp_async16(dst + sw128_off(r, kb * 8 + cc, kKBlockT), src + kb * 64, ok ? 16 : 0);
      }
      // each lane's arrival fires when its copies of this tile have landed
      tc::cp_async_arrive_noinc(smem_u32(&aux->full[stage]));
      if (pw == 0 && lane == 0) SA_TRACE(kTrIssue, t);
    }
    cp_async_wait<0>();
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      const uint32_t hi_sw128 = tc::desc_hi(1024, tc::kLayoutSw128);
      const uint32_t hi_v = tc::desc_hi(1024, tc::kLayoutSw128);
      const uint32_t hi_p = tc::desc_hi(C::kPSbo, tc::kLayoutNone);
      const uint32_t q_lo = tc::desc_lo(sQ, 16);
      tc::mbar_wait(smem_u32(&aux->q_full), 0, a.status, kStatusTimeout);
      auto issue_pv = [&](int u) {
        tc::mbar_wait(smem_u32(&aux->p_full[u & 1]), (u >> 1) & 1, a.status, kStatusTimeout);
        tc::fence_after_sync();
        const uint32_t v_lo = tc::desc_lo(sK + (u % NS) * kTileBytes, kKBlockT);
        const uint32_t p_lo = tc::desc_lo(sP + (u & 1) * kPBytes, 128);
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk) {
#pragma unroll
          for (int jb = 0; jb < 4; ++jb) {
            const uint64_t ad = tc::desc_pack(v_lo + ((2 * jb) * kKBlockT + kk * 16 * 128) / 16, hi_v);
            const uint64_t bd = tc::desc_pack(p_lo + (kk * 256) / 16, hi_p);
            tc::mma_bf16(tmem + kColO + 64 * jb, ad, bd, kIdescPV, (u > 0 || kk > 0) ? 1u : 0u);
          }
        }
        tc::mma_commit(smem_u32(&aux->o_done[u & 1]));
        tc::mma_commit(smem_u32(&aux->empty[u % NS]));
        SA_TRACE(kTrPV, u);
      };
      for (int t = 0; t < n; ++t) {
        const int stage = t % NS;
        tc::mbar_wait(smem_u32(&aux->full[stage]), (t / NS) & 1, a.status, kStatusTimeout);
        SA_TRACE(kTrMmaGot, t);
        if (t >= 2) tc::mbar_wait(smem_u32(&aux->s_free[t & 1]), ((t - 2) >> 1) & 1, a.status, kStatusTimeout);
        tc::fence_after_sync();
        const uint32_t kt = sK + stage * kTileBytes;
        // S(t) = Q K_t^T: 32 MMAs of M=64 heads x N=64 keys x K=16 (an MMA costs
        // ~47 cycles up to N=64, so a 64-key tile halves the per-key issue cost)
        const uint32_t sbuf = tmem + kColS + (t & 1) * TK;
        const uint32_t kt_lo = tc::desc_lo(kt, 16);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint64_t ad = tc::desc_pack(q_lo + ((ks >> 2) * kKBlockQ + (ks & 3) * 32) / 16, hi_sw128);
          const uint64_t bd = tc::desc_pack(kt_lo + ((ks >> 2) * kKBlockT + (ks & 3) * 32) / 16, hi_sw128);
          tc::mma_bf16(sbuf, ad, bd, C::kIdescS, ks > 0 ? 1u : 0u);
        }
        tc::mma_commit(smem_u32(&aux->s_full[t & 1]));
        SA_TRACE(kTrS, t);
        if (t >= 1) issue_pv(t - 1);
      }
      issue_pv(n - 1);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps 0-3
    // S rows (heads) 16w..16w+15 live in TMEM lanes 32w..32w+15 (M=64 layout);
    // the 16x256b load spreads each row over a quad: thread i holds heads
    // h0 = 16w + i/4 and h1 = h0 + 8, keys 8r + 2(i%4) + {0,1}, r = 0..7.
    const int q4 = lane & 3, g = lane >> 2;
    const int h0 = warp * 16 + g, h1 = h0 + 8;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    for (int t = 0; t < n; ++t) {
      uint64_t vmask = __ballot_sync(0xffffffffu, s_idx[t * TK + lane] >= 0);
      vmask |= uint64_t(__ballot_sync(0xffffffffu, s_idx[t * TK + 32 + lane] >= 0)) << 32;
      tc::mbar_wait(smem_u32(&aux->s_full[t & 1]), (t >> 1) & 1, a.status, kStatusTimeout);
      tc::fence_after_sync();
      if (tid == 0) SA_TRACE(kTrSGot, t);
      float v[32];
      tc::tmem_ld16x256b_x8(trow + kColS + TK * (t & 1), v);
      tc::tmem_wait_ld();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(smem_u32(&aux->s_free[t & 1]));
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool ok = (vmask >> (8 * r + 2 * q4 + e)) & 1ull;
          v[4 * r + e] = ok ? v[4 * r + e] * a.scale_log2 : -INFINITY;
          v[4 * r + 2 + e] = ok ? v[4 * r + 2 + e] * a.scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, v[4 * r + e]);
          mx1 = fmaxf(mx1, v[4 * r + 2 + e]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const bool need0 = mx0 > m0 + kRescaleThreshold, need1 = mx1 > m1 + kRescaleThreshold;
      const float mn0 = need0 ? mx0 : m0, mn1 = need1 ? mx1 : m1;
      const float al0 = need0 ? tc::ex2(m0 - mn0) : 1.f, al1 = need1 ? tc::ex2(m1 - mn1) : 1.f;
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          v[4 * r + e] = (v[4 * r + e] == -INFINITY) ? 0.f : tc::ex2(v[4 * r + e] - mn0);
          v[4 * r + 2 + e] = (v[4 * r + 2 + e] == -INFINITY) ? 0.f : tc::ex2(v[4 * r + 2 + e] - mn1);
          rs0 += v[4 * r + e];
          rs1 += v[4 * r + 2 + e];
        }
      }
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
      l0 = l0 * al0 + rs0;
      l1 = l1 * al1 + rs1;
      m0 = mn0;
      m1 = mn1;
      if (q4 == 0) {
        aux->alpha[h0] = al0;
        aux->alpha[h1] = al1;
      }
      // P(t) goes to buffer t&1, last read by PV(t-2); a rescale of O^T also
      // needs PV(t-1) finished.  One o_done barrier per buffer keeps every
      // wait within one phase of its barrier.
      if (t >= 2) tc::mbar_wait(smem_u32(&aux->o_done[t & 1]), ((t - 2) >> 1) & 1, a.status, kStatusTimeout);
      const bool any = tc::named_bar_red_or(1, 128, need0 || need1);
      if (any && t >= 1) {
        tc::mbar_wait(smem_u32(&aux->o_done[(t - 1) & 1]), ((t - 1) >> 1) & 1, a.status, kStatusTimeout);
        tc::fence_after_sync();
#pragma unroll 1
        for (int jb = 0; jb < 4; ++jb) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            float o[32];
            const uint32_t ta = trow + kColO + 64 * jb + 32 * hf;
            tc::tmem_ld32(ta, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= aux->alpha[32 * hf + i];
            tc::tmem_st32(ta, o);
          }
        }
        tc::tmem_wait_st();
      }
      {
        // P rows h0/h1: keys 8r + 2 q4 + {0,1} -> core matrix (h/8, r), row h%8, bytes 4 q4
        const uint32_t pb = sP + (t & 1) * kPBytes + q4 * 4;
        const uint32_t p0 = pb + (h0 >> 3) * C::kPSbo + (h0 & 7) * 16;
        const uint32_t p1 = pb + (h1 >> 3) * C::kPSbo + (h1 & 7) * 16;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(p0 + r * 128), "r"(pack_bf16x2(v[4 * r], v[4 * r + 1]))
                       : "memory");
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(p1 + r * 128), "r"(pack_bf16x2(v[4 * r + 2], v[4 * r + 3]))
                       : "memory");
        }
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      tc::named_bar_sync(1, 128);
      if (tid == 0) tc::mbar_arrive(smem_u32(&aux->p_full[t & 1]));
      if (tid == 0) SA_TRACE(kTrPDone, t);
    }
    // ---------------------------------------------------------------- epilogue
    if (n > 0) tc::mbar_wait(smem_u32(&aux->o_done[(n - 1) & 1]), ((n - 1) >> 1) & 1, a.status, kStatusTimeout);
    tc::fence_after_sync();
    if (q4 == 0) {
      aux->m[h0] = m0;
      aux->l[h0] = l0;
      aux->m[h1] = m1;
      aux->l[h1] = l1;
    }
    tc::named_bar_sync(1, 128);
    if (tid < H) {
      const float mh = aux->m[tid], lh = aux->l[tid];
      if (a.final_mode) {
        const float sk = a.sink[tid] * kLog2e;
        const float Mx = fmaxf(mh, sk);
        const float w = (mh == -INFINITY) ? 0.f : exp2f(mh - Mx);
        const float L = lh * w + exp2f(sk - Mx);
        aux->f[tid] = w / L;
        if (a.lse) a.lse[int64_t(m) * H + tid] = (Mx + log2f(L)) * kLn2;
      } else {
        const int64_t base = int64_t(split) * a.M + m;
        a.part_ml[(base * H + tid) * 2 + 0] = (mh == -INFINITY) ? -INFINITY : mh * kLn2;
        a.part_ml[(base * H + tid) * 2 + 1] = lh;
        aux->f[tid] = 1.f;
      }
    }
    tc::named_bar_sync(1, 128);
    const int dloc = warp * 32 + lane;
#pragma unroll 1
    for (int jb = 0; jb < 4; ++jb) {
      const int d = 128 * jb + dloc;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float v[32];
        if (n > 0) {
          tc::tmem_ld32(trow + kColO + 64 * jb + 32 * hf, v);
          tc::tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
        if (a.final_mode) {
          __nv_bfloat16* om = a.out + int64_t(m) * H * D + d;
#pragma unroll
          for (int i = 0; i < 32; ++i) om[(32 * hf + i) * D] = f2bf(v[i] * aux->f[32 * hf + i]);
        } else {
          float* po = a.part_o + (int64_t(split) * a.M + m) * H * D + d;
#pragma unroll
          for (int i = 0; i < 32; ++i) po[(32 * hf + i) * D] = v[i];
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0) SA_TRACE(kTrMisc, 1);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace satc
}  // namespace dsa
