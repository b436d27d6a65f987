// attn.sparse on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA per (query row, key split); 6 warps with fixed roles:
//   warp 4      gather producer: 16-byte cp.async of the selected kv rows into
//               a 4-stage ring of 32-row tiles (128-B swizzled, K-major), the
//               query's 64 x 512 Q block once; signals `full[stage]`.
//   warp 5      MMA issuer (one thread): S(t) = Q K_t^T  (M=64 heads, N=32
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

namespace dsa {
namespace satc {

constexpr int H = 64;
constexpr int D = 512;
constexpr int TK = 32;            // keys per tile
constexpr int NS = 4;             // ring stages
constexpr int DEPTH = NS - 1;     // tiles in flight ahead of the consumer
constexpr int THREADS = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

constexpr int kQBytes = H * D * 2;          // 64 KB, 8 k-blocks of [64 rows x 128 B]
constexpr int kTileBytes = TK * D * 2;      // 32 KB, 8 k-blocks of [32 rows x 128 B]
constexpr int kKBlockQ = H * 128;           // 8 KB
constexpr int kKBlockT = TK * 128;          // 4 KB
constexpr int kPBytes = H * TK * 2;         // 4 KB, core matrices 8 heads x 8 keys

constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQBytes;
constexpr int kOffP = kOffK + NS * kTileBytes;
constexpr int kOffAux = kOffP + kPBytes;    // floats / barriers
constexpr int kAuxBytes = 2048;
constexpr int kSmemBytes = kOffAux + kAuxBytes + 1024;  // + alignment slack

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0;     // O^T: 4 blocks x 64 columns
constexpr uint32_t kColS = 256;   // S: 2 buffers x 32 columns

constexpr uint32_t kIdescS = tc::idesc_bf16(64, TK, false, false);
constexpr uint32_t kIdescPV = tc::idesc_bf16(128, 64, true, false);

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
};

struct Aux {
  uint64_t full[NS];
  uint64_t empty[NS];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full;
  uint64_t o_done;
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

__global__ void __launch_bounds__(THREADS, 1) sparse_attn_tc_kernel(const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Aux* aux = reinterpret_cast<Aux*>(smem + kOffAux);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase + kOffQ, sK = sbase + kOffK, sP = sbase + kOffP;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = blockIdx.y, split = blockIdx.x;
  const int b = m / a.S;
  const int j_begin = split * a.tiles_per_split * TK;
  const int j_end = min(a.K, j_begin + a.tiles_per_split * TK);
  const int n = j_end > j_begin ? (j_end - j_begin + TK - 1) / TK : 0;
  const int32_t* idxr = a.idx + int64_t(m) * a.ld_idx;

  if (warp == 0) {
    tc::tmem_alloc(smem_u32(&aux->tmem_base), kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(smem_u32(&aux->full[s]), 1);
      tc::mbar_init(smem_u32(&aux->empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(smem_u32(&aux->s_full[s]), 1);
      tc::mbar_init(smem_u32(&aux->s_free[s]), 4);
    }
    tc::mbar_init(smem_u32(&aux->p_full), 1);
    tc::mbar_init(smem_u32(&aux->o_done), 1);
    tc::mbar_fence_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = aux->tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    const __nv_bfloat16* kvb = a.kv + int64_t(b) * a.kv_bstride;
    const __nv_bfloat16* qm = a.q + int64_t(m) * H * D;
    if (n > 0) {
      for (int e = lane; e < H * 64; e += 32) {
        const int r = e >> 6, c = e & 63;
        cp_async16(sQ + sw128_off(r, c, kKBlockQ), qm + r * D + c * 8, 16);
      }
    }
    const int rr = lane >> 3, cc = lane & 7;
    // Signal tile t - DEPTH before (possibly) waiting for a free stage: the
    // MMA warp needs that tile to issue the PV that frees the stage.
    for (int t = 0; t < n + DEPTH; ++t) {
      if (t >= DEPTH) {
        cp_async_wait<DEPTH - 1>();
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(smem_u32(&aux->full[(t - DEPTH) % NS]));
      }
      if (t < n) {
        const int stage = t % NS;
        if (t >= NS) tc::mbar_wait(smem_u32(&aux->empty[stage]), ((t / NS) - 1) & 1, a.status, kStatusTimeout);
        const int j = j_begin + t * TK + lane;
        int id = (j < j_end) ? idxr[j] : -1;
        if (id >= a.kv_rows) {
          if (a.status) atomicOr(a.status, kStatusBadIndex);
          id = int(a.kv_rows - 1);
        }
        const uint32_t dst = sK + stage * kTileBytes;
#pragma unroll 2
        for (int rg = 0; rg < TK / 4; ++rg) {
          const int r = rg * 4 + rr;
          const int rid = __shfl_sync(0xffffffffu, id, r);
          const bool ok = rid >= 0;
          const __nv_bfloat16* src = kvb + int64_t(ok ? rid : 0) * D + cc * 8;
#pragma unroll
          for (int kb = 0; kb < 8; ++kb)
            cp_async16(dst + sw128_off(r, kb * 8 + cc, kKBlockT), src + kb * 64, ok ? 16 : 0);
        }
      }
      cp_async_commit();
    }
    cp_async_wait<0>();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      auto issue_pv = [&](int u) {
        tc::mbar_wait(smem_u32(&aux->p_full), u & 1, a.status, kStatusTimeout);
        tc::fence_after_sync();
        const uint32_t kt = sK + (u % NS) * kTileBytes;
#pragma unroll
        for (int jb = 0; jb < 4; ++jb) {
#pragma unroll
          for (int kk = 0; kk < TK / 16; ++kk) {
            const uint64_t ad = tc::smem_desc(kt + (2 * jb) * kKBlockT + kk * 16 * 128, kKBlockT, 1024,
                                              tc::kLayoutSw128);
            const uint64_t bd = tc::smem_desc(sP + kk * 256, 128, 512, tc::kLayoutNone);
            tc::mma_bf16(tmem + kColO + 64 * jb, ad, bd, kIdescPV, (u > 0 || kk > 0) ? 1u : 0u);
          }
        }
        tc::mma_commit(smem_u32(&aux->o_done));
        tc::mma_commit(smem_u32(&aux->empty[u % NS]));
      };
      for (int t = 0; t < n; ++t) {
        const int stage = t % NS;
        tc::mbar_wait(smem_u32(&aux->full[stage]), (t / NS) & 1, a.status, kStatusTimeout);
        if (t >= 2) tc::mbar_wait(smem_u32(&aux->s_free[t & 1]), ((t - 2) >> 1) & 1, a.status, kStatusTimeout);
        tc::fence_after_sync();
        const uint32_t kt = sK + stage * kTileBytes;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint64_t ad = tc::smem_desc(sQ + (ks >> 2) * kKBlockQ + (ks & 3) * 32, 16, 1024, tc::kLayoutSw128);
          const uint64_t bd = tc::smem_desc(kt + (ks >> 2) * kKBlockT + (ks & 3) * 32, 16, 1024, tc::kLayoutSw128);
          tc::mma_bf16(tmem + kColS + 32 * (t & 1), ad, bd, kIdescS, ks > 0 ? 1u : 0u);
        }
        tc::mma_commit(smem_u32(&aux->s_full[t & 1]));
        if (t >= 1) issue_pv(t - 1);
      }
      issue_pv(n - 1);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps 0-3
    const int h = warp * 16 + lane;  // valid for lane < 16
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    float m_run = -INFINITY, l_run = 0.f;
    for (int t = 0; t < n; ++t) {
      const int j = j_begin + t * TK + lane;
      const int id = (j < j_end) ? idxr[j] : -1;
      const uint32_t vmask = __ballot_sync(0xffffffffu, id >= 0);
      tc::mbar_wait(smem_u32(&aux->s_full[t & 1]), (t >> 1) & 1, a.status, kStatusTimeout);
      tc::fence_after_sync();
      float s[TK];
      tc::tmem_ld32(trow + kColS + 32 * (t & 1), s);
      tc::tmem_wait_ld();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(smem_u32(&aux->s_free[t & 1]));
      bool need = false;
      float alpha = 1.f;
      if (lane < 16) {
        float tmax = -INFINITY;
#pragma unroll
        for (int i = 0; i < TK; ++i) {
          s[i] = ((vmask >> i) & 1u) ? s[i] * a.scale_log2 : -INFINITY;
          tmax = fmaxf(tmax, s[i]);
        }
        need = tmax > m_run + kRescaleThreshold;
        float m_new = m_run;
        if (need) {
          m_new = tmax;
          alpha = exp2f(m_run - m_new);
        }
        float rs = 0.f;
#pragma unroll
        for (int i = 0; i < TK; ++i) {
          s[i] = (s[i] == -INFINITY) ? 0.f : exp2f(s[i] - m_new);
          rs += s[i];
        }
        l_run = l_run * alpha + rs;
        m_run = m_new;
        aux->alpha[h] = alpha;
      }
      const bool wany = __any_sync(0xffffffffu, need);
      if (lane == 0) aux->any[warp] = wany ? 1 : 0;
      if (t >= 1) tc::mbar_wait(smem_u32(&aux->o_done), (t - 1) & 1, a.status, kStatusTimeout);
      tc::named_bar_sync(1, 128);
      const bool any = (aux->any[0] | aux->any[1] | aux->any[2] | aux->any[3]) != 0;
      if (any && t >= 1) {
        tc::fence_after_sync();
#pragma unroll 1
        for (int jb = 0; jb < 4; ++jb) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            float v[32];
            const uint32_t ta = trow + kColO + 64 * jb + 32 * hf;
            tc::tmem_ld32(ta, v);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= aux->alpha[32 * hf + i];
            tc::tmem_st32(ta, v);
          }
        }
        tc::tmem_wait_st();
      }
      if (lane < 16) {
        // P row of head h: keys 8c..8c+7 -> core matrix (h/8, c)
        const uint32_t prow = sP + (h >> 3) * 512 + (h & 7) * 16;
#pragma unroll
        for (int c = 0; c < TK / 8; ++c) {
          const uint32_t w0 = pack_bf16x2(s[8 * c + 0], s[8 * c + 1]);
          const uint32_t w1 = pack_bf16x2(s[8 * c + 2], s[8 * c + 3]);
          const uint32_t w2 = pack_bf16x2(s[8 * c + 4], s[8 * c + 5]);
          const uint32_t w3 = pack_bf16x2(s[8 * c + 6], s[8 * c + 7]);
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(prow + c * 128), "r"(w0), "r"(w1), "r"(w2),
                       "r"(w3)
                       : "memory");
        }
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      tc::named_bar_sync(1, 128);
      if (tid == 0) tc::mbar_arrive(smem_u32(&aux->p_full));
    }
    // ---------------------------------------------------------------- epilogue
    if (n > 0) tc::mbar_wait(smem_u32(&aux->o_done), (n - 1) & 1, a.status, kStatusTimeout);
    tc::fence_after_sync();
    if (lane < 16) {
      aux->m[h] = m_run;
      aux->l[h] = l_run;
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
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace satc
}  // namespace dsa
