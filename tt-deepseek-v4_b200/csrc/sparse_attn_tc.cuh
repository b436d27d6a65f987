// attn.sparse on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA per (query row, key split), 16 warps with fixed roles, 64-key tiles
// held in a two-slot ring (2 x 64 KB) next to the query block Q (64 KB):
//
//   warps 5-7, 9-11, 13-15  gather producers.  Each selected kv row (1 KB) is copied whole,
//               one 512-B half per warp instruction (16-byte cp.async from 32
//               lanes), and scattered into the tile's eight 64-dim k-block
//               slabs (128-B swizzled).  Measured on B200: random 1 KB rows
//               requested whole reach ~7 TB/s from HBM, the same rows fetched
//               128 B at a time only ~4.7 TB/s, and L2 prefetches do not help
//               (they lowered it), so each row is read once, whole.  A tile
//               completes on its slot's mbarrier through
//               cp.async.mbarrier.arrive.
//   warp 4      MMA issuer (one thread), ready-first over two kinds of batch:
//               S(t)  = K_t Q^T as one block-diagonal product: the tile is
//                       read as 128 rows x 256 dims (a key's dims 0-255 in
//                       one row, its dims 256-511 in another) against
//                       Q' = [Q dims 0-255 | Q dims 256-511] as 128 columns,
//                       so 16 MMAs of M=128 x N=128 x K=16 replace 32 of
//                       M=64 x N=64 (a tcgen05.mma below N=128 costs ~80
//                       cycles whatever its size, measured on B200).  Row r
//                       of a key's first half pairs with columns 0-63, its
//                       second half with columns 64-127; the two partials
//                       of a key sit in the same TMEM sub-partition (rows
//                       interleaved in 16-key chunks) and the softmax adds
//                       them.  Issued once tile t has landed;
//               PV(t): O^T += V_t^T P_t^T  (M=128 dims per block, N=64 heads,
//                       K=64 keys; A = two adjacent k-block slabs read
//                       MN-major, B = P, MN-major) into a TMEM accumulator that
//                       lives for the whole split (lane = dim, column = head),
//                       issued once the softmax of tile t wrote P; it then
//                       releases the tile's slot for the next copy.
//               A wait between dependent batches drains the tensor pipe
//               (about 700 cycles measured), so the issuer keeps whichever
//               batch is ready queued.
//   warps 0-3   softmax.  Two 16x256b TMEM loads per warp (the two dim
//               halves of its 16 keys) spread the 64 x 64 scores over 128
//               threads: thread i of warp w holds keys 16w + i/4 and
//               16w + 8 + i/4, heads 8r + 2(i%4) + {0,1}, r = 0..7.  The
//               running max per head lives in shared memory and moves only
//               when some score beats it by 2^8 (one barrier with an OR tells
//               all 128 threads), so O^T is rescaled rarely and P <= 256.  P
//               goes to one of two buffers as 128-B swizzled rows per key,
//               written by stmatrix (the 16x256b fragment is its 8x8 layout).
//               The epilogue reads O^T back (lane = output dim) and stores
//               coalesced rows.
//
// Every mbarrier wait is bounded (about a second); a wait that runs out sets
// a status bit and an abort flag that makes all later waits of the CTA return
// at once, so a lost arrival ends the launch with an error instead of a hang.
#pragma once

#include "common.cuh"
#include "tc05.cuh"
#include "tma.cuh"

namespace dsa {
namespace satc {

constexpr int H = 64;
constexpr int D = 512;
constexpr int TK = 64;                                // keys per tile
constexpr int KB = D / 64;                            // 64-dim k-blocks per row
constexpr int NT = 2;                                 // tile slots
constexpr int kSlabBytes = TK * 128;                  // one 64-dim k-block of a tile: 8 KB
constexpr int kTileBytes = KB * kSlabBytes;           // 64 KB
// A tile slot holds four 16 KB pair blocks; pair block j holds k-blocks j
// (dims 64j..64j+63, "low") and j + 4 (dims 256 + 64j.., "high") of the 64
// keys as 128 rows of 128 B: rows 32q..32q+15 = low half of keys
// 16q..16q+15, rows 32q+16..32q+31 = their high half.
constexpr int kPairBytes = 2 * kSlabBytes;            // 16 KB
// 16 warps, four per scheduler (warp % 4): softmax 0-3, MMA issuer 4, and the
// producers on the schedulers of warps 1-3 only (5-7, 9-11, 13-15), so the
// MMA issuer shares its scheduler with one softmax warp; warps 8 and 12 idle.
constexpr int kProducerWarps = 9;
constexpr int kMmaWarp = 4;
constexpr int THREADS = 512;
__device__ __forceinline__ bool is_producer_warp(int w) { return w >= 5 && (w & 3) != 0; }
__device__ __forceinline__ int producer_index(int w) { return w - 5 - ((w - 4) >> 2); }
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;             // log2 units
constexpr int kQBytes = H * D * 2;                    // 64 KB: 8 k-blocks of [64 heads x 128 B]
constexpr int kQBlock = H * 128;                      // 8 KB
constexpr int kPBytes = TK * H * 2;                   // 8 KB per buffer: [64 keys x 64 heads] bf16
constexpr int kMaxTilesPerSplit = 36;
constexpr int kIdxCap = kMaxTilesPerSplit * TK;       // indices staged per split
constexpr int kAuxBytes = 4096;
constexpr int kOffQ = 0;
constexpr int kOffRing = kOffQ + kQBytes;
constexpr int kOffP = kOffRing + NT * kTileBytes;
constexpr int kOffAux = kOffP + 2 * kPBytes;
constexpr int kOffIdx = kOffAux + kAuxBytes;
constexpr int kSmemBytes = kOffIdx + kIdxCap * 4 + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0;                          // O^T: 4 blocks of [128 dims x 64 heads]
constexpr uint32_t kColS = 256;                        // S: 2 buffers of [128 rows x 128 cols], M=128 layout
constexpr uint32_t kSCols = 128;
constexpr uint32_t kIdescS = tc::idesc_bf16(128, 128, false, false);
constexpr uint32_t kIdescPV = tc::idesc_bf16(128, 64, true, true);
static_assert(kSmemBytes <= 232448, "shared memory budget");
static_assert(kColS + 2 * kSCols <= kTmemCols, "TMEM columns");
static_assert(TK % 16 == 0 && TK <= 64, "tile");

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

// trace slots (each kTrTiles long): producers issued tile t / MMA got tile t /
// MMA issued S(t) / MMA issued PV(t) / softmax got S(t) / softmax wrote P(t) /
// misc (0: start, 1: end, 2: last PV done, 3: l reduced, 4: O stored)
enum : int { kTrTiles = 256, kTrIssue = 0, kTrFull = 1, kTrMmaGot = 2, kTrS = 3, kTrPV = 4, kTrSGot = 5, kTrPDone = 6,
             kTrMisc = 7 };
// Per-tile clock stamps for timeline analysis: compiled in only with
// -DDSA_ATTN_TRACE (the hot build carries no trace branches).
#ifdef DSA_ATTN_TRACE
#define SA_TRACE(slot, t)                                                                         \
  do {                                                                                            \
    if (tr && (t) < kTrTiles) tr[(slot) * kTrTiles + (t)] = clock64();                            \
  } while (0)
#else
#define SA_TRACE(slot, t) \
  do {                    \
  } while (0)
#endif

struct Aux {
  float m[H];        // running max per head (log2 units)
  float alpha[H];    // rescale factor of the last max update
  float f[H];        // epilogue scale per head
  float red[4][H];   // per-warp partial reductions
  uint64_t q_full;
  uint64_t full[NT];
  uint64_t empty[NT];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t pv_done[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Aux) <= kAuxBytes, "aux block");

// byte offset of 16-B chunk c (0..63) of key k of a tile: k-block kb = c / 8
// lives in pair block kb % 4, half kb / 4, at row 32 (k / 16) + 16 half + k % 16,
// then the 128-B swizzle of that row
__device__ __forceinline__ uint32_t chunk_off(int k, int c) {
  const int kb = c >> 3;
  const int row = ((k >> 4) << 5) + ((kb >> 2) << 4) + (k & 15);
  return (kb & 3) * kPairBytes + row * 128 + ((((c & 7) ^ (k & 7))) << 4);
}
// Q is loaded in the same pairing: k-block kb at slab position 2 (kb % 4) + kb / 4
__host__ __device__ constexpr int q_slab_pos(int kb) { return 2 * (kb & 3) + (kb >> 2); }

__global__ void __launch_bounds__(THREADS, 1) sparse_attn_tc_kernel(const Args a,
                                                                    const __grid_constant__ CUtensorMap tm_q,
                                                                    int64_t kv_row_base_stride) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Aux* aux = reinterpret_cast<Aux*>(smem + kOffAux);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase + kOffQ, sRing = sbase + kOffRing, sP = sbase + kOffP;
  volatile int* abort_flag = &aux->abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = blockIdx.y, split = blockIdx.x;
  const int b = m / a.S;
  const int j_begin = split * a.tiles_per_split * TK;
  const int j_end = min(a.K, j_begin + a.tiles_per_split * TK);
  const int n = j_end > j_begin ? (j_end - j_begin + TK - 1) / TK : 0;
  const int32_t* idxr = a.idx + int64_t(m) * a.ld_idx;
  int32_t* s_idx = reinterpret_cast<int32_t*>(smem + kOffIdx);
#ifdef DSA_ATTN_TRACE
  long long* tr = (a.trace && blockIdx.x == 0 && blockIdx.y == 0) ? a.trace : nullptr;
#endif
  if (tid == 0) SA_TRACE(kTrMisc, 0);

  if (tid < H) aux->m[tid] = -INFINITY;
  if (tid == 0) aux->abort = 0;

  if (warp == 0) {
    tc::tmem_alloc(smem_u32(&aux->tmem_base), kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 32) {
    tc::mbar_init(smem_u32(&aux->q_full), 1);
    for (int s = 0; s < NT; ++s) {
      tc::mbar_init(smem_u32(&aux->full[s]), 32 * kProducerWarps);  // one cp.async arrival per producer lane
      tc::mbar_init(smem_u32(&aux->empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(smem_u32(&aux->s_full[s]), 1);
      tc::mbar_init(smem_u32(&aux->s_free[s]), 4);
    }
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(smem_u32(&aux->p_full[s]), 1);
      tc::mbar_init(smem_u32(&aux->pv_done[s]), 1);
    }
    tc::mbar_init(smem_u32(&aux->mma_done), 1);
    tc::mbar_fence_init();
  }
  // set-up above touches no global memory; the index list and q are the
  // previous kernels' outputs
  pdl_wait();
  pdl_launch_dependents();
  // The split's index list, staged once: -1 for masked / padding slots,
  // out-of-range rows clamped (and reported through status).
  for (int e = tid; e < n * TK; e += THREADS) {
    const int j = j_begin + e;
    int id = (j < j_end) ? idxr[j] : -1;
    if (id >= a.kv_rows) {
      if (a.status) atomicOr(a.status, kStatusBadIndex);
      id = int(a.kv_rows - 1);
    }
    s_idx[e] = id < 0 ? -1 : id;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = aux->tmem_base;

  auto wait = [&](const uint64_t* bar, uint32_t parity) {
    if (*abort_flag) return;
    if (!tc::mbar_wait(smem_u32(bar), parity, a.status, kStatusTimeout)) *abort_flag = 1;
  };
  // whole-warp wait with one polling lane
  auto warp_wait = [&](const uint64_t* bar, uint32_t parity) {
    if (lane == 0) wait(bar, parity);
    __syncwarp();
  };

  if (is_producer_warp(warp)) {
    // ------------------------------------------------------------ producers
    const int pw = producer_index(warp);
    if (pw == 0 && lane == 0 && n > 0) {
      tma::prefetch_map(&tm_q);
      tma::mbar_arrive_expect_tx(smem_u32(&aux->q_full), kQBytes);
#pragma unroll
      for (int kb = 0; kb < KB; ++kb)
        tma::load_2d(sQ + q_slab_pos(kb) * kQBlock, &tm_q, kb * 64, m * H, smem_u32(&aux->q_full));
    }
    const __nv_bfloat16* kvb = a.kv + int64_t(b) * kv_row_base_stride * D;
    for (int t = 0; t < n; ++t) {
      const int slot = t % NT;
      if (t >= NT) warp_wait(&aux->empty[slot], ((t / NT) - 1) & 1);
      const uint32_t dst = sRing + slot * kTileBytes;
      // rows pw, pw + P, ...: lane copies 16-B chunks lane and lane + 32
      for (int r = pw; r < TK; r += kProducerWarps) {
        const int id = s_idx[t * TK + r];
        const bool ok = id >= 0;
        const __nv_bfloat16* src = kvb + int64_t(ok ? id : 0) * D;
        cp_async16(dst + chunk_off(r, lane), src + lane * 8, ok ? 16 : 0);
        cp_async16(dst + chunk_off(r, lane + 32), src + (lane + 32) * 8, ok ? 16 : 0);
      }
      // this lane's arrival fires when its copies of the tile have landed
      tc::cp_async_arrive_noinc(smem_u32(&aux->full[slot]));
      if (pw == 0 && lane == 0) SA_TRACE(kTrIssue, t);
    }
    cp_async_wait<0>();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      const uint32_t hi = tc::desc_hi(1024, tc::kLayoutSw128);
      const uint32_t q_lo = tc::desc_lo(sQ, 16);
      const uint32_t k_lo = tc::desc_lo(sRing, 16);          // K-major: LBO unused
      const uint32_t v_lo = tc::desc_lo(sRing, kPairBytes);  // MN-major: LBO = the next 64 dims (next pair block)
      const uint32_t p_lo = tc::desc_lo(sP, kPBytes);        // MN-major, one 64-head group
      wait(&aux->q_full, 0);
      // Ready-first issue: PV(np) as soon as P(np) is written (it frees the
      // tile's slot for the next copy), else S(ns) as soon as tile ns has
      // landed and its S buffer is free.  Keeping MMAs queued avoids the
      // ~700-cycle drain and refill of the tensor pipe that a wait between
      // dependent batches costs.
      int ns = 0, np = 0;
      long long last = clock64();
      while (np < n) {
        bool did = false;
        if (np < ns && tc::mbar_try_wait(smem_u32(&aux->p_full[np & 1]), (np >> 1) & 1)) {
          tc::fence_after_sync();
          const uint32_t vs = v_lo + (np % NT) * (kTileBytes / 16);
          const uint32_t ps = p_lo + (np & 1) * (kPBytes / 16);
          // PV(np): 16 MMAs of M=128 dims x N=64 heads x K=16 keys.  Dims
          // 128jb.. are k-blocks 2jb, 2jb+1: pair blocks 2 (jb % 2) and the
          // next, half jb / 2; keys 16kk.. are the 16 rows at 32kk + 16 half.
#pragma unroll
          for (int jb = 0; jb < KB / 2; ++jb) {
#pragma unroll
            for (int kk = 0; kk < TK / 16; ++kk) {
              const uint32_t off = (jb & 1) * 2 * kPairBytes + (jb >> 1) * 2048 + kk * 4096;
              const uint64_t ad = tc::desc_pack(vs + off / 16, hi);
              const uint64_t bd = tc::desc_pack(ps + (kk * 2048) / 16, hi);
              tc::mma_bf16(tmem + kColO + H * jb, ad, bd, kIdescPV, (np > 0 || kk > 0) ? 1u : 0u);
            }
          }
          tc::mma_commit(smem_u32(&aux->empty[np % NT]));
          tc::mma_commit(smem_u32(&aux->pv_done[np & 1]));
          SA_TRACE(kTrPV, np);
          ++np;
          did = true;
        } else if (ns < n && ns < np + NT && tc::mbar_try_wait(smem_u32(&aux->full[ns % NT]), (ns / NT) & 1) &&
                   (ns < 2 || tc::mbar_try_wait(smem_u32(&aux->s_free[ns & 1]), ((ns - 2) >> 1) & 1))) {
          tc::fence_after_sync();
          SA_TRACE(kTrMmaGot, ns);
          const uint32_t ks0 = k_lo + (ns % NT) * (kTileBytes / 16);
          const uint32_t d = tmem + kColS + kSCols * (ns & 1);
          // S(ns): 16 block-diagonal MMAs of M=128 rows x N=128 x K=16 dims
          // over the four pair blocks (tile and Q' alike)
#pragma unroll
          for (int j = 0; j < KB / 2; ++j) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t ad = tc::desc_pack(ks0 + (j * kPairBytes + ks * 32) / 16, hi);
              const uint64_t bd = tc::desc_pack(q_lo + (j * 2 * kQBlock + ks * 32) / 16, hi);
              tc::mma_bf16(d, ad, bd, kIdescS, (j | ks) ? 1u : 0u);
            }
          }
          tc::mma_commit(smem_u32(&aux->s_full[ns & 1]));
          SA_TRACE(kTrS, ns);
          ++ns;
          did = true;
        }
        if (did) {
          last = clock64();
        } else if (*abort_flag || clock64() - last > tc::kWaitCycles) {
          if (!*abort_flag && a.status) atomicOr(a.status, kStatusTimeout);
          *abort_flag = 1;
          break;
        }
      }
      // every MMA of this CTA has completed before TMEM is released
      tc::mma_commit(smem_u32(&aux->mma_done));
      tc::mbar_wait(smem_u32(&aux->mma_done), 0, a.status, kStatusTimeout);
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------ softmax warps 0-3
    // Keys 16w..16w+15: their low-dim partials sit in TMEM lanes 32w..32w+15
    // (columns 0-63 of the S buffer), their high-dim partials in lanes
    // 32w+16..32w+31 (columns 64-127); S = low + high.
    const int q4 = lane & 3, g8 = lane >> 2;
    const int ka = warp * 16 + g8, kb2 = ka + 8;  // this thread's two keys
    const uint32_t tq = tmem + ((uint32_t)(warp * 32) << 16);
    const uint32_t tq_hi = tmem + ((uint32_t)(warp * 32 + 16) << 16) + H;
    // [r][e] -> head 8r + 2 q4 + e: running max (a register copy of aux->m)
    // and partial sums of p over this thread's keys
    float mr[16], lp[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      mr[i] = -INFINITY;
      lp[i] = 0.f;
    }
    // stmatrix x4 number j writes the 8x8 blocks (keys 16w + 8g.., heads
    // 8r..) for (g, r) = (0, 2j), (1, 2j), (0, 2j+1), (1, 2j+1); lane l gives
    // the address of row l % 8 of block l / 8: one 16-B chunk of a P row
    const int sm_g = (lane >> 3) & 1, sm_r = lane >> 4, sm_key = warp * 16 + 8 * sm_g + (lane & 7);
    for (int t = 0; t < n; ++t) {
      const bool va = s_idx[t * TK + ka] >= 0, vb = s_idx[t * TK + kb2] >= 0;
      warp_wait(&aux->s_full[t & 1], (t >> 1) & 1);
      tc::fence_after_sync();
      if (tid == 0) SA_TRACE(kTrSGot, t);
      float v[32], vh[32];
      tc::tmem_ld16x256b_x8(tq + kColS + kSCols * (t & 1), v);
      tc::tmem_ld16x256b_x8(tq_hi + kColS + kSCols * (t & 1), vh);
      tc::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += vh[i];
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(smem_u32(&aux->s_free[t & 1]));
      bool need = false;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        v[4 * r + 0] = va ? v[4 * r + 0] * a.scale_log2 : -INFINITY;
        v[4 * r + 1] = va ? v[4 * r + 1] * a.scale_log2 : -INFINITY;
        v[4 * r + 2] = vb ? v[4 * r + 2] * a.scale_log2 : -INFINITY;
        v[4 * r + 3] = vb ? v[4 * r + 3] * a.scale_log2 : -INFINITY;
        need |= fmaxf(v[4 * r + 0], v[4 * r + 2]) > mr[2 * r] + kRescaleThreshold;
        need |= fmaxf(v[4 * r + 1], v[4 * r + 3]) > mr[2 * r + 1] + kRescaleThreshold;
      }
      const bool any = tc::named_bar_red_or(1, 128, need);
      if (any) {
        // tile max per head: this thread's two keys, then the 8 lanes that
        // share q4 (xor 4, 8, 16), then the 4 warps through shared memory
        float mx[16];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          mx[2 * r] = fmaxf(v[4 * r + 0], v[4 * r + 2]);
          mx[2 * r + 1] = fmaxf(v[4 * r + 1], v[4 * r + 3]);
        }
#pragma unroll
        for (int off = 4; off < 32; off <<= 1)
#pragma unroll
          for (int i = 0; i < 16; ++i) mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], off));
        if (g8 == 0) {
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            aux->red[warp][8 * r + 2 * q4] = mx[2 * r];
            aux->red[warp][8 * r + 2 * q4 + 1] = mx[2 * r + 1];
          }
        }
        tc::named_bar_sync(1, 128);
        if (tid < H) {
          const float tmax = fmaxf(fmaxf(aux->red[0][tid], aux->red[1][tid]), fmaxf(aux->red[2][tid], aux->red[3][tid]));
          const float mo = aux->m[tid];
          const float mn = fmaxf(mo, tmax);
          aux->alpha[tid] = (mn == -INFINITY) ? 1.f : tc::ex2(mo - mn);
          aux->m[tid] = mn;
        }
        tc::named_bar_sync(1, 128);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const float2 al = *reinterpret_cast<const float2*>(&aux->alpha[8 * r + 2 * q4]);
          const float2 mn = *reinterpret_cast<const float2*>(&aux->m[8 * r + 2 * q4]);
          lp[2 * r] *= al.x;
          lp[2 * r + 1] *= al.y;
          mr[2 * r] = mn.x;
          mr[2 * r + 1] = mn.y;
        }
        if (t >= 1) {
          // (rare) O^T *= alpha per column, once PV(t-1) has completed
          warp_wait(&aux->pv_done[(t - 1) & 1], ((t - 1) >> 1) & 1);
          tc::fence_after_sync();
          const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
          const volatile float* alv = aux->alpha;
#pragma unroll 1
          for (int cb = 0; cb < 8; ++cb) {
            float o[32];
            const uint32_t ta = tl + kColO + 32 * cb;
            tc::tmem_ld32(ta, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alv[32 * (cb & 1) + i];
            tc::tmem_st32(ta, o);
          }
          tc::tmem_wait_st();
        }
      }
      // p = 2^(x - m) <= 2^8, packed to bf16 pairs: pa[r] for key ka, pb[r]
      // for key kb2, heads 8r + 2 q4 + {0, 1}
      uint32_t pa[8], pb[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float p0 = (v[4 * r + 0] == -INFINITY) ? 0.f : tc::ex2(v[4 * r + 0] - mr[2 * r]);
        const float p1 = (v[4 * r + 1] == -INFINITY) ? 0.f : tc::ex2(v[4 * r + 1] - mr[2 * r + 1]);
        const float p2 = (v[4 * r + 2] == -INFINITY) ? 0.f : tc::ex2(v[4 * r + 2] - mr[2 * r]);
        const float p3 = (v[4 * r + 3] == -INFINITY) ? 0.f : tc::ex2(v[4 * r + 3] - mr[2 * r + 1]);
        lp[2 * r] += p0 + p2;
        lp[2 * r + 1] += p1 + p3;
        pa[r] = pack_bf16x2(p0, p1);
        pb[r] = pack_bf16x2(p2, p3);
      }
      // P buffer t & 1 was last read by PV(t-2)
      if (t >= 2) warp_wait(&aux->pv_done[t & 1], ((t - 2) >> 1) & 1);
      const uint32_t pbuf = sP + (t & 1) * kPBytes;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = 2 * j + sm_r;
        const uint32_t addr = pbuf + sm_key * 128 + ((r ^ (sm_key & 7)) << 4);
        asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pa[2 * j]),
                     "r"(pb[2 * j]), "r"(pa[2 * j + 1]), "r"(pb[2 * j + 1])
                     : "memory");
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      tc::named_bar_sync(1, 128);
      if (tid == 0) tc::mbar_arrive(smem_u32(&aux->p_full[t & 1]));
      if (tid == 0) SA_TRACE(kTrPDone, t);
    }
    // ---------------------------------------------------------------- epilogue
    if (n > 0) warp_wait(&aux->pv_done[(n - 1) & 1], ((n - 1) >> 1) & 1);
    tc::fence_after_sync();
    if (tid == 0) SA_TRACE(kTrMisc, 2);
    // l per head: each head's partial sums sit in 32 threads (8 lanes of
    // each warp); gather them through the P buffers, free now that the last
    // PV has completed.  (A shuffle tree here measured ~10k cycles, this ~1k.)
    float* lbuf = reinterpret_cast<float*>(smem + kOffP);
#pragma unroll
    for (int i = 0; i < 16; ++i) lbuf[i * 128 + tid] = lp[i];
    tc::named_bar_sync(1, 128);
    if (tid < H) {
      const float mh = aux->m[tid];
      const float* lr = lbuf + (2 * (tid >> 3) + (tid & 1)) * 128 + ((tid & 7) >> 1);
      float lw[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        lw[w] = 0.f;
#pragma unroll
        for (int g = 0; g < 8; ++g) lw[w] += lr[w * 32 + g * 4];
      }
      const float lh = (lw[0] + lw[1]) + (lw[2] + lw[3]);
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
    if (tid == 0) SA_TRACE(kTrMisc, 3);
    const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
    const int dloc = warp * 32 + lane;
#pragma unroll 1
    for (int jb = 0; jb < 4; ++jb) {
      const int d = 128 * jb + dloc;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float o[32];
        if (n > 0) {
          tc::tmem_ld32(tl + kColO + H * jb + 32 * hf, o);
          tc::tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (a.final_mode) {
          __nv_bfloat16* om = a.out + int64_t(m) * H * D + d;
#pragma unroll
          for (int i = 0; i < 32; ++i) om[(32 * hf + i) * D] = f2bf(o[i] * aux->f[32 * hf + i]);
        } else {
          float* po = a.part_o + (int64_t(split) * a.M + m) * H * D + d;
#pragma unroll
          for (int i = 0; i < 32; ++i) po[(32 * hf + i) * D] = o[i];
        }
      }
    }
  }
  if (tid == 0) SA_TRACE(kTrMisc, 4);
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
