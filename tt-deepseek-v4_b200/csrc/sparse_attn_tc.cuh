// attn.sparse on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA per (query row, key split), 16 warps with fixed roles, 64-key tiles
// held in a three-slot ring (3 x 64 KB); the query block lives in tensor
// memory, so shared memory holds only the ring, P and the index list.
//
// Measured tcgen05.mma costs on B200 (one issuing thread, bf16): about 80
// cycles per instruction whatever its size below N = 128 (M = 64 or 128),
// 89 at M = 128 x N = 128 with both operands in shared memory, 78 with A in
// tensor memory, 128 at N = 256.  So the kernel issues few, wide MMAs:
//
//   S(t) = Q K_t^T as one block-diagonal product per 64-key tile: the tile
//          is read as 128 rows x 256 dims (each key once with its dims
//          0-255 and once with its dims 256-511) and Q' as 128 rows x 256
//          dims the same way (each head's two dim halves), so 16 MMAs of
//          M = 128 x N = 128 x K = 16 (A = Q' in TMEM, B = the tile in shared
//          memory) cover the 64 heads x 64 keys x 512 dims; the two
//          off-diagonal blocks are never read.  Rows are interleaved in
//          16-row chunks (rows 32q..32q+15 = first halves, 32q+16..32q+31 =
//          second halves) so that both partials of a (head, key) pair sit in
//          the same TMEM sub-partition, where the softmax adds them.
//   PV(t): O^T += V_t^T P_t^T  (M = 128 dims per block, N = 64 heads, K = 16
//          keys: 16 MMAs; A = the tile read MN-major, B = P K-major) into a
//          TMEM accumulator that lives for the whole split.
//
// Roles:
//   warps 5-7, 9-11, 13-15  gather producers.  Each selected kv row (1 KB) is
//               copied whole, one 512-B half per warp instruction (16-byte
//               cp.async from 32 lanes), into the tile's four 16 KB pair
//               blocks (128-B swizzled).  Measured on B200: random 1 KB rows
//               requested whole reach ~7 TB/s from HBM, the same rows fetched
//               128 B at a time only ~4.7 TB/s, so each row is read once,
//               whole.  A tile completes on its slot's mbarrier through
//               cp.async.mbarrier.arrive.
//   warp 8      S issuer (one thread): S(t) as soon as tile t has landed and
//               the softmax has read S(t-1).
//   warps 4, 12 PV issuers (one thread each, output dims 0-255 / 256-511):
//               PV(t) as soon as P(t) is written (it frees the tile's slot
//               once both halves completed).  A tcgen05.mma of these shapes
//               costs ~90 cycles; issuing S and the two PV halves from three
//               threads keeps them from queueing behind one another (one
//               ready-first issuer: ~3.1K cycles a tile).
//   warps 0-3   softmax.  Warp w owns heads 16w..16w+15: per 16 keys, two
//               16x256b TMEM loads (the two dim halves) give thread i the
//               scores of heads 16w + i/4 and 16w + 8 + i/4 for keys
//               2(i%4) + {0,1} (+8).  Per-head maxima are a 4-lane shuffle.
//               The running max moves only when a score beats it by 2^8
//               (one barrier with an OR tells all 128 threads), so O^T is
//               rescaled rarely and P <= 256.  P goes to one of two buffers
//               as 128-B swizzled rows per head (stmatrix: the 16x256b
//               fragment is its 8x8 layout).  The epilogue reads O^T back
//               (lane = output dim) and stores coalesced rows.
//   all warps   at the start, the query block is brought into the third
//               ring slot by TMA (128-B swizzled, 8 boxes of 64 heads x 64
//               dims); each warp then moves a quarter of its sub-partition's
//               rows of Q' into tensor memory (conflict-free ld.shared,
//               tcgen05.st), after which the slot takes its first tile.
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
constexpr int NT = 3;                                 // tile slots
constexpr int kSlabBytes = TK * 128;                  // one 64-dim k-block of a tile: 8 KB
constexpr int kTileBytes = KB * kSlabBytes;           // 64 KB
// A tile slot holds four 16 KB pair blocks; pair block j holds k-blocks j
// (dims 64j..64j+63, "low") and j + 4 (dims 256 + 64j.., "high") of the 64
// keys as 128 rows of 128 B: rows 32q..32q+15 = low half of keys
// 16q..16q+15, rows 32q+16..32q+31 = their high half.
constexpr int kPairBytes = 2 * kSlabBytes;            // 16 KB
// 16 warps, four per scheduler (warp % 4): softmax 0-3, PV issuers 4 and 12,
// S issuer 8, and the producers on the schedulers of warps 1-3 only (5-7,
// 9-11, 13-15), so the issuers share their scheduler with one softmax warp.
constexpr int kProducerWarps = 9;
constexpr int kMmaWarp = 4;
constexpr int THREADS = 512;
__device__ __forceinline__ bool is_producer_warp(int w) { return w >= 5 && (w & 3) != 0; }
__device__ __forceinline__ int producer_index(int w) { return w - 5 - ((w - 4) >> 2); }
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;             // log2 units
constexpr int kPBytes = H * TK * 2;                   // 8 KB per buffer: [64 heads x 64 keys] bf16
constexpr int kMaxTilesPerSplit = 36;
constexpr int kIdxCap = kMaxTilesPerSplit * TK;       // indices staged per split
constexpr int kIdxPerThread = (kIdxCap + THREADS - 1) / THREADS;
constexpr int kAuxBytes = 4096;
constexpr int kOffRing = 0;
constexpr int kOffP = kOffRing + NT * kTileBytes;
constexpr int kOffAux = kOffP + 2 * kPBytes;
constexpr int kOffIdx = kOffAux + kAuxBytes;
constexpr int kSmemBytes = kOffIdx + kIdxCap * 4 + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0;     // O^T: 4 blocks of [128 dims x 64 heads]
constexpr uint32_t kColQ = 256;   // Q': 128 rows x 256 bf16 (128 columns)
constexpr uint32_t kColS = 384;   // S: [128 Q' rows x 128 tile rows] fp32
// pair combine exchange per (row, receiving CTA): 32 heads' O^T as
// [8 chunks][512 dims][4] fp32, then (m, l) of the 32 heads
constexpr int kPairXFloats = 8 * D * 4 + 64;
constexpr uint32_t kIdescS = tc::idesc_bf16(128, 128, false, false);
constexpr uint32_t kIdescPV = tc::idesc_bf16(128, 64, true, false);
static_assert(kSmemBytes <= 232448, "shared memory budget");
static_assert(kColS + 128 <= kTmemCols, "TMEM columns");
static_assert(TK == 64, "the block-diagonal layout assumes 64-key tiles");
static_assert(kIdxCap % 32 == 0 && THREADS % 32 == 0, "index staging ballots whole warps");

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
  __nv_bfloat16* part_ob;  // non-null: the split partial as bf16 O / l (the library's own split-K workspace)
  int32_t* status;
  int S, M, K, tiles_per_split;
  // lead tiles: with lead_tiles > 0, split s < lead_tiles takes the 64
  // entries [64 s, 64 s + 64) of the index row as its first tile, and every
  // split then a contiguous run of rest_tps tiles of the entries after
  // 64 lead_tiles.  early: those lead entries, q and the kv rows they name
  // were complete before the previous kernel on the stream began, so the
  // lead tile and q are requested before the dependency wait.
  int lead_tiles, rest_tps, early;
  float scale_log2;
  int final_mode;
  // the row's two key splits run as one thread-block cluster and finish
  // the row between them (see the pair combine at the end of the kernel):
  // out / lse are written; pair_x (M x 2 x kPairXFloats fp32) carries the
  // halves they exchange
  int pair_combine;
  float* pair_x;
  long long wait_limit;  // spin budget of every bounded wait, SM cycles
  long long* trace;  // optional: per-tile clock64 stamps of CTA (0, 0), see kTr*
};

// trace slots (each kTrTiles long): producers issued tile t / MMA got tile t /
// MMA issued S(t) / MMA issued PV(t) / softmax got S(t) / softmax wrote P(t) /
// misc (0: start, 1: end, 2: last PV done, 3: l reduced, 4: O stored,
// 5: indices staged, 6: Q' stored)
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
  float alpha[H];                 // rescale factor of the last max update
  float f[H];                     // epilogue scale per head
  float m_fin[H], l_fin[H];       // pair combine: this split's (m, l) per head, m in log2 units
  float peer_ml[H];               // pair combine: the peer split's (m, l) of the heads this CTA finishes,
                                  // written by the peer through distributed shared memory
  float coef[2][H / 2];           // pair combine: weight / L of split 0 and split 1 per finished head
  uint32_t vmask[kIdxCap / 32];   // validity bits of the staged indices
  uint64_t q_tma;
  uint64_t q_full;
  uint64_t full[NT];
  uint64_t empty[NT];
  uint64_t s_full;
  uint64_t s_free;
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

// Q' rows: warp w's sub-partition (w % 4) holds rows 32 (w % 4) + i = head
// 16 (w % 4) + i % 16, dim half i / 16; warp w moves column quarter w / 4
// (64 dims = k-block 4 half + w / 4) of those rows from the TMA copy of Q in
// shared memory (box kb at kb * 8 KB, row h at h * 128 B, 16-B chunks
// swizzled by h % 8) into tensor memory, then arrives on q_full.
__device__ __forceinline__ void q_part_to_tmem(uint32_t sq, uint32_t tmem, int warp, int lane, uint64_t* q_full) {
  const int sp = warp & 3, cq = warp >> 2;
  const int h = 16 * sp + (lane & 15), kb = 4 * (lane >> 4) + cq;
  const uint32_t row = sq + kb * (H * 128) + h * 128;
  uint32_t w[32];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint32_t addr = row + ((c ^ (h & 7)) << 4);
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[4 * c]), "=r"(w[4 * c + 1]), "=r"(w[4 * c + 2]), "=r"(w[4 * c + 3])
                 : "r"(addr));
  }
  tc::tmem_st32_u(tmem + ((uint32_t)(32 * sp) << 16) + kColQ + 32 * cq, w);
  tc::tmem_wait_st();
  tc::fence_before_sync();
  tc::mbar_arrive(smem_u32(q_full));
}

// a 32-bit store into CTA `rank`'s shared memory at the address of `p` in
// this CTA's (distributed shared memory)
__device__ __forceinline__ void st_peer_f32(const void* p, uint32_t rank, float v) {
  uint32_t addr;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(addr) : "r"(smem_u32(p)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// the pair combine's cluster barrier: release / acquire at cluster scope
// orders each CTA's exchange writes before the peer's reads
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(THREADS, 1) sparse_attn_tc_kernel(const Args a,
                                                                    const __grid_constant__ CUtensorMap tm_q,
                                                                    int64_t kv_row_base_stride) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Aux* aux = reinterpret_cast<Aux*>(smem + kOffAux);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sRing = sbase + kOffRing, sP = sbase + kOffP;
  volatile int* abort_flag = &aux->abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mrow = blockIdx.y, split = blockIdx.x;
  const int b = mrow / a.S;
  // this split's tiles: an optional lead tile, then the run [j_begin, j_end)
  const bool has_lead = split < a.lead_tiles;
  const int n_lead = has_lead ? 1 : 0;
  const int j_begin = a.lead_tiles > 0 ? a.lead_tiles * TK + split * a.rest_tps * TK : split * a.tiles_per_split * TK;
  const int j_end = max(j_begin, min(a.K, j_begin + (a.lead_tiles > 0 ? a.rest_tps : a.tiles_per_split) * TK));
  const int n = n_lead + (j_end > j_begin ? (j_end - j_begin + TK - 1) / TK : 0);
  const bool early_lead = a.early && has_lead;
  const int32_t* idxr = a.idx + int64_t(mrow) * a.ld_idx;
  int32_t* s_idx = reinterpret_cast<int32_t*>(smem + kOffIdx);
#ifdef DSA_ATTN_TRACE
  long long* tr = (a.trace && blockIdx.x == 0 && blockIdx.y == 0) ? a.trace : nullptr;
#endif
  if (tid == 0) SA_TRACE(kTrMisc, 0);

  if (tid == 0) aux->abort = 0;
  if (warp == 0) {
    tc::tmem_alloc(smem_u32(&aux->tmem_base), kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 32) {
    tc::mbar_init(smem_u32(&aux->q_tma), 1);
    tc::mbar_init(smem_u32(&aux->q_full), THREADS);  // every thread stores its part of Q'
    for (int s = 0; s < NT; ++s) {
      tc::mbar_init(smem_u32(&aux->full[s]), 32 * kProducerWarps);  // one cp.async arrival per producer lane
      tc::mbar_init(smem_u32(&aux->empty[s]), 2);  // both PV issuers' commits
    }
    tc::mbar_init(smem_u32(&aux->s_full), 1);
    tc::mbar_init(smem_u32(&aux->s_free), 4);
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(smem_u32(&aux->p_full[s]), 1);
      tc::mbar_init(smem_u32(&aux->pv_done[s]), 2);
    }
    tc::mbar_init(smem_u32(&aux->mma_done), 3);  // one commit from each issuer
    tc::mbar_fence_init();
  }
  // the barriers are initialised before any thread arrives on them (the
  // lead tile's copies may start before the dependency wait)
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  // The query block into the last ring slot (free until Q' is in TMEM).
  const uint32_t sQstage = sRing + (NT - 1) * kTileBytes;
  auto load_q = [&]() {
    if (tid == 32) {
      tma::prefetch_map(&tm_q);
      tma::mbar_arrive_expect_tx(smem_u32(&aux->q_tma), H * D * 2);
#pragma unroll
      for (int kb = 0; kb < KB; ++kb)
        tma::load_2d(sQstage + kb * (H * 128), &tm_q, kb * 64, mrow * H, smem_u32(&aux->q_tma));
    }
  };
  // index-row position of staged entry e (e < n * TK): the lead tile's 64
  // entries, then the run; -1 past the run's end
  auto index_at = [&](int e) -> int {
    if (e < n_lead * TK) return __ldg(idxr + split * TK + e);
    const int j = j_begin + e - n_lead * TK;
    return j < j_end ? __ldg(idxr + j) : -1;
  };
  const __nv_bfloat16* kvb = a.kv + int64_t(b) * kv_row_base_stride * D;
  // producers: the 16-B copies of tile t's rows pw, pw + P, ... into its slot
  auto issue_tile = [&](int t, int pw) {
    const int slot = t % NT;
    const uint32_t dst = sRing + slot * kTileBytes;
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
  };
  // staged entry: -1 for masked / padding slots, out-of-range rows clamped
  // (and reported through status), one validity bit per entry (whole warps)
  auto stage = [&](int e, int id) {
    if (id >= a.kv_rows) {
      if (a.status) atomicOr(a.status, kStatusBadIndex);
      id = int(a.kv_rows - 1);
    }
    s_idx[e] = id < 0 ? -1 : id;
    const uint32_t bits = __ballot_sync(0xffffffffu, id >= 0);
    if (lane == 0) aux->vmask[e >> 5] = bits;
  };
  const uint32_t tmem = aux->tmem_base;
  auto wait = [&](const uint64_t* bar, uint32_t parity) {
    if (*abort_flag) return;
    if (!tc::mbar_wait(smem_u32(bar), parity, a.status, kStatusTimeout, a.wait_limit)) *abort_flag = 1;
  };
  // whole-warp wait with one polling lane
  auto warp_wait = [&](const uint64_t* bar, uint32_t parity) {
    if (lane == 0) wait(bar, parity);
    __syncwarp();
  };
  // every warp moves its part of Q' once the TMA copy has landed
  auto q_part = [&]() {
    warp_wait(&aux->q_tma, 0);
    q_part_to_tmem(sQstage, tmem, warp, lane, &aux->q_full);
  };
  if (early_lead) {
    // before the dependency wait: q and the lead tile
    load_q();
    if (tid < TK) stage(tid, index_at(tid));
    __syncthreads();
    if (is_producer_warp(warp)) issue_tile(0, producer_index(warp));
  } else if (a.early) {
    load_q();
  }
  // q is ready before the dependency wait: Q' goes into tensor memory now,
  // so the first score MMA and the third tile's copies (into the slot that
  // staged q) need not wait for it once the index list is in
  if (a.early) q_part();
  pdl_wait();
  pdl_launch_dependents();
  if (!a.early) load_q();
  // The rest of the split's index list, staged once.  All loads are issued
  // before the first store.
  {
    const int e0 = early_lead ? TK : 0;
    int ids[kIdxPerThread];
#pragma unroll
    for (int k = 0; k < kIdxPerThread; ++k) {
      const int e = tid + k * THREADS;
      ids[k] = (e >= e0 && e < n * TK) ? index_at(e) : -1;
    }
#pragma unroll
    for (int k = 0; k < kIdxPerThread; ++k) {
      const int e = tid + k * THREADS;
      if (e >= e0 && e < n * TK) {  // whole warps: n * TK and e0 are multiples of 64
        stage(e, ids[k]);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (tid == 0) SA_TRACE(kTrMisc, 5);
  const bool q_late = !a.early;  // Q' still to be moved (q was loaded after the wait)

  if (is_producer_warp(warp)) {
    // ------------------------------------------------------------ producers
    // Tiles 0 .. NT-2 are requested first; the last slot holds the query
    // block until every thread has moved its part of Q' (q_full).
    const int pw = producer_index(warp);
    for (int t = early_lead ? 1 : 0; t < n; ++t) {
      if (t == NT - 1) {
        if (q_late) q_part();
        warp_wait(&aux->q_full, 0);
      }
      if (t >= NT) warp_wait(&aux->empty[t % NT], ((t / NT) - 1) & 1);
      issue_tile(t, pw);
    }
    if (n < NT && q_late) q_part();
    cp_async_wait<0>();
  } else if (warp == kMmaWarp || warp == 12) {
    // ------------------------------------------------------------ PV issuers
    // warp 4: output dims 0-255 (O^T blocks 0, 1), warp 12: dims 256-511
    if (q_late) q_part();
    const int jb0 = warp == kMmaWarp ? 0 : 2;
    if (lane == 0 && n > 0) {
      const uint32_t hi = tc::desc_hi(1024, tc::kLayoutSw128);
      const uint32_t v_lo = tc::desc_lo(sRing, kPairBytes);  // MN-major: LBO = the next 64 dims (next pair block)
      const uint32_t p_lo = tc::desc_lo(sP, 16);             // K-major rows of 64 keys per head
      wait(&aux->q_full, 0);
      tc::fence_after_sync();
      // PV issuer: PV(np) as soon as P(np) is written (S runs from warp 8)
      for (int np = 0; np < n; ++np) {
        wait(&aux->p_full[np & 1], (np >> 1) & 1);
        if (*abort_flag) break;
        tc::fence_after_sync();
        const uint32_t vs = v_lo + (np % NT) * (kTileBytes / 16);
        const uint32_t ps = p_lo + (np & 1) * (kPBytes / 16);
#pragma unroll
        for (int jb = jb0; jb < jb0 + 2; ++jb) {
#pragma unroll
          for (int kk = 0; kk < TK / 16; ++kk) {
            const uint32_t off = (jb & 1) * 2 * kPairBytes + (jb >> 1) * 2048 + kk * 4096;
            const uint64_t ad = tc::desc_pack(vs + off / 16, hi);
            const uint64_t bd = tc::desc_pack(ps + (kk * 32) / 16, hi);
            tc::mma_bf16(tmem + kColO + H * jb, ad, bd, kIdescPV, (np > 0 || kk > 0) ? 1u : 0u);
          }
        }
        tc::mma_commit(smem_u32(&aux->empty[np % NT]));
        tc::mma_commit(smem_u32(&aux->pv_done[np & 1]));
        if (jb0 == 0) SA_TRACE(kTrPV, np);
      }
      // every MMA of this CTA has completed before TMEM is released
      tc::mma_commit(smem_u32(&aux->mma_done));
      tc::mbar_wait(smem_u32(&aux->mma_done), 0, a.status, kStatusTimeout, a.wait_limit);
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------ softmax warps 0-3
    if (q_late) q_part();
    if (tid == 0) SA_TRACE(kTrMisc, 6);
    // Heads 16w..16w+15: first-half partials in TMEM lanes 32w..32w+15,
    // second-half partials in lanes 32w+16..32w+31.  Keys 16q..16q+15 are S
    // columns 32q..32q+15 for the first halves and 32q+16.. for the second.
    const int q4 = lane & 3, g8 = lane >> 2;
    const int ha = warp * 16 + g8, hb = ha + 8;  // this thread's two heads
    const uint32_t t_lo = tmem + ((uint32_t)(warp * 32) << 16) + kColS;
    const uint32_t t_hi = tmem + ((uint32_t)(warp * 32 + 16) << 16) + kColS + 16;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    // stmatrix x4 number j writes the 8x8 blocks (head group g = a/b, key
    // chunk c) = (a, 2j), (b, 2j), (a, 2j+1), (b, 2j+1); lane l gives the
    // address of row l % 8 of block l / 8: one 16-B chunk of a P row
    const int sm_head = warp * 16 + 8 * ((lane >> 3) & 1) + (lane & 7), sm_c = lane >> 4;
    for (int t = 0; t < n; ++t) {
      const uint64_t vm = (uint64_t(aux->vmask[2 * t + 1]) << 32) | aux->vmask[2 * t];
      warp_wait(&aux->s_full, t & 1);
      tc::fence_after_sync();
      if (tid == 0) SA_TRACE(kTrSGot, t);
      // v[8q + 4r + e]: head a, key 16q + 8r + 2 q4 + e; v[8q + 4r + 2 + e]: head b
      float v[32];
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        float lo[16], hi[16];
        tc::tmem_ld16x256b_x2(t_lo + 64 * h2, lo);
        tc::tmem_ld16x256b_x2(t_lo + 64 * h2 + 32, lo + 8);
        tc::tmem_ld16x256b_x2(t_hi + 64 * h2, hi);
        tc::tmem_ld16x256b_x2(t_hi + 64 * h2 + 32, hi + 8);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) v[16 * h2 + i] = lo[i] + hi[i];
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(smem_u32(&aux->s_free));
      float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const bool ok = (vm >> (16 * q + 8 * r + 2 * q4 + e)) & 1u;
            float& xa = v[8 * q + 4 * r + e];
            float& xb = v[8 * q + 4 * r + 2 + e];
            xa = ok ? xa * a.scale_log2 : -INFINITY;
            xb = ok ? xb * a.scale_log2 : -INFINITY;
            mxa = fmaxf(mxa, xa);
            mxb = fmaxf(mxb, xb);
          }
        }
      }
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
      const bool need = (mxa > m_a + kRescaleThreshold) || (mxb > m_b + kRescaleThreshold);
      const bool any = tc::named_bar_red_or(1, 128, need);
      if (any) {
        const float na = fmaxf(m_a, mxa), nb = fmaxf(m_b, mxb);
        const float al_a = (na == -INFINITY) ? 1.f : tc::ex2(m_a - na);
        const float al_b = (nb == -INFINITY) ? 1.f : tc::ex2(m_b - nb);
        l_a *= al_a;
        l_b *= al_b;
        m_a = na;
        m_b = nb;
        if (q4 == 0) {
          aux->alpha[ha] = al_a;
          aux->alpha[hb] = al_b;
        }
        tc::named_bar_sync(1, 128);
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
      // p = 2^(x - m) <= 2^8, packed to bf16 pairs: wa[c] for head a, keys
      // 8c + 2 q4 + {0, 1}; wb[c] for head b
      uint32_t wa[8], wb[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int i0 = 8 * q + 4 * r;
          const float p0 = (v[i0 + 0] == -INFINITY) ? 0.f : tc::ex2(v[i0 + 0] - m_a);
          const float p1 = (v[i0 + 1] == -INFINITY) ? 0.f : tc::ex2(v[i0 + 1] - m_a);
          const float p2 = (v[i0 + 2] == -INFINITY) ? 0.f : tc::ex2(v[i0 + 2] - m_b);
          const float p3 = (v[i0 + 3] == -INFINITY) ? 0.f : tc::ex2(v[i0 + 3] - m_b);
          l_a += p0 + p1;
          l_b += p2 + p3;
          wa[2 * q + r] = pack_bf16x2(p0, p1);
          wb[2 * q + r] = pack_bf16x2(p2, p3);
        }
      }
      // P buffer t & 1 was last read by PV(t-2)
      if (t >= 2) warp_wait(&aux->pv_done[t & 1], ((t - 2) >> 1) & 1);
      const uint32_t pbuf = sP + (t & 1) * kPBytes;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = 2 * j + sm_c;
        const uint32_t addr = pbuf + sm_head * 128 + ((c ^ (sm_head & 7)) << 4);
        asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(wa[2 * j]),
                     "r"(wb[2 * j]), "r"(wa[2 * j + 1]), "r"(wb[2 * j + 1])
                     : "memory");
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      tc::named_bar_sync(1, 128);
      if (tid == 0) tc::mbar_arrive(smem_u32(&aux->p_full[t & 1]));
      if (tid == 0) SA_TRACE(kTrPDone, t);
    }
    // ---------------------------------------------------------------- epilogue
    // (m, l) per head while the last PV still runs: the quad shuffles and
    // the stores below took ~1K cycles here, measured, when they came
    // after the wait for it
    // l per head: this thread's partial sums over its keys, then the 4 lanes
    // of the quad
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    if (q4 == 0) {
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const int h = g ? hb : ha;
        const float mh = g ? m_b : m_a, lh = g ? l_b : l_a;
        if (a.pair_combine) {
          aux->m_fin[h] = mh;
          aux->l_fin[h] = lh;
        } else if (a.final_mode) {
          const float sk = a.sink[h] * kLog2e;
          const float Mx = fmaxf(mh, sk);
          const float w = (mh == -INFINITY) ? 0.f : exp2f(mh - Mx);
          const float L = lh * w + exp2f(sk - Mx);
          aux->f[h] = w / L;
          if (a.lse) a.lse[int64_t(mrow) * H + h] = (Mx + log2f(L)) * kLn2;
        } else {
          const int64_t base = int64_t(split) * a.M + mrow;
          a.part_ml[(base * H + h) * 2 + 0] = (mh == -INFINITY) ? -INFINITY : mh * kLn2;
          a.part_ml[(base * H + h) * 2 + 1] = lh;
          aux->f[h] = a.part_ob ? (lh > 0.f ? 1.f / lh : 0.f) : 1.f;
        }
      }
    }
    if (n > 0) warp_wait(&aux->pv_done[(n - 1) & 1], ((n - 1) >> 1) & 1);
    tc::fence_after_sync();
    if (tid == 0) SA_TRACE(kTrMisc, 2);
  } else if (warp == 8) {
    // ------------------------------------------------------------ S issuer
    if (q_late) q_part();
    if (lane == 0 && n > 0) {
      const uint32_t hi = tc::desc_hi(1024, tc::kLayoutSw128);
      const uint32_t k_lo = tc::desc_lo(sRing, 16);  // K-major: LBO unused
      wait(&aux->q_full, 0);
      tc::fence_after_sync();
      for (int ns = 0; ns < n; ++ns) {
        wait(&aux->full[ns % NT], (ns / NT) & 1);
        if (ns > 0) wait(&aux->s_free, (ns - 1) & 1);
        if (*abort_flag) break;
        tc::fence_after_sync();
        SA_TRACE(kTrMmaGot, ns);
        const uint32_t ks0 = k_lo + (ns % NT) * (kTileBytes / 16);
#pragma unroll
        for (int j = 0; j < KB / 2; ++j) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t bd = tc::desc_pack(ks0 + (j * kPairBytes + ks * 32) / 16, hi);
            tc::mma_bf16_ts(tmem + kColS, tmem + kColQ + 32 * j + 8 * ks, bd, kIdescS, (j | ks) ? 1u : 0u);
          }
        }
        tc::mma_commit(smem_u32(&aux->s_full));
        SA_TRACE(kTrS, ns);
      }
      tc::mma_commit(smem_u32(&aux->mma_done));
      tc::mbar_wait(smem_u32(&aux->mma_done), 0, a.status, kStatusTimeout, a.wait_limit);
    }
    __syncwarp();
  }
  // -------------------------------------------------------------- O^T drain
  // Every warp drains part of O^T: warp w reads TMEM lanes 32 (w % 4).. (its
  // sub-partition) of block w / 4, i.e. output dims 128 (w / 4) + 32 (w % 4)
  // + lane, for all 64 heads, and stores coalesced 128-B rows per head.
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (tid == 0) SA_TRACE(kTrMisc, 3);
  if (a.pair_combine) {
    // ------------------------------------------------------ pair combine
    // The row's splits 0 and 1 are this cluster's two CTAs (cluster rank =
    // split).  CTA r finishes heads 32r..32r+31: it writes the other half
    // of its O^T (thread = output dim d, 32 heads rounded to bf16, four
    // 16-B stores) to the peer's slot of pair_x (L2-resident) and the
    // (m, l) of those heads into the peer's shared memory, the cluster
    // barrier orders those writes before the peer's reads, and each CTA
    // combines its own half (fp32, from tensor memory) with the peer's:
    // out = (w0 o0 + w1 o1) / L, w_s = 2^(m_s - M),
    // L = l0 w0 + l1 w1 + 2^(sink - M), M = max(m0, m1, sink) - split 0's
    // partial first on both CTAs, so the result does not depend on which
    // CTA runs first.  The tail is bound by the SM's traffic to L2 (the
    // exchange out, the peer's half in, the output rows): bf16 halves the
    // exchange (the split-K drain of other row shapes stores its partials
    // in bf16 as well).  Distributed shared memory moved only ~28 GB/s per
    // SM here, so it carries just the 64 (m, l) values.
    const int r = split, pr = split ^ 1;
    const int sp = warp & 3, jb = warp >> 2;
    const uint32_t tl = tmem + ((uint32_t)(32 * sp) << 16);
    const int d = 128 * jb + 32 * sp + lane;
    // [4 groups of 8 heads][D dims] x 16 B of bf16
    uint4* x_out = reinterpret_cast<uint4*>(a.pair_x + (int64_t(mrow) * 2 + pr) * kPairXFloats);
    const uint4* x_in = reinterpret_cast<const uint4*>(a.pair_x + (int64_t(mrow) * 2 + r) * kPairXFloats);
    {
      float o[32];
      if (n > 0) {
        tc::tmem_ld32(tl + kColO + H * jb + 32 * pr, o);
        tc::tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0.f;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        x_out[c * D + d] = make_uint4(pack_bf16x2(o[8 * c], o[8 * c + 1]), pack_bf16x2(o[8 * c + 2], o[8 * c + 3]),
                                      pack_bf16x2(o[8 * c + 4], o[8 * c + 5]), pack_bf16x2(o[8 * c + 6], o[8 * c + 7]));
      if (tid < 32) {
        const int h = 32 * pr + tid;
        st_peer_f32(&aux->peer_ml[2 * tid], uint32_t(pr), aux->m_fin[h]);
        st_peer_f32(&aux->peer_ml[2 * tid + 1], uint32_t(pr), aux->l_fin[h]);
      }
    }
    // this CTA's own half and the sinks are read while the partner may
    // still be on its last tiles
    float own[32], peer[32];
    if (n > 0) {
      tc::tmem_ld32(tl + kColO + H * jb + 32 * r, own);
      tc::tmem_wait_ld();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) own[i] = 0.f;
    }
    const float sink_h = tid < 32 ? a.sink[32 * r + tid] : 0.f;
    cluster_sync();  // the last access of either CTA's shared memory by the other
    uint4 xp[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) xp[c] = __ldcg(x_in + c * D + d);
    if (tid < 32) {
      const int h = 32 * r + tid;
      const float mo = aux->m_fin[h], lo = aux->l_fin[h], mp = aux->peer_ml[2 * tid], lp = aux->peer_ml[2 * tid + 1];
      const float m0 = r == 0 ? mo : mp, l0 = r == 0 ? lo : lp, m1 = r == 0 ? mp : mo, l1 = r == 0 ? lp : lo;
      const float sk = sink_h * kLog2e;
      const float Mx = fmaxf(fmaxf(m0, m1), sk);
      const float w0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - Mx);
      const float w1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - Mx);
      const float L = l0 * w0 + l1 * w1 + exp2f(sk - Mx);
      aux->coef[0][tid] = w0 / L;
      aux->coef[1][tid] = w1 / L;
      if (a.lse) a.lse[int64_t(mrow) * H + h] = (Mx + log2f(L)) * kLn2;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t w[4] = {xp[c].x, xp[c].y, xp[c].z, xp[c].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        peer[8 * c + 2 * e] = __uint_as_float(w[e] << 16);
        peer[8 * c + 2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
      }
    }
    __syncthreads();  // coefficients
    // out[h][d]: lanes d, d ^ 1 trade one value per head pair so that each
    // store writes two adjacent dims (even lane: head i, odd lane: head i + 1)
    __nv_bfloat16* om = a.out + (int64_t(mrow) * H + 32 * r) * D;
    const bool odd = lane & 1;
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const float x0a = r == 0 ? own[i] : peer[i], x1a = r == 0 ? peer[i] : own[i];
      const float x0b = r == 0 ? own[i + 1] : peer[i + 1], x1b = r == 0 ? peer[i + 1] : own[i + 1];
      const float va = fmaf(aux->coef[1][i], x1a, aux->coef[0][i] * x0a);
      const float vb = fmaf(aux->coef[1][i + 1], x1b, aux->coef[0][i + 1] * x0b);
      const float got = __shfl_xor_sync(0xffffffffu, odd ? va : vb, 1);
      if (odd)
        *reinterpret_cast<uint32_t*>(om + (i + 1) * D + d - 1) = pack_bf16x2(got, vb);
      else
        *reinterpret_cast<uint32_t*>(om + i * D + d) = pack_bf16x2(va, got);
    }
  } else {
    const int sp = warp & 3, jb = warp >> 2;
    const uint32_t tl = tmem + ((uint32_t)(32 * sp) << 16);
    const int d = 128 * jb + 32 * sp + lane;
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
        __nv_bfloat16* om = a.out + int64_t(mrow) * H * D + d;
#pragma unroll
        for (int i = 0; i < 32; ++i) om[(32 * hf + i) * D] = f2bf(o[i] * aux->f[32 * hf + i]);
      } else if (a.part_ob) {
        __nv_bfloat16* pb = a.part_ob + (int64_t(split) * a.M + mrow) * H * D + d;
#pragma unroll
        for (int i = 0; i < 32; ++i) pb[(32 * hf + i) * D] = f2bf(o[i] * aux->f[32 * hf + i]);
      } else {
        float* po = a.part_o + (int64_t(split) * a.M + mrow) * H * D + d;
#pragma unroll
        for (int i = 0; i < 32; ++i) po[(32 * hf + i) * D] = o[i];
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
