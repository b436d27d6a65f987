// The decode-step projections around the path on the tcgen05 tensor cores:
//   Y[b, g*N + n] = bf16( sum_k X[b, g*K + k] * W[g*N + n, k] )   b < B, n < N, g < G
// with an optional interleaved rotary on the last rope_dim columns of every
// head_dim block of Y (applied to the bf16-rounded product, then rounded
// again, as the reference's matmul followed by its rotary kernel does) and
// an optional fp32 output (of the bf16-rounded value).
//
// Reference call sites: the fused compressor wkv || wgate matmul
// (inference.py:4954-4966), the indexer's wq_b + rotary Lk-D-idx-q kernel and
// weights_proj (5177-5185, 5226-5258), the attention's wq_a / wq_b / wkv
// (5934-5960) and the output side's head-grouped wo_a and wo_b (6096-6126).
//
// At decode a projection is weight-streaming: B is a few token rows while W
// is megabytes, so the kernel reads every weight byte once, from as many SMs
// as the shape allows, and keeps the tensor pipe fed from the weight stream.
//
// Weight layout.  The weights are static, so they are stored once (at module
// set-up, dsa_linear_pack) as the tiles the tensor cores read: per (group g,
// 128-row tile t, 64-wide k-block kb) 16 KB holding rows n = 128 t + r
// (zero past N) and k = 64 kb + 8 c + e at byte r*128 + ((c ^ (r & 7)) * 16)
// + 2e - the 128-byte swizzle of a K-major operand - tiles in (g, t, kb)
// order.  A CTA's k-range of an item is then one contiguous run of HBM that
// it streams with 16 KB bulk copies (a row-major W read as [128 x 64] boxes
// touches 128 separate 128-B pieces per box and streams markedly slower).
//
// A work item is (group g, 128 weight rows); with a split of C > 1 the C CTAs
// of a thread-block cluster share an item, each over its own 1/C of K, and
// reduce their fp32 partials through distributed shared memory:
//   warp 0      producer: per k-block the 16 KB weight tile (bulk copy, L2
//               evict-first: each byte is read once) and the [Bp x 64] slice
//               of X (2-D TMA; Bp = B rounded up to 16, rows past B zero
//               fill) into an NS-stage ring;
//   warp 1      MMA issuer: Y^T tile = W_tile . X^T, M = 128 weight rows,
//               N = Bp tokens, K = 16 per MMA, into one of two TMEM
//               accumulators (the epilogue of item i overlaps item i + 1);
//   warps 2-5   epilogue, thread = weight row (TMEM lane).  C = 1: the Bp
//               token values of its row from TMEM -> rounding / rotary (the
//               pair partner of an interleaved rotary sits in the neighbouring
//               lane) -> Y, consecutive lanes writing consecutive columns.
//               C > 1: token rows are owned in C slices (CTA r owns rows
//               [r R, (r+1) R), R = ceil(B / C)); every CTA stores its partial
//               of each row straight into the owner's buffer [C][R][128] fp32
//               (remote shared-memory stores), the owner sums the C partials
//               of its rows in cluster-rank order - the same sum on every
//               run - and applies the C = 1 epilogue math.
// Cross-CTA ordering uses mbarriers in every CTA: `ready` (one release
// arrival from each CTA of the cluster per item) before an owner reads its
// buffer, `freed` (one from each owner) before a CTA stores into the owners'
// buffers for its next item; the cluster barrier is arrived at after the
// barrier initialisation and waited on before the first remote access, and
// a full cluster barrier at exit keeps every CTA resident while a peer may
// still touch its shared memory.  No TMA or bulk load uses multicast.
#include "common.cuh"
#include "tc05.cuh"
#include "tma.cuh"

#include <algorithm>
#include <cstring>
#include <type_traits>

namespace dsa {
namespace lin {

constexpr int TILE_N = 128;
constexpr int KBW = 64;                    // k per stage: one 128-B swizzled k-block
constexpr int kMaxStages = 12;
constexpr int THREADS = 192;
constexpr int kMaxB = 128;                 // token rows per launch (MMA N <= 256; two accumulators)
constexpr int kMaxSplit = 16;              // CTAs per cluster (16 needs the non-portable opt-in)
constexpr int kWBytes = TILE_N * KBW * 2;  // 16 KB
constexpr int kSmemBytes = 232448;         // the whole per-CTA budget: one CTA per SM
constexpr int kAuxBytes = 256;
constexpr uint32_t kTmemCols = 256;        // 2 accumulators x up to 128 columns

struct Args {
  const uint8_t* w;          // packed weight tiles
  void* y;
  int64_t ld_y;
  int B, Bp, N, K, G, n_tiles;
  int split;                 // C: CTAs per item (cluster size), each over 1/C of K
  int rows_per;              // R = ceil(B / C): token rows each CTA of a cluster finishes
  int n_stages;              // ring depth
  int tma_store;             // Y tiles leave through a TMA store (else per-element stores)
  uint32_t stage_bytes;      // 16 KB of W + Bp x 128 B of X
  uint32_t part_off;         // split > 1: this CTA's partial [Bp][128] fp32
  uint32_t recv_off;         // split > 1: the owned rows' partials [C][R][128] fp32
  uint32_t out_off;          // Y staging [rows][128] (bf16 or fp32)
  uint32_t rope_off;         // rotary factors (cos, sin) [rope_rows][rope_dim / 2] of the finished rows
  int rope_rows;
  uint32_t aux_off;
  int out_f32;
  const float* cos;
  const float* sin;
  int n_pos;
  const int32_t* pos;
  int head_dim, rope_dim;
  int rope_col0;             // the rotary covers columns >= rope_col0 of each group, head blocks from there
  int32_t* status;
  long long wait_limit;
};

struct Aux {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t ready;
  uint64_t freed;
  uint32_t tmem_base;
};
static_assert(sizeof(Aux) <= kAuxBytes, "aux block");

// ---- bulk copies (no multicast)
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// one contiguous weight tile, global -> this CTA
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}
// this CTA's shared memory -> a peer's (cluster addresses for dst and bar)
__device__ __forceinline__ void bulk_to_peer(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst),
               "r"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// Y tile store: box [128 cols, rows, 1 group] at (x, y, z)
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// ---- cluster helpers (distributed shared memory)
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded, like tc::mbar_wait: a lost arrival ends in an error status
__device__ __forceinline__ void mbar_wait_cluster(uint32_t bar, uint32_t parity, int32_t* status,
                                                  long long limit) {
  if (mbar_try_wait_cluster(bar, parity)) return;
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (clock64() - t0 > limit) {
      if (status) atomicOr(status, 2);
      return;
    }
  }
}

// The epilogue runs 4 warps on an SM: its speed is instruction latency, so
// values are finished and stored CNT at a time with independent chains
// (one CTA per SM leaves nothing else to hide a serial chain behind).
//
// bf16 rounding of CNT token rows' values of this thread's weight row, then
// (kRope, rope columns) the interleaved rotary: the pair partner is the
// neighbouring lane's value of the same token row.
template <bool kRope, int CNT>
__device__ __forceinline__ void finish_rows(const float2* rtab, int half, int n, bool rope, int kpair, float* v) {
#pragma unroll
  for (int i = 0; i < CNT; ++i) v[i] = bf2f(f2bf(v[i]));  // the matmul's bf16 result
  if constexpr (kRope) {
    float partner[CNT];
#pragma unroll
    for (int i = 0; i < CNT; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, v[i], 1);
    if (rope) {
#pragma unroll
      for (int i = 0; i < CNT; ++i) {
        const float2 f = rtab[i * half + kpair];  // (cos, sin) of token row i at this pair
        // pair (a, c) = (even, odd): a cos - c sin, a sin + c cos
        v[i] = (n & 1) ? __fadd_rn(__fmul_rn(partner[i], f.y), __fmul_rn(v[i], f.x))
                       : __fsub_rn(__fmul_rn(v[i], f.x), __fmul_rn(partner[i], f.y));
      }
    }
  }
}

// (cos, sin) of every (token row, rotary pair) the CTA finishes, gathered
// once per launch into shared memory by the epilogue warps while the weight
// stream runs: rows [b0, b0 + rows); positions outside [0, n_pos) clamped
// and flagged (status bit 1)
__device__ __forceinline__ void load_rope_table(const Args& a, float2* rtab, int b0, int rows, int t) {
  const int half = a.rope_dim >> 1;
  const int total = rows * half;
  bool bad = false;
  for (int i0 = t; i0 < total; i0 += 128 * 8) {
    int p[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * 128;
      const int b = b0 + (i < total ? i / half : 0);
      p[u] = a.pos[min(b, a.B - 1)];
      if (i < total && b < a.B && (p[u] < 0 || p[u] >= a.n_pos)) bad = true;
      p[u] = min(max(p[u], 0), a.n_pos - 1);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * 128;
      if (i < total) {
        const int k = i % half;
        rtab[i] = make_float2(a.cos[int64_t(p[u]) * half + k], a.sin[int64_t(p[u]) * half + k]);
      }
    }
  }
  if (bad && a.status) atomicOr(a.status, 1);
}

// CNT finished values of rows [b0, b0 + CNT): into the staging tile rows
// [srow, srow + CNT) (TMA store), or straight to Y (rows below B only)
template <bool kF32, int CNT>
__device__ __forceinline__ void put_rows(const Args& a, uint8_t* ostage, int srow, int nr, int b0, int64_t col,
                                         bool n_ok, const float* v) {
  using T = typename std::conditional<kF32, float, __nv_bfloat16>::type;
  if (a.tma_store) {
    T* o = reinterpret_cast<T*>(ostage) + srow * TILE_N + nr;
#pragma unroll
    for (int i = 0; i < CNT; ++i) {
      if constexpr (kF32) o[i * TILE_N] = bf2f(f2bf(v[i]));
      else o[i * TILE_N] = f2bf(v[i]);
    }
  } else if (n_ok) {
    T* o = static_cast<T*>(a.y) + int64_t(b0) * a.ld_y + col;
#pragma unroll
    for (int i = 0; i < CNT; ++i) {
      if (b0 + i < a.B) {
        if constexpr (kF32) o[i * a.ld_y] = bf2f(f2bf(v[i]));
        else o[i * a.ld_y] = f2bf(v[i]);
      }
    }
  }
}

template <bool kRope, bool kF32>
__global__ void __launch_bounds__(THREADS, 1) linear_tc_kernel(const Args a,
                                                               const __grid_constant__ CUtensorMap tm_x,
                                                               const __grid_constant__ CUtensorMap tm_y) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Aux* aux = reinterpret_cast<Aux*>(smem + a.aux_off);
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = a.split;
  const int rank = C > 1 ? int(cluster_rank()) : 0;
  const int cid = blockIdx.x / C, n_cl = gridDim.x / C;
  const int n_items = a.G * a.n_tiles;
  const int nkb = a.K / KBW;
  const int kb0 = rank * nkb / C, kb1 = (rank + 1) * nkb / C;  // this CTA's k-blocks (C <= nkb)
  const int NS = a.n_stages;
  const uint32_t x_bytes = uint32_t(a.Bp) * KBW * 2;
  const uint32_t idesc = tc::idesc_bf16(128, a.Bp, false, false);

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
    tc::mbar_init(smem_u32(&aux->ready), 1);  // the owner's own arrival + the peers' copied bytes
    tc::mbar_init(smem_u32(&aux->freed), C);  // one arrival from every owner
    tc::mbar_fence_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  // every peer's barriers must be initialised before the first remote
  // access: arrive now, wait just before that access (epilogue) or at exit
  if (C > 1) cluster_arrive();
  tc::fence_after_sync();
  const uint32_t tmem = aux->tmem_base;
  const uint8_t* wbase = a.w;
  // the weights are not produced by the previous kernel: their first tiles
  // are requested before the dependency wait; X (the activations) after it
  int npre = 0;
  uint64_t policy = 0;
  if (warp == 0 && lane == 0) {
    policy = evict_first_policy();
    for (int item = cid; item < n_items && npre < NS; item += n_cl) {
      const uint8_t* wt = wbase + (int64_t(item) * nkb + kb0) * kWBytes;
      for (int kb = kb0; kb < kb1 && npre < NS; ++kb, ++npre, wt += kWBytes) {
        const uint32_t fb = smem_u32(&aux->full[npre]);
        tma::mbar_arrive_expect_tx(fb, kWBytes + x_bytes);
        bulk_load(sbase + npre * a.stage_bytes, wt, kWBytes, fb, policy);
      }
    }
  }
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      tma::prefetch_map(&tm_x);
      int it = 0;
      for (int item = cid; item < n_items; item += n_cl) {
        const int g = item / a.n_tiles;
        const uint8_t* wt = wbase + (int64_t(item) * nkb + kb0) * kWBytes;
        for (int kb = kb0; kb < kb1; ++kb, ++it, wt += kWBytes) {
          const int s = it % NS;
          const uint32_t st = sbase + s * a.stage_bytes;
          const uint32_t fb = smem_u32(&aux->full[s]);
          if (it >= npre) {
            if (it >= NS) tc::mbar_wait(smem_u32(&aux->empty[s]), ((it / NS) - 1) & 1, a.status, 2, a.wait_limit);
            tma::mbar_arrive_expect_tx(fb, kWBytes + x_bytes);
            bulk_load(st, wt, kWBytes, fb, policy);
          }
          tma::load_2d(st + kWBytes, &tm_x, g * a.K + kb * KBW, 0, fb);
        }
      }
    }
    __syncwarp();
    if (C > 1) cluster_wait();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0, li = 0;
      for (int item = cid; item < n_items; item += n_cl, ++li) {
        const int acc = li & 1;
        if (li >= 2) tc::mbar_wait(smem_u32(&aux->acc_empty[acc]), ((li - 2) >> 1) & 1, a.status, 2, a.wait_limit);
        tc::fence_after_sync();
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % NS;
          tc::mbar_wait(smem_u32(&aux->full[s]), (it / NS) & 1, a.status, 2, a.wait_limit);
          tc::fence_after_sync();
          const uint32_t st = sbase + s * a.stage_bytes;
#pragma unroll
          for (int ks = 0; ks < KBW / 16; ++ks) {
            const uint64_t ad = tc::smem_desc(st + ks * 32, 16, 1024, tc::kLayoutSw128);
            const uint64_t bd = tc::smem_desc(st + kWBytes + ks * 32, 16, 1024, tc::kLayoutSw128);
            tc::mma_bf16(tmem + uint32_t(kMaxB) * acc, ad, bd, idesc, (kb > kb0 || ks) ? 1u : 0u);
          }
          tc::mma_commit(smem_u32(&aux->empty[s]));
        }
        tc::mma_commit(smem_u32(&aux->acc_full[acc]));
      }
    }
    __syncwarp();
    if (C > 1) cluster_wait();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int quarter = warp & 3;  // TMEM lanes [32 quarter, 32 quarter + 32)
    const int nr = quarter * 32 + lane;  // this thread's row of the 128-row tile
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    float* part = reinterpret_cast<float*>(smem + a.part_off);
    const float* recv = reinterpret_cast<const float*>(smem + a.recv_off);
    uint8_t* ostage = smem + a.out_off;
    const int R = a.rows_per;
    const int b_lo = rank * R, b_hi = min(a.B, b_lo + R);
    const bool lead = tid == 64;
    const float2* rtab = reinterpret_cast<const float2*>(smem + a.rope_off);
    const int half = a.rope_dim >> 1;
    if constexpr (kRope) {
      // the finished rows: all Bp (C = 1) or the owned slice
      load_rope_table(a, reinterpret_cast<float2*>(smem + a.rope_off), C > 1 ? b_lo : 0, a.rope_rows, tid - 64);
      tc::named_bar_sync(1, 128);
    }
    if (lead && a.tma_store) tma::prefetch_map(&tm_y);
    if (C > 1) cluster_wait();
    int li = 0;
    for (int item = cid; item < n_items; item += n_cl, ++li) {
      const int acc = li & 1;
      const int g = item / a.n_tiles, t = item - g * a.n_tiles;
      const int n = t * TILE_N + nr;  // this thread's weight row
      const bool n_ok = n < a.N;
      // rotary: the interleaved pair (n, n ^ 1) of a rope column of a head
      const int nn = n - a.rope_col0;
      const int hd = (a.head_dim > 0 && nn >= 0) ? nn % a.head_dim : 0;
      const bool rope = a.rope_dim > 0 && nn >= 0 && n < a.N && hd >= a.head_dim - a.rope_dim;
      const int kpair = (hd - (a.head_dim - a.rope_dim)) >> 1;
      const int64_t col = int64_t(g) * a.N + n;
      // the previous item's Y tile has left the staging buffer
      if (a.tma_store && li > 0) {
        if (lead) bulk_wait_read();
        tc::named_bar_sync(1, 128);
      }
      tc::mbar_wait(smem_u32(&aux->acc_full[acc]), (li >> 1) & 1, a.status, 2, a.wait_limit);
      tc::fence_after_sync();
      if (C == 1) {
        for (int c0 = 0; c0 < a.Bp; c0 += 32) {
          float v[32];
          tc::tmem_ld32(trow + uint32_t(kMaxB) * acc + c0, v);
          tc::tmem_wait_ld();
          finish_rows<kRope, 32>(rtab + c0 * half, half, n, rope, kpair, v);
          put_rows<kF32, 32>(a, ostage, c0, nr, c0, col, n_ok, v);
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(smem_u32(&aux->acc_empty[acc]));
        if (a.tma_store) {
          tc::fence_proxy_async();
          tc::named_bar_sync(1, 128);
          if (lead) tma_store_3d(&tm_y, smem_u32(ostage), t * TILE_N, 0, g);
        }
        continue;
      }
      // split: this CTA's partial of every token row goes to the row's owner
      // (one bulk copy per owner into its [rank] slot); then the owned rows
      // are summed over the C slots and finished
      if (li > 0) mbar_wait_cluster(smem_u32(&aux->freed), (li - 1) & 1, a.status, a.wait_limit);
      for (int c0 = 0; c0 < a.Bp; c0 += 32) {
        float v[32];
        tc::tmem_ld32(trow + uint32_t(kMaxB) * acc + c0, v);
        tc::tmem_wait_ld();
        float* pr = part + c0 * TILE_N + nr;  // part holds Bp rows: no guard
#pragma unroll
        for (int i = 0; i < 32; ++i) pr[i * TILE_N] = v[i];
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(smem_u32(&aux->acc_empty[acc]));
      tc::fence_proxy_async();  // the partial is read by the copy engine
      tc::named_bar_sync(1, 128);
      if (lead) {
        // expect C copies of the owned rows, then send every owner its rows
        tma::mbar_arrive_expect_tx(smem_u32(&aux->ready), uint32_t(C * max(0, b_hi - b_lo)) * TILE_N * 4u);
        for (int q = 0; q < C; ++q) {
          const int rows = min(R, a.B - q * R);
          if (rows <= 0) continue;
          bulk_to_peer(mapa(smem_u32(recv) + uint32_t(rank * R) * TILE_N * 4u, q),
                       smem_u32(part) + uint32_t(q * R) * TILE_N * 4u, uint32_t(rows) * TILE_N * 4u,
                       mapa(smem_u32(&aux->ready), q));
        }
      }
      mbar_wait_cluster(smem_u32(&aux->ready), li & 1, a.status, a.wait_limit);
      // 8 owned rows at a time, 8 independent sums, C slots in rank order
      const int nrows = b_hi - b_lo;
      for (int lb0 = 0; lb0 < nrows; lb0 += 8) {
        float v[8];
        const float* rp[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[j] = 0.f;
          rp[j] = recv + min(lb0 + j, R - 1) * TILE_N + nr;  // rows past the slice: any in-slot row
        }
        for (int q = 0; q < C; ++q) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] += rp[j][q * R * TILE_N];
        }
        finish_rows<kRope, 8>(rtab + lb0 * half, half, n, rope, kpair, v);
        if (lb0 + 8 <= nrows) {
          put_rows<kF32, 8>(a, ostage, lb0, nr, b_lo + lb0, col, n_ok, v);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (lb0 + j < nrows) put_rows<kF32, 1>(a, ostage, lb0 + j, nr, b_lo + lb0 + j, col, n_ok, v + j);
        }
      }
      if (a.tma_store) tc::fence_proxy_async();
      tc::named_bar_sync(1, 128);
      if (lead && a.tma_store && b_hi > b_lo) tma_store_3d(&tm_y, smem_u32(ostage), t * TILE_N, b_lo, g);
      // this CTA's received partials are consumed: every sender may send again
      if (warp == 2 && lane < C) mbar_arrive_cluster(mapa(smem_u32(&aux->freed), lane));
    }
    if (lead) bulk_wait_read();  // the Y tiles have left shared memory
  }
  tc::fence_before_sync();
  __syncthreads();
  if (C > 1) {  // no CTA leaves while a peer may still touch its shared memory
    cluster_arrive();
    cluster_wait();
  }
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// W [G*N, K] row-major -> the tile layout above, one 16-byte chunk a thread
__global__ void pack_kernel(const __nv_bfloat16* __restrict__ w, uint8_t* __restrict__ out, int N, int K, int G,
                            int n_tiles, int64_t chunks) {
  const int nkb = K / KBW;
  for (int64_t id = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; id < chunks; id += int64_t(gridDim.x) * blockDim.x) {
    const int64_t tile = id >> 10;
    const int within = int(id & 1023);
    const int r = within >> 3, c = within & 7;
    const int kb = int(tile % nkb);
    const int64_t gt = tile / nkb;
    const int t = int(gt % n_tiles), g = int(gt / n_tiles);
    const int n = t * TILE_N + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n < N) v = *reinterpret_cast<const uint4*>(w + (int64_t(g) * N + n) * K + kb * KBW + c * 8);
    *reinterpret_cast<uint4*>(out + tile * kWBytes + r * 128 + ((c ^ (r & 7)) << 4)) = v;
  }
}

// clusters of C CTAs that can be resident at once (one CTA per SM), per device
int max_clusters(int C) {
  static int cache[64][kMaxSplit + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 0;
  if (cache[dev][C] == 0) {
    int n = 0;
    if (C == 1) {
      n = num_sms();
    } else {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(C);
      cfg.blockDim = dim3(THREADS);
      cfg.dynamicSmemBytes = kSmemBytes;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = C;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, linear_tc_kernel<false, false>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
    }
    cache[dev][C] = n > 0 ? n : -1;
  }
  return cache[dev][C] > 0 ? cache[dev][C] : 0;
}

// the split with the fewest k-blocks on the busiest CTA, counting a fixed
// cost per item (2 k-blocks: set-up and epilogue) and per split reduction
// (3 more: the partial exchange and the owners' sums), among the splits
// whose clusters fit.  Measured on B200 at B = 64: 40960 x 1024 (320 items)
// 24.6 us unsplit against 28.8 us with C = 2 (5 waves of 74 clusters).
int pick_split(int items, int nkb) {
  int best = 1;
  long best_cost = -1;
  for (int C = 1; C <= std::min(kMaxSplit, nkb); ++C) {
    const int mc = max_clusters(C);
    if (mc <= 0) continue;
    const int n_cl = std::min(items, mc);
    const long waves = (items + n_cl - 1) / n_cl;
    const long per = (nkb + C - 1) / C;
    const long cost = waves * (per + 2 + (C > 1 ? 3 : 0));
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = C;
    }
  }
  return best;
}

}  // namespace lin
}  // namespace dsa

using namespace dsa;

extern "C" size_t dsa_linear_packed_bytes(int N, int K, int G) {
  if (N <= 0 || K <= 0 || G <= 0 || K % lin::KBW) return 0;
  const int64_t tiles = int64_t(G) * ((N + lin::TILE_N - 1) / lin::TILE_N) * (K / lin::KBW);
  return size_t(tiles) * lin::kWBytes;
}

extern "C" int dsa_linear_pack(const void* w, int N, int K, int G, void* packed, size_t packed_bytes,
                               dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(w && packed, "linear_pack: null w/packed");
  DSA_CHECK_ARG(N > 0 && K > 0 && G >= 1 && K % lin::KBW == 0, "linear_pack: bad N/K/G (K a multiple of %d)",
                lin::KBW);
  DSA_CHECK_ARG(aligned(w, 16) && aligned(packed, 16), "linear_pack: w/packed must be 16-byte aligned");
  const size_t need = dsa_linear_packed_bytes(N, K, G);
  DSA_CHECK_ARG(packed_bytes >= need, "linear_pack: packed buffer %zu bytes < %zu", packed_bytes, need);
  const int n_tiles = (N + lin::TILE_N - 1) / lin::TILE_N;
  const int64_t chunks = int64_t(need / 16);
  const int grid = int(std::min<int64_t>((chunks + 255) / 256, int64_t(num_sms()) * 16));
  lin::pack_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(w), static_cast<uint8_t*>(packed), N, K, G, n_tiles, chunks);
  DSA_CHECK_LAUNCH("linear_pack");
  return DSA_OK;
}

extern "C" int dsa_linear(const void* x, int64_t ld_x, const void* w_packed, void* y, int64_t ld_y, int B, int N,
                          int K, int G, int out_f32, const float* cos, const float* sin, int n_pos,
                          const int32_t* pos, int head_dim, int rope_dim, int rope_col0, int32_t* status,
                          dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(x && w_packed && y, "linear: null x/w/y");
  DSA_CHECK_ARG(B >= 0 && N > 0 && K > 0 && G >= 1, "linear: bad B/N/K/G");
  DSA_CHECK_ARG(K % lin::KBW == 0, "linear: K=%d must be a multiple of %d", K, lin::KBW);
  DSA_CHECK_ARG(ld_x >= int64_t(G) * K && ld_x % 8 == 0 && aligned(x, 16) && aligned(w_packed, 16),
                "linear: x needs 16-byte alignment and a row stride >= G*K, a multiple of 8; w 16-byte aligned");
  DSA_CHECK_ARG(ld_y >= int64_t(G) * N, "linear: ld_y < G*N");
  DSA_CHECK_ARG(int64_t(G) * N < (1ll << 31) && int64_t(G) * K < (1ll << 31), "linear: G*N or G*K too large");
  if (rope_dim > 0) {
    DSA_CHECK_ARG(cos && sin && pos && n_pos > 0, "linear: rotary needs cos/sin tables and positions");
    DSA_CHECK_ARG(head_dim > 0 && rope_dim % 2 == 0 && rope_dim <= head_dim && head_dim % 32 == 0 &&
                      rope_col0 >= 0 && rope_col0 % 2 == 0 && rope_col0 < N && (N - rope_col0) % head_dim == 0,
                  "linear: rotary needs head_dim | N - rope_col0 (rope_col0 even), head_dim a multiple of 32, "
                  "an even rope_dim <= head_dim");
  }
  if (B == 0) return DSA_OK;
  static int attr_dev[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_dev[dev]) {
    for (auto k : {lin::linear_tc_kernel<false, false>, lin::linear_tc_kernel<false, true>,
                   lin::linear_tc_kernel<true, false>, lin::linear_tc_kernel<true, true>}) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, lin::kSmemBytes);
      cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    }
    attr_dev[dev] = 1;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int n_tiles = (N + lin::TILE_N - 1) / lin::TILE_N;
  const int items = G * n_tiles;
  const int nkb = K / lin::KBW;
  const int C_pick = lin::pick_split(items, nkb);
  // token rows in chunks of up to kMaxB (one accumulator column each)
  for (int b0 = 0; b0 < B; b0 += lin::kMaxB) {
    const int nb = std::min(lin::kMaxB, B - b0);
    lin::Args a{};
    a.w = static_cast<const uint8_t*>(w_packed);
    a.y = static_cast<void*>(static_cast<uint8_t*>(y) + int64_t(b0) * ld_y * (out_f32 ? 4 : 2));
    a.ld_y = ld_y;
    a.B = nb;
    a.Bp = (nb + 15) / 16 * 16;
    if (a.Bp < 32) a.Bp = 32;  // the epilogue reads accumulator columns 32 at a time
    a.N = N;
    a.K = K;
    a.G = G;
    a.n_tiles = n_tiles;
    const int es = out_f32 ? 4 : 2;
    const int64_t y_off = int64_t(b0) * ld_y * es;
    // the picked split, or a smaller one where its buffers leave the weight
    // ring fewer than 2 stages (large B with a deep split)
    int C = C_pick;
    for (;; --C) {
      a.split = C;
      a.rows_per = (nb + C - 1) / C;
      a.stage_bytes = uint32_t(lin::kWBytes + a.Bp * lin::KBW * 2);
      // Y tiles leave through a TMA store when Y's rows and groups start on
      // 16-byte boundaries; otherwise element by element
      a.tma_store = aligned(y, 16) && (ld_y * es) % 16 == 0 && (G == 1 || (int64_t(N) * es) % 16 == 0) ? 1 : 0;
      // rows the epilogue touches: accumulator columns go 32 at a time (C = 1,
      // and the partial writes of C > 1), owned rows 8 at a time (C > 1)
      const int rows32 = (a.Bp + 31) / 32 * 32;
      const int done_rows = C > 1 ? (a.rows_per + 7) / 8 * 8 : rows32;
      a.rope_rows = done_rows;
      const uint32_t part_bytes = C > 1 ? uint32_t(rows32) * lin::TILE_N * 4 : 0;
      const uint32_t recv_bytes = C > 1 ? uint32_t(C * a.rows_per) * lin::TILE_N * 4 : 0;
      const uint32_t out_bytes = a.tma_store ? (uint32_t(done_rows) * lin::TILE_N * es + 127u) & ~127u : 0;
      const uint32_t rope_bytes = rope_dim > 0 ? uint32_t(done_rows) * uint32_t(rope_dim / 2) * 8u : 0;
      const uint32_t fixed = uint32_t(1024 + lin::kAuxBytes) + part_bytes + recv_bytes + out_bytes + rope_bytes;
      a.n_stages = fixed < uint32_t(lin::kSmemBytes)
                       ? std::min<int>(lin::kMaxStages, int((uint32_t(lin::kSmemBytes) - fixed) / a.stage_bytes))
                       : 0;
      a.part_off = uint32_t(a.n_stages) * a.stage_bytes;
      a.recv_off = a.part_off + part_bytes;
      a.out_off = a.recv_off + recv_bytes;
      a.rope_off = a.out_off + out_bytes;
      a.aux_off = (a.rope_off + rope_bytes + 15u) & ~15u;
      if (C == 1 || (a.n_stages >= 2 && lin::max_clusters(C) > 0)) break;
    }
    const int n_cl = std::min(items, C == 1 ? num_sms() : lin::max_clusters(C));
    const int out_rows = C > 1 ? a.rows_per : a.Bp;  // the Y box
    a.out_f32 = out_f32;
    a.cos = cos;
    a.sin = sin;
    a.n_pos = n_pos;
    a.pos = pos ? pos + b0 : nullptr;
    a.head_dim = rope_dim > 0 ? head_dim : 0;
    a.rope_dim = rope_dim > 0 ? rope_dim : 0;
    a.rope_col0 = rope_dim > 0 ? rope_col0 : 0;
    a.status = status;
    a.wait_limit = wait_limit_cycles();
    if (n_cl <= 0 || a.n_stages < 2 || a.aux_off + lin::kAuxBytes + 1024 > uint32_t(lin::kSmemBytes)) {
      set_error("linear: no launch configuration fits");
      return DSA_ERR_CUDA;
    }
    CUtensorMap tm_x, tm_y;
    memset(&tm_y, 0, sizeof(tm_y));
    if (!tma::make_2d_bf16(&tm_x, static_cast<const __nv_bfloat16*>(x) + int64_t(b0) * ld_x, uint64_t(G) * K,
                           uint64_t(nb), uint64_t(ld_x) * 2, lin::KBW, uint32_t(a.Bp))) {
      set_error("linear: cuTensorMapEncodeTiled failed");
      return DSA_ERR_CUDA;
    }
    if (a.tma_store) {
      // Y as [G][rows][N]: column n of group g at g*N + n, rows ld_y apart
      tma::EncodeTiledFn fn = tma::encode_fn();
      const cuuint64_t dims[3] = {uint64_t(N), uint64_t(nb), uint64_t(G)};
      const cuuint64_t strides[2] = {uint64_t(ld_y) * es, G > 1 ? uint64_t(N) * es : uint64_t(ld_y) * es * nb};
      const cuuint32_t box[3] = {uint32_t(lin::TILE_N), uint32_t(out_rows), 1};
      const cuuint32_t estr[3] = {1, 1, 1};
      if (!fn || fn(&tm_y, out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                    static_cast<uint8_t*>(y) + y_off, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        set_error("linear: cuTensorMapEncodeTiled (Y) failed");
        return DSA_ERR_CUDA;
      }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_cl * C);
    cfg.blockDim = dim3(lin::THREADS);
    cfg.dynamicSmemBytes = lin::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = C;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = C > 1 ? 2 : 1;
    auto kern = rope_dim > 0 ? (out_f32 ? lin::linear_tc_kernel<true, true> : lin::linear_tc_kernel<true, false>)
                             : (out_f32 ? lin::linear_tc_kernel<false, true> : lin::linear_tc_kernel<false, false>);
    cudaLaunchKernelEx(&cfg, kern, a, tm_x, tm_y);
    DSA_CHECK_LAUNCH("linear");
  }
  return DSA_OK;
}
