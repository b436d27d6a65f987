// attn.sparse: index gather + sink-softmax attention over the selected rows.
//
// Reference: DeviceSparseAttn.forward_device (inference.py:4459-4501) with
// the index->mask conversion _idxs_int_tile_to_idxs_and_mask (4444-4457)
// folded in: a -1 index contributes nothing, the per-head sink logit joins
// the softmax denominator once.  K = V = the 512-d latent row (MQA).
//
// Flash-decoding layout: one CTA per (query row, key split).  The query's
// 64 heads x 512 dims (64 KB) stay in shared memory; the selected kv rows
// are gathered 64 at a time by 16-byte cp.async (keyed by the index list;
// masked / padded rows zero-fill) into a double-buffered, XOR-swizzled
// 2 x 64 KB ring.  Per tile, warps 0-3 compute S = Q K^T for 16 heads each
// on the tensor cores, run the online softmax in registers and publish P
// (bf16) plus the per-head rescale factor; then all 8 warps accumulate
// O += P V for a 16-head x 256-dim block each.  Splits of one query row are
// merged by lse_combine_kernel (sink counted once).  The kernel reads each
// gathered row exactly once from HBM; its roofline is the gather stream.
#include "common.cuh"
#include "sparse_attn_tc.cuh"
#include <stdlib.h>
#include <mutex>

namespace dsa {

constexpr int kSaH = 64;
constexpr int kSaD = 512;
constexpr int kSaTile = 64;
constexpr int kSaThreads = 256;
constexpr int kSaRow = kSaD * 2;  // 1024 B per head / per kv row
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

constexpr int kSaSmemQ = kSaH * kSaRow;           // 64 KB
constexpr int kSaSmemK = 2 * kSaTile * kSaRow;    // 128 KB
constexpr int kSaSmemP = kSaH * kSaTile * 2;      // 8 KB
constexpr int kSaSmem = kSaSmemQ + kSaSmemK + kSaSmemP + 3 * kSaH * 4 + 2 * kSaTile * 4;

__device__ __forceinline__ uint32_t sa_swz(int r, int c) { return r * kSaRow + ((c ^ (r & 7)) << 4); }
__device__ __forceinline__ uint32_t sp_swz(int r, int c) { return r * (kSaTile * 2) + ((c ^ (r & 7)) << 4); }

struct SaArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* kv;
  int64_t kv_bstride;
  int64_t kv_rows;
  const int32_t* idx;
  int64_t ld_idx;
  const float* sink;
  __nv_bfloat16* out;   // final mode
  float* lse;           // final mode, may be null
  float* part_ml;       // partial mode [nsplit, M, H, 2]
  float* part_o;        // partial mode [nsplit, M, H, D]
  int32_t* status;
  int S;                // query rows per batch element
  int M;                // total query rows
  int K;
  int tiles_per_split;
  float scale_log2;     // softmax scale * log2(e)
  int final_mode;
};

__global__ void __launch_bounds__(kSaThreads, 1) sparse_attn_mma_kernel(SaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kSaSmemQ;
  uint8_t* sP = sK + kSaSmemK;
  float* s_alpha = reinterpret_cast<float*>(sP + kSaSmemP);
  float* s_m = s_alpha + kSaH;
  float* s_l = s_m + kSaH;
  int* s_valid = reinterpret_cast<int*>(s_l + kSaH);  // [2][64]

  const int m = blockIdx.y, split = blockIdx.x;
  const int b = m / a.S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j_begin = split * a.tiles_per_split * kSaTile;
  const int j_end = min(a.K, j_begin + a.tiles_per_split * kSaTile);
  const int ntiles = (j_end - j_begin + kSaTile - 1) / kSaTile;
  const __nv_bfloat16* kvb = a.kv + int64_t(b) * a.kv_bstride;
  const int32_t* idxr = a.idx + int64_t(m) * a.ld_idx;

  {  // Q -> smem
    const __nv_bfloat16* qm = a.q + int64_t(m) * kSaH * kSaD;
    for (int e = tid; e < kSaH * 64; e += kSaThreads) {
      const int r = e >> 6, c = e & 63;
      cp_async16(smem_u32(sQ + sa_swz(r, c)), qm + r * kSaD + c * 8, 16);
    }
  }
  auto load_tile = [&](int t, int stage) {
    uint8_t* dst = sK + stage * (kSaTile * kSaRow);
    const int c = tid & 63;
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int r = (tid >> 6) + 4 * i;
      const int j = j_begin + t * kSaTile + r;
      int id = (j < j_end) ? idxr[j] : -1;
      const bool valid = id >= 0;
      if (valid && id >= a.kv_rows) {
        if (a.status) atomicOr(a.status, 1);
        id = int(a.kv_rows - 1);
      }
      const __nv_bfloat16* src = kvb + int64_t(valid ? id : 0) * kSaD + c * 8;
      cp_async16(smem_u32(dst + sa_swz(r, c)), src, valid ? 16 : 0);
      if (c == 0) s_valid[stage * kSaTile + r] = valid ? 1 : 0;
    }
  };

  if (ntiles > 0) load_tile(0, 0);
  cp_async_commit();

  const int g = lane >> 2, qd = lane & 3;
  // softmax state for head rows 16w+g and 16w+g+8 (warps 0-3), replicated in the quad
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[32][4];
#pragma unroll
  for (int n = 0; n < 32; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[n][i] = 0.f;
  const int hg = warp & 3, dh = warp >> 2;

  for (int t = 0; t < ntiles; ++t) {
    const int stage = t & 1;
    if (t + 1 < ntiles) load_tile(t + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint8_t* tK = sK + stage * (kSaTile * kSaRow);
    const int* valid = s_valid + stage * kSaTile;

    if (warp < 4) {
      float acc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
#pragma unroll 4
      for (int ks = 0; ks < kSaD / 16; ++ks) {
        uint32_t af[4];
        ldmatrix_x4(smem_u32(sQ + sa_swz(warp * 16 + (lane & 15), 2 * ks + (lane >> 4))), af[0], af[1], af[2],
                    af[3]);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t r0, r1, r2, r3;
          ldmatrix_x4(smem_u32(tK + sa_swz(np * 16 + (lane & 7) + ((lane >> 4) << 3), 2 * ks + ((lane >> 3) & 1))),
                      r0, r1, r2, r3);
          const uint32_t b0[2] = {r0, r1}, b1[2] = {r2, r3};
          mma_bf16_16816(acc[2 * np], af, b0);
          mma_bf16_16816(acc[2 * np + 1], af, b1);
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool ok = valid[8 * n + 2 * qd + e] != 0;
          acc[n][e] = ok ? acc[n][e] * a.scale_log2 : -INFINITY;
          acc[n][2 + e] = ok ? acc[n][2 + e] * a.scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, acc[n][e]);
          mx1 = fmaxf(mx1, acc[n][2 + e]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float al0 = (mn0 == -INFINITY) ? 1.f : exp2f(m0 - mn0);
      const float al1 = (mn1 == -INFINITY) ? 1.f : exp2f(m1 - mn1);
      float rs0 = 0.f, rs1 = 0.f;
      const int h0 = warp * 16 + g, h1 = h0 + 8;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float p00 = acc[n][0] == -INFINITY ? 0.f : exp2f(acc[n][0] - mn0);
        const float p01 = acc[n][1] == -INFINITY ? 0.f : exp2f(acc[n][1] - mn0);
        const float p10 = acc[n][2] == -INFINITY ? 0.f : exp2f(acc[n][2] - mn1);
        const float p11 = acc[n][3] == -INFINITY ? 0.f : exp2f(acc[n][3] - mn1);
        rs0 += p00 + p01;
        rs1 += p10 + p11;
        *reinterpret_cast<uint32_t*>(sP + sp_swz(h0, n) + qd * 4) = pack_bf16x2(p00, p01);
        *reinterpret_cast<uint32_t*>(sP + sp_swz(h1, n) + qd * 4) = pack_bf16x2(p10, p11);
      }
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
      l0 = l0 * al0 + rs0;
      l1 = l1 * al1 + rs1;
      m0 = mn0;
      m1 = mn1;
      if (qd == 0) {
        s_alpha[h0] = al0;
        s_alpha[h1] = al1;
      }
    }
    __syncthreads();

    {  // O[16 heads x 256 dims] += P V for this warp's block
      const float al0 = s_alpha[hg * 16 + g], al1 = s_alpha[hg * 16 + g + 8];
#pragma unroll
      for (int n = 0; n < 32; ++n) {
        o[n][0] *= al0;
        o[n][1] *= al0;
        o[n][2] *= al1;
        o[n][3] *= al1;
      }
#pragma unroll
      for (int kk = 0; kk < kSaTile / 16; ++kk) {
        uint32_t af[4];
        ldmatrix_x4(smem_u32(sP + sp_swz(hg * 16 + (lane & 15), 2 * kk + (lane >> 4))), af[0], af[1], af[2],
                    af[3]);
#pragma unroll
        for (int np = 0; np < 16; ++np) {
          uint32_t r0, r1, r2, r3;
          const int key = 16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int ch = 32 * dh + 2 * np + (lane >> 4);
          ldmatrix_x4_trans(smem_u32(tK + sa_swz(key, ch)), r0, r1, r2, r3);
          const uint32_t b0[2] = {r0, r1}, b1[2] = {r2, r3};
          mma_bf16_16816(o[2 * np], af, b0);
          mma_bf16_16816(o[2 * np + 1], af, b1);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  if (warp < 4 && qd == 0) {
    s_m[warp * 16 + g] = m0;
    s_m[warp * 16 + g + 8] = m1;
    s_l[warp * 16 + g] = l0;
    s_l[warp * 16 + g + 8] = l1;
  }
  __syncthreads();

  const int h0 = hg * 16 + g, h1 = h0 + 8;
  const float mm[2] = {s_m[h0], s_m[h1]};
  const float ll[2] = {s_l[h0], s_l[h1]};
  if (a.final_mode) {
    float f[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int h = r ? h1 : h0;
      const float sk = a.sink[h] * kLog2e;
      const float M = fmaxf(mm[r], sk);
      const float w = (mm[r] == -INFINITY) ? 0.f : exp2f(mm[r] - M);
      const float L = ll[r] * w + exp2f(sk - M);
      f[r] = w / L;
      if (a.lse && dh == 0 && qd == 0) a.lse[int64_t(m) * kSaH + h] = (M + log2f(L)) * kLn2;
    }
    __nv_bfloat16* om = a.out + int64_t(m) * kSaH * kSaD;
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      const int d0 = dh * 256 + 8 * n + 2 * qd;
      *reinterpret_cast<uint32_t*>(om + h0 * kSaD + d0) = pack_bf16x2(o[n][0] * f[0], o[n][1] * f[0]);
      *reinterpret_cast<uint32_t*>(om + h1 * kSaD + d0) = pack_bf16x2(o[n][2] * f[1], o[n][3] * f[1]);
    }
  } else {
    const int64_t base = int64_t(split) * a.M + m;
    if (dh == 0 && qd == 0) {
      a.part_ml[(base * kSaH + h0) * 2 + 0] = mm[0] == -INFINITY ? -INFINITY : mm[0] * kLn2;
      a.part_ml[(base * kSaH + h0) * 2 + 1] = ll[0];
      a.part_ml[(base * kSaH + h1) * 2 + 0] = mm[1] == -INFINITY ? -INFINITY : mm[1] * kLn2;
      a.part_ml[(base * kSaH + h1) * 2 + 1] = ll[1];
    }
    float* po = a.part_o + base * kSaH * kSaD;
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      const int d0 = dh * 256 + 8 * n + 2 * qd;
      *reinterpret_cast<float2*>(po + h0 * kSaD + d0) = make_float2(o[n][0], o[n][1]);
      *reinterpret_cast<float2*>(po + h1 * kSaD + d0) = make_float2(o[n][2], o[n][3]);
    }
  }
}

// Merge of the split-K partials of each query row: final mode writes
// o = sum_p o_p e^{m_p - M} / L with the sink in L; partial mode writes
// (M, L, sum_p o_p e^{m_p-M}) without the sink.  One warp per (query row,
// head, slice of DPL * 32 output dims): the split statistics are reduced
// across lanes (any number of splits), then lane l combines DPL dims of
// every split, four splits' loads in flight at a time.  DPL = 16 covers the
// 512 dims with one warp (many query rows); DPL = 4 spreads a row over 4x
// more warps for the few-row case (a single long context), where the
// combine would otherwise run on M * 8 CTAs.
constexpr int kCombineWarps = 8;
template <int DPL>
__global__ void __launch_bounds__(32 * kCombineWarps) lse_combine_kernel(
    const float* __restrict__ part_ml, const float* __restrict__ part_o, const float* __restrict__ sink, int P, int M,
    int H, int D, int64_t ml_ps, int64_t o_ps, int final_mode, __nv_bfloat16* __restrict__ out,
    float* __restrict__ lse, float* __restrict__ out_ml, float* __restrict__ out_o) {
  const int m = blockIdx.x, lane = threadIdx.x & 31;
  const int h = blockIdx.y * kCombineWarps + (threadIdx.x >> 5);
  pdl_wait();
  pdl_launch_dependents();
  if (h >= H) return;
  auto ml = [&](int p, int j) { return part_ml[int64_t(p) * ml_ps + (int64_t(m) * H + h) * 2 + j]; };
  float Mx = final_mode ? sink[h] : -INFINITY;
  for (int p0 = 0; p0 < P; p0 += 32) {
    const float mp = p0 + lane < P ? ml(p0 + lane, 0) : -INFINITY;
    Mx = fmaxf(Mx, warp_max(mp));
  }
  float lsum = 0.f;
  for (int p0 = 0; p0 < P; p0 += 32) {
    if (p0 + lane < P) {
      const float mp = ml(p0 + lane, 0);
      if (mp != -INFINITY) lsum += ml(p0 + lane, 1) * expf(mp - Mx);
    }
  }
  float L = warp_sum(lsum);
  if (final_mode && Mx != -INFINITY) L += expf(sink[h] - Mx);
  const int d0 = blockIdx.z * (32 * DPL) + DPL * lane;
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
#pragma unroll 4
  for (int p = 0; p < P; ++p) {
    const float mp = ml(p, 0);
    const float w = (mp == -INFINITY) ? 0.f : expf(mp - Mx);
    const float4* src = reinterpret_cast<const float4*>(part_o + int64_t(p) * o_ps + (int64_t(m) * H + h) * D + d0);
    float4 v[DPL / 4];
#pragma unroll
    for (int i = 0; i < DPL / 4; ++i) v[i] = __ldg(src + i);
#pragma unroll
    for (int i = 0; i < DPL / 4; ++i) {
      acc[4 * i + 0] = fmaf(w, v[i].x, acc[4 * i + 0]);
      acc[4 * i + 1] = fmaf(w, v[i].y, acc[4 * i + 1]);
      acc[4 * i + 2] = fmaf(w, v[i].z, acc[4 * i + 2]);
      acc[4 * i + 3] = fmaf(w, v[i].w, acc[4 * i + 3]);
    }
  }
  if (final_mode) {
    const float inv = 1.f / L;
    uint2* op = reinterpret_cast<uint2*>(out + (int64_t(m) * H + h) * D + d0);
#pragma unroll
    for (int i = 0; i < DPL / 4; ++i)
      op[i] = make_uint2(pack_bf16x2(acc[4 * i] * inv, acc[4 * i + 1] * inv),
                         pack_bf16x2(acc[4 * i + 2] * inv, acc[4 * i + 3] * inv));
  } else {
    float4* op = reinterpret_cast<float4*>(out_o + (int64_t(m) * H + h) * D + d0);
#pragma unroll
    for (int i = 0; i < DPL / 4; ++i) op[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
  }
  if (lane == 0 && blockIdx.z == 0) {
    if (final_mode) {
      if (lse) lse[int64_t(m) * H + h] = Mx + logf(L);
    } else {
      out_ml[(int64_t(m) * H + h) * 2] = Mx;
      out_ml[(int64_t(m) * H + h) * 2 + 1] = L;
    }
  }
}

// Launch of the combine: DPL = 4 (4 CTAs per 8 heads) when the rows alone
// would leave most SMs idle.
static void launch_lse_combine(const float* part_ml, const float* part_o, const float* sink, int P, int M, int H,
                               int D, int final_mode, __nv_bfloat16* out, float* lse, float* out_ml, float* out_o,
                               cudaStream_t st, int64_t ml_ps = -1, int64_t o_ps = -1) {
  const int hb = (H + kCombineWarps - 1) / kCombineWarps;
  if (ml_ps < 0) ml_ps = int64_t(M) * H * 2;
  if (o_ps < 0) o_ps = int64_t(M) * H * D;
  if (int64_t(M) * hb < 2 * num_sms()) {
    launch_pdl(lse_combine_kernel<4>, dim3(M, hb, D / 128), dim3(32 * kCombineWarps), 0, st, part_ml, part_o, sink, P,
               M, H, D, ml_ps, o_ps, final_mode, out, lse, out_ml, out_o);
  } else {
    launch_pdl(lse_combine_kernel<16>, dim3(M, hb, D / 512), dim3(32 * kCombineWarps), 0, st, part_ml, part_o, sink,
               P, M, H, D, ml_ps, o_ps, final_mode, out, lse, out_ml, out_o);
  }
}

struct SplitPlan {
  int nsplit;
  int tiles_per_split;
};

static long long* g_trace = nullptr;

static bool use_mma_v0() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("DSV4_SPARSE_ATTN_MMA");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

static int split_tile() { return use_mma_v0() ? kSaTile : satc::TK; }
static int idx_cap() { return satc::kIdxCap; }

static SplitPlan plan_splits(int M, int K) {
  const int tile = split_tile();
  const int ntiles = std::max(1, (K + tile - 1) / tile);
  int want = std::max(1, num_sms() / std::max(1, M));
  want = std::min(want, ntiles);
  int tps = (ntiles + want - 1) / want;
  // at least two tiles per split: a CTA's fixed cost (Q load, TMEM set-up,
  // 128 KB partial out, its share of the combine) outweighs a second tile
  // (few-row shapes: 1 row x 34 tiles 18.2 -> 15.8 us, 4 rows 21.5 -> 18.0 us)
  tps = std::max(tps, std::min(2, ntiles));
  if (!use_mma_v0()) tps = std::min(tps, idx_cap() / tile);  // the tc kernel stages <= kIdxCap indices
  return {(ntiles + tps - 1) / tps, tps};
}

static size_t ws_bytes_for(const SplitPlan& p, int M) {
  return p.nsplit <= 1 ? 0 : size_t(p.nsplit) * M * kSaH * (2 + kSaD) * sizeof(float);
}

static void ensure_attr() {
  static int done_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (done_dev != dev) {
    cudaFuncSetAttribute(sparse_attn_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSaSmem);
    cudaFuncSetAttribute(satc::sparse_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         satc::kSmemBytes);

    done_dev = dev;
  }
}

static int check_common(const void* q, const void* kv, int64_t kv_bstride, int64_t kv_rows, const int32_t* idx,
                        int64_t ld_idx, int B, int S, int H, int D, int K) {
  DSA_CHECK_ARG(q && kv && idx, "sparse_attn: null q/kv/idx");
  DSA_CHECK_ARG(H == kSaH && D == kSaD, "sparse_attn: built for H=64, D=512 (got H=%d D=%d)", H, D);
  DSA_CHECK_ARG(B >= 0 && S >= 1 && K >= 0 && kv_rows > 0, "sparse_attn: bad B/S/K/kv_rows");
  DSA_CHECK_ARG(kv_bstride >= kv_rows * D && kv_bstride % 8 == 0, "sparse_attn: bad kv batch stride");
  DSA_CHECK_ARG(ld_idx >= K, "sparse_attn: ld_idx < K");
  DSA_CHECK_ARG(aligned(q, 16) && aligned(kv, 16), "sparse_attn: q/kv must be 16-byte aligned");
  return DSA_OK;
}

}  // namespace dsa

using namespace dsa;

extern "C" size_t dsa_sparse_attn_workspace_size(int B, int S, int H, int D, int K) {
  (void)H;
  (void)D;
  const int M = B * S;
  return ws_bytes_for(plan_splits(M, K), M);
}

static int sparse_attn_run(const void* q, const void* kv, int64_t kv_bstride, int64_t kv_rows, const int32_t* idx,
                           int64_t ld_idx, const float* sink, void* out, float* lse, float* part_ml_out,
                           float* part_o_out, int B, int S, int H, int D, int K, float scale, void* ws,
                           size_t ws_bytes, int32_t* status, cudaStream_t st, bool final_mode) {
  int rc = check_common(q, kv, kv_bstride, kv_rows, idx, ld_idx, B, S, H, D, K);
  if (rc) return rc;
  const int M = B * S;
  if (M == 0) return DSA_OK;
  ensure_attr();
  const SplitPlan p = plan_splits(M, K);
  // the split-K combine writes 16-byte vectors
  DSA_CHECK_ARG(p.nsplit <= 1 || (final_mode ? aligned(out, 16) : aligned(part_o_out, 16)),
                "sparse_attn: out / part_o must be 16-byte aligned");
  SaArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.kv = static_cast<const __nv_bfloat16*>(kv);
  a.kv_bstride = kv_bstride;
  a.kv_rows = kv_rows;
  a.idx = idx;
  a.ld_idx = ld_idx;
  a.sink = sink;
  a.status = status;
  a.S = S;
  a.M = M;
  a.K = K;
  a.tiles_per_split = p.tiles_per_split;
  a.scale_log2 = scale * kLog2e;
  float* ws_ml = nullptr;
  float* ws_o = nullptr;
  if (p.nsplit > 1) {
    const size_t need = ws_bytes_for(p, M);
    if (ws == nullptr || ws_bytes < need) {
      set_error("sparse_attn: needs %zu bytes of workspace (got %zu)", need, ws_bytes);
      return DSA_ERR_WORKSPACE;
    }
    ws_ml = static_cast<float*>(ws);
    ws_o = ws_ml + size_t(p.nsplit) * M * kSaH * 2;
    a.final_mode = 0;
    a.part_ml = ws_ml;
    a.part_o = ws_o;
  } else if (final_mode) {
    a.final_mode = 1;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.lse = lse;
  } else {
    a.final_mode = 0;
    a.part_ml = part_ml_out;
    a.part_o = part_o_out;
  }
  if (use_mma_v0()) {
    sparse_attn_mma_kernel<<<dim3(p.nsplit, M), kSaThreads, kSaSmem, st>>>(a);
  } else {
    satc::Args t{};
    t.q = a.q;
    t.kv = a.kv;
    t.kv_bstride = a.kv_bstride;
    t.kv_rows = a.kv_rows;
    t.idx = a.idx;
    t.ld_idx = a.ld_idx;
    t.sink = a.sink;
    t.out = a.out;
    t.lse = a.lse;
    t.part_ml = a.part_ml;
    t.part_o = a.part_o;
    t.status = a.status;
    t.S = a.S;
    t.M = a.M;
    t.K = a.K;
    t.tiles_per_split = a.tiles_per_split;
    t.scale_log2 = a.scale_log2;
    t.final_mode = a.final_mode;
    t.trace = g_trace;
    CUtensorMap tm_q;
    DSA_CHECK_ARG(kv_bstride % kSaD == 0, "sparse_attn: kv batch stride must be a multiple of D");
    const int64_t row_stride = kv_bstride / kSaD;
    if (!tma::make_2d_bf16(&tm_q, q, kSaD, uint64_t(M) * kSaH, kSaD * 2, 64, 64)) {
      set_error("sparse_attn: cuTensorMapEncodeTiled failed");
      return DSA_ERR_CUDA;
    }
    launch_pdl(satc::sparse_attn_tc_kernel, dim3(p.nsplit, M), dim3(satc::THREADS), satc::kSmemBytes, st, t, tm_q,
               row_stride);
  }
  DSA_CHECK_LAUNCH("sparse_attn");
  if (p.nsplit > 1) {
    launch_lse_combine(ws_ml, ws_o, sink, p.nsplit, M, kSaH, kSaD, final_mode ? 1 : 0,
                       static_cast<__nv_bfloat16*>(out), lse, part_ml_out, part_o_out, st);
    DSA_CHECK_LAUNCH("sparse_attn(combine)");
  }
  return DSA_OK;
}

extern "C" int dsa_sparse_attn(const void* q, const void* kv, int64_t kv_bstride, int64_t kv_rows,
                               const int32_t* idx, int64_t ld_idx, const float* sink, void* out, float* lse, int B,
                               int S, int H, int D, int K, float scale, void* workspace, size_t workspace_bytes,
                               int32_t* status, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(sink && out, "sparse_attn: null sink/out");
  return sparse_attn_run(q, kv, kv_bstride, kv_rows, idx, ld_idx, sink, out, lse, nullptr, nullptr, B, S, H, D, K,
                         scale, workspace, workspace_bytes, status, reinterpret_cast<cudaStream_t>(stream), true);
}

extern "C" int dsa_sparse_attn_partial(const void* q, const void* kv, int64_t kv_bstride, int64_t kv_rows,
                                       const int32_t* idx, int64_t ld_idx, float* part_ml, float* part_o, int B,
                                       int S, int H, int D, int K, float scale, void* workspace,
                                       size_t workspace_bytes, int32_t* status, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(part_ml && part_o, "sparse_attn_partial: null outputs");
  return sparse_attn_run(q, kv, kv_bstride, kv_rows, idx, ld_idx, nullptr, nullptr, nullptr, part_ml, part_o, B, S,
                         H, D, K, scale, workspace, workspace_bytes, status, reinterpret_cast<cudaStream_t>(stream),
                         false);
}

extern "C" int dsa_lse_combine(const float* part_ml, const float* part_o, const float* sink, void* out, int P, int M,
                               int H, int D, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(part_ml && part_o && sink && out, "lse_combine: null pointer");
  DSA_CHECK_ARG(P > 0 && M >= 0 && H > 0, "lse_combine: bad P/M/H");
  DSA_CHECK_ARG(D == kSaD, "lse_combine: built for D=%d (got %d)", kSaD, D);
  DSA_CHECK_ARG(aligned(part_o, 16) && aligned(out, 16), "lse_combine: part_o / out must be 16-byte aligned");
  if (M == 0) return DSA_OK;
  launch_lse_combine(part_ml, part_o, sink, P, M, H, D, 1, static_cast<__nv_bfloat16*>(out), nullptr, nullptr,
                     nullptr, reinterpret_cast<cudaStream_t>(stream));
  DSA_CHECK_LAUNCH("lse_combine");
  return DSA_OK;
}

extern "C" int dsa_lse_combine_strided(const float* part_ml, int64_t ml_pstride, const float* part_o,
                                       int64_t o_pstride, const float* sink, void* out, int P, int M, int H, int D,
                                       dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(part_ml && part_o && sink && out, "lse_combine_strided: null pointer");
  DSA_CHECK_ARG(P > 0 && M >= 0 && H > 0, "lse_combine_strided: bad P/M/H");
  DSA_CHECK_ARG(D == kSaD, "lse_combine_strided: built for D=%d (got %d)", kSaD, D);
  DSA_CHECK_ARG(ml_pstride >= int64_t(M) * H * 2 && o_pstride >= int64_t(M) * H * D && o_pstride % 4 == 0,
                "lse_combine_strided: partial strides must cover M*H*2 / M*H*D floats (o stride a multiple of 4)");
  DSA_CHECK_ARG(aligned(part_o, 16) && aligned(out, 16), "lse_combine_strided: part_o / out must be 16-byte aligned");
  if (M == 0) return DSA_OK;
  launch_lse_combine(part_ml, part_o, sink, P, M, H, D, 1, static_cast<__nv_bfloat16*>(out), nullptr, nullptr,
                     nullptr, reinterpret_cast<cudaStream_t>(stream), ml_pstride, o_pstride);
  DSA_CHECK_LAUNCH("lse_combine_strided");
  return DSA_OK;
}

extern "C" int dsa_set_trace(void* dev_buffer, size_t bytes) {
  clear_error();
  const size_t need = size_t(satc::kTrMisc + 1) * satc::kTrTiles * sizeof(long long);
  DSA_CHECK_ARG(dev_buffer == nullptr || bytes >= need, "set_trace: buffer needs %zu bytes", need);
  g_trace = static_cast<long long*>(dev_buffer);
  return DSA_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of dsa_sparse_attn.
//
// Some callers cannot allocate device memory at the point where they call the
// attention: a host runtime that owns a fixed device arena and forbids other
// allocations, a plugin called from inside another framework's memory
// manager, or code running where cudaMalloc is unavailable or too slow.  For
// them the split-K partials (the only scratch dsa_sparse_attn needs) live in
// a file-scope device array that the library reserves once at load time.
// Every GPU that loads the library holds these 8 MiB until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
static void* g_noalloc_ptr[kMaxDevices] = {nullptr};
static std::mutex g_noalloc_mu;

// Device address of the scratch array for the current device.  The array's
// name is only a host-side handle; its device address comes from
// cudaGetSymbolAddress, resolved once per device with that device current.
static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("sparse_attn_noalloc: no usable current device");
    return DSA_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("sparse_attn_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return DSA_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return DSA_OK;
}

}  // namespace

extern "C" int dsa_sparse_attn_noalloc(const void* q, const void* kv, int64_t kv_bstride, int64_t kv_rows,
                                       const int32_t* idx, int64_t ld_idx, const float* sink, void* out, float* lse,
                                       int B, int S, int H, int D, int K, float scale, int32_t* status,
                                       dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(sink && out, "sparse_attn_noalloc: null sink/out");
  DSA_CHECK_ARG(B >= 0 && S >= 1 && K >= 0, "sparse_attn_noalloc: bad B/S/K");
  const size_t need = dsa_sparse_attn_workspace_size(B, S, H, D, K);
  if (need > kNoAllocScratchBytes) {
    set_error("sparse_attn_noalloc: this shape needs %zu bytes of scratch, above the built-in maximum of %zu "
              "(use dsa_sparse_attn with a caller-owned workspace)",
              need, kNoAllocScratchBytes);
    return DSA_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = noalloc_scratch(&scratch);
    if (rc != DSA_OK) return rc;
  }
  // Every split-K partial is written before it is read, so the scratch needs
  // no clearing between calls.
  return sparse_attn_run(q, kv, kv_bstride, kv_rows, idx, ld_idx, sink, out, lse, nullptr, nullptr, B, S, H, D, K,
                         scale, scratch, need > 0 ? kNoAllocScratchBytes : 0, status,
                         reinterpret_cast<cudaStream_t>(stream), true);
}
