// attn.sparse: index gather + sink-softmax attention over the selected rows.
//
// Reference: DeviceSparseAttn.forward_device (inference.py:4459-4501) with
// the index->mask conversion _idxs_int_tile_to_idxs_and_mask (4444-4457)
// folded in: a -1 index contributes nothing, the per-head sink logit joins
// the softmax denominator once.  K = V = the 512-d latent row (MQA).
//
// Flash-decoding over key splits: one CTA per (query row, key split) runs
// the tcgen05 kernel of sparse_attn_tc.cuh; a row with one split is
// finished by that CTA (sink included), the splits of a row with several
// are merged, with the sink counted once, by lse_combine_kernel (which also
// merges the partials that the sequence split gathers from other GPUs).
#include "common.cuh"
#include "sparse_attn_tc.cuh"
#include <stdlib.h>
#include <mutex>

namespace dsa {

constexpr int kSaH = 64;
constexpr int kSaD = 512;
constexpr float kLog2e = 1.4426950408889634f;

// Merge of the split-K partials of each query row.  Partials come as fp32
// (m, l, unnormalised o) - the sequence split's exchanged partials - or, for
// the library's own split-K workspace (kNormBF16), as fp32 (m, l) with the
// bf16 o / l, half the bytes to write and read back; the weight of a
// partial is then l e^{m - M} instead of e^{m - M}.  Final mode writes
// o = sum_p o_p e^{m_p - M} / L with the sink in L; partial mode writes
// (M, L, sum_p o_p e^{m_p-M}) without the sink.  One warp per (query row,
// head, slice of DPL * 32 output dims): the split statistics are reduced
// across lanes (any number of splits), then lane l combines DPL dims of
// every split, four splits' loads in flight at a time.  DPL = 16 covers the
// 512 dims with one warp (many query rows); DPL = 4 spreads a row over 4x
// more warps for the few-row case (a single long context), where the
// combine would otherwise run on M * 8 CTAs.
constexpr int kCombineWarps = 8;
template <int DPL, bool kNormBF16>
__global__ void __launch_bounds__(32 * kCombineWarps) lse_combine_kernel(
    const float* __restrict__ part_ml, const void* __restrict__ part_o, const float* __restrict__ sink, int P, int M,
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
    float w = (mp == -INFINITY) ? 0.f : expf(mp - Mx);
    const int64_t off = int64_t(p) * o_ps + (int64_t(m) * H + h) * D + d0;
    if constexpr (kNormBF16) {
      w *= ml(p, 1);
      // DPL bf16 values = DPL / 4 8-byte words
      const uint2* src = reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(part_o) + off);
      uint2 v[DPL / 4];
#pragma unroll
      for (int i = 0; i < DPL / 4; ++i) v[i] = __ldg(src + i);
#pragma unroll
      for (int i = 0; i < DPL / 4; ++i) {
        acc[4 * i + 0] = fmaf(w, __uint_as_float(v[i].x << 16), acc[4 * i + 0]);
        acc[4 * i + 1] = fmaf(w, __uint_as_float(v[i].x & 0xffff0000u), acc[4 * i + 1]);
        acc[4 * i + 2] = fmaf(w, __uint_as_float(v[i].y << 16), acc[4 * i + 2]);
        acc[4 * i + 3] = fmaf(w, __uint_as_float(v[i].y & 0xffff0000u), acc[4 * i + 3]);
      }
    } else {
      const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(part_o) + off);
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
static void launch_lse_combine(const float* part_ml, const void* part_o, bool norm_bf16, const float* sink, int P,
                               int M, int H, int D, int final_mode, __nv_bfloat16* out, float* lse, float* out_ml,
                               float* out_o, cudaStream_t st, int64_t ml_ps = -1, int64_t o_ps = -1) {
  const int hb = (H + kCombineWarps - 1) / kCombineWarps;
  if (ml_ps < 0) ml_ps = int64_t(M) * H * 2;
  if (o_ps < 0) o_ps = int64_t(M) * H * D;
  const bool few = int64_t(M) * hb < 2 * num_sms();
  const dim3 grid(M, hb, few ? D / 128 : D / 512);
  auto k = few ? (norm_bf16 ? lse_combine_kernel<4, true> : lse_combine_kernel<4, false>)
               : (norm_bf16 ? lse_combine_kernel<16, true> : lse_combine_kernel<16, false>);
  launch_pdl(k, grid, dim3(32 * kCombineWarps), 0, st, part_ml, part_o, sink, P, M, H, D, ml_ps, o_ps, final_mode,
             out, lse, out_ml, out_o);
}

struct SplitPlan {
  int nsplit;
  int tiles_per_split;
};

static long long* g_trace = nullptr;

static int split_tile() { return satc::TK; }
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
  tps = std::min(tps, idx_cap() / tile);  // the kernel stages <= kIdxCap indices
  return {(ntiles + tps - 1) / tps, tps};
}

static size_t ws_bytes_for(const SplitPlan& p, int M) {
  // per (split, row, head): fp32 (m, l) and the bf16 o / l
  return p.nsplit <= 1 ? 0 : size_t(p.nsplit) * M * kSaH * (2 * sizeof(float) + kSaD * sizeof(__nv_bfloat16));
}

static void ensure_attr() {
  static int done_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (done_dev != dev) {
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
  DSA_CHECK_ARG(int64_t(B) * S <= INT32_MAX / kSaH, "sparse_attn: B*S = %lld query rows is too many",
                (long long)B * S);
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
  // shapes the attention rejects (B*S beyond its row limit) need no workspace
  if (B < 0 || S < 1 || int64_t(B) * S > INT32_MAX / kSaH) return 0;
  const int M = B * S;
  return ws_bytes_for(plan_splits(M, K), M);
}

static int sparse_attn_run(const void* q, const void* kv, int64_t kv_bstride, int64_t kv_rows, const int32_t* idx,
                           int64_t ld_idx, const float* sink, void* out, float* lse, float* part_ml_out,
                           float* part_o_out, int B, int S, int H, int D, int K, float scale, void* ws,
                           size_t ws_bytes, int32_t* status, cudaStream_t st, bool final_mode, int lead_cols = 0,
                           unsigned flags = 0) {
  int rc = check_common(q, kv, kv_bstride, kv_rows, idx, ld_idx, B, S, H, D, K);
  if (rc) return rc;
  const int M = B * S;
  if (M == 0) return DSA_OK;
  ensure_attr();
  const SplitPlan p = plan_splits(M, K);
  // the split-K combine writes 16-byte vectors
  DSA_CHECK_ARG(p.nsplit <= 1 || (final_mode ? aligned(out, 16) : aligned(part_o_out, 16)),
                "sparse_attn: out / part_o must be 16-byte aligned");
  satc::Args t{};
  t.q = static_cast<const __nv_bfloat16*>(q);
  t.kv = static_cast<const __nv_bfloat16*>(kv);
  t.kv_bstride = kv_bstride;
  t.kv_rows = kv_rows;
  t.idx = idx;
  t.ld_idx = ld_idx;
  t.sink = sink;
  t.status = status;
  t.S = S;
  t.M = M;
  t.K = K;
  t.tiles_per_split = p.tiles_per_split;
  // lead tiles: one per split, first, when the caller names leading index
  // columns that are ready early (requested before the dependency wait)
  if ((flags & DSA_LEAD_READY) && lead_cols > 0 && lead_cols % satc::TK == 0 && lead_cols < K &&
      p.nsplit >= lead_cols / satc::TK) {
    const int lead_tiles = lead_cols / satc::TK;
    const int rest_tiles = (K - lead_cols + satc::TK - 1) / satc::TK;
    const int rest_tps = (rest_tiles + p.nsplit - 1) / p.nsplit;
    if (1 + rest_tps <= satc::kMaxTilesPerSplit) {
      t.lead_tiles = lead_tiles;
      t.rest_tps = rest_tps;
      t.early = 1;
    }
  }
  t.scale_log2 = scale * kLog2e;
  t.wait_limit = wait_limit_cycles();
  t.trace = g_trace;
  float* ws_ml = nullptr;
  __nv_bfloat16* ws_o = nullptr;
  // two key splits with a final output: the splits of a row run as one
  // cluster and finish the row between them, exchanging half of each
  // accumulator through the workspace (no combine launch)
  const bool pair = p.nsplit == 2 && final_mode;
  static_assert(2 * satc::kPairXFloats * sizeof(float) <= kSaH * (2 * sizeof(float) + kSaD * 2) * 2,
                "the pair exchange fits the two-split workspace");
  if (p.nsplit > 1) {
    const size_t need = ws_bytes_for(p, M);
    if (ws == nullptr || ws_bytes < need) {
      set_error("sparse_attn: needs %zu bytes of workspace (got %zu)", need, ws_bytes);
      return DSA_ERR_WORKSPACE;
    }
  }
  if (pair) {
    DSA_CHECK_ARG(aligned(ws, 16), "sparse_attn: the workspace must be 16-byte aligned");
    t.final_mode = 0;
    t.pair_combine = 1;
    t.pair_x = static_cast<float*>(ws);
    t.out = static_cast<__nv_bfloat16*>(out);
    t.lse = lse;
  } else if (p.nsplit > 1) {
    ws_ml = static_cast<float*>(ws);
    ws_o = reinterpret_cast<__nv_bfloat16*>(ws_ml + size_t(p.nsplit) * M * kSaH * 2);
    t.final_mode = 0;
    t.part_ml = ws_ml;
    t.part_ob = ws_o;
  } else if (final_mode) {
    t.final_mode = 1;
    t.out = static_cast<__nv_bfloat16*>(out);
    t.lse = lse;
  } else {
    t.final_mode = 0;
    t.part_ml = part_ml_out;
    t.part_o = part_o_out;
  }
  DSA_CHECK_ARG(kv_bstride % kSaD == 0, "sparse_attn: kv batch stride must be a multiple of D");
  const int64_t row_stride = kv_bstride / kSaD;
  CUtensorMap tm_q;
  if (!tma::make_2d_bf16(&tm_q, q, kSaD, uint64_t(M) * kSaH, kSaD * 2, 64, 64)) {
    set_error("sparse_attn: cuTensorMapEncodeTiled failed");
    return DSA_ERR_CUDA;
  }
  if (pair) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, M);
    cfg.blockDim = dim3(satc::THREADS);
    cfg.dynamicSmemBytes = satc::kSmemBytes;
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
    cudaLaunchKernelEx(&cfg, satc::sparse_attn_tc_kernel, t, tm_q, row_stride);
    DSA_CHECK_LAUNCH("sparse_attn");
    return DSA_OK;
  }
  launch_pdl(satc::sparse_attn_tc_kernel, dim3(p.nsplit, M), dim3(satc::THREADS), satc::kSmemBytes, st, t, tm_q,
             row_stride);
  DSA_CHECK_LAUNCH("sparse_attn");
  if (p.nsplit > 1) {
    launch_lse_combine(ws_ml, ws_o, true, sink, p.nsplit, M, kSaH, kSaD, final_mode ? 1 : 0,
                       static_cast<__nv_bfloat16*>(out), lse, part_ml_out, part_o_out, st);
    DSA_CHECK_LAUNCH("sparse_attn(combine)");
  }
  return DSA_OK;
}

extern "C" int dsa_sparse_attn_ex(const void* q, const void* kv, int64_t kv_bstride, int64_t kv_rows,
                                  const int32_t* idx, int64_t ld_idx, const float* sink, void* out, float* lse, int B,
                                  int S, int H, int D, int K, float scale, void* workspace, size_t workspace_bytes,
                                  int lead_cols, unsigned flags, int32_t* status, dsa_stream_t stream) {
  clear_error();
  DSA_CHECK_ARG(sink && out, "sparse_attn: null sink/out");
  DSA_CHECK_ARG(lead_cols >= 0 && lead_cols <= K, "sparse_attn: lead_cols %d outside [0, K]", lead_cols);
  DSA_CHECK_ARG((flags & ~unsigned(DSA_LEAD_READY)) == 0, "sparse_attn: unknown flags 0x%x", flags);
  return sparse_attn_run(q, kv, kv_bstride, kv_rows, idx, ld_idx, sink, out, lse, nullptr, nullptr, B, S, H, D, K,
                         scale, workspace, workspace_bytes, status, reinterpret_cast<cudaStream_t>(stream), true,
                         lead_cols, flags);
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
  launch_lse_combine(part_ml, part_o, false, sink, P, M, H, D, 1, static_cast<__nv_bfloat16*>(out), nullptr, nullptr,
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
  launch_lse_combine(part_ml, part_o, false, sink, P, M, H, D, 1, static_cast<__nv_bfloat16*>(out), nullptr, nullptr,
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
  DSA_CHECK_ARG(int64_t(B) * S <= INT32_MAX / kSaH, "sparse_attn_noalloc: B*S = %lld query rows is too many",
                (long long)B * S);
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
