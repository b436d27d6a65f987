// The decode layer's small per-sequence stages as one launch: the indexer
// compressor's step followed by the newest compressed row's indexer score
// (CTA row 0 of the grid), and the window-ring KV write, the window indices
// and the attention compressor's step (CTA row 1).  The same device code as
// dsa_compressor_step, dsa_indexer_score_newest, dsa_kv_window_write and
// dsa_window_indices, one CTA per (sequence, group).
//
// Why one launch: in a decode step these stages feed the top-k and the
// attention but depend on nothing the indexer score computes, so they run
// beside it.  Issued on their own streams, every join placed before the
// top-k or the attention turned that kernel's programmatic dependent launch
// into a full dependency (~4 us of idle SMs at each hand-over, measured),
// and the small kernels, dispatched at the layer's start, held SMs the
// persistent score kernel then started late on.  As one kernel placed after
// the score on the same stream, it is dispatched after the score's CTAs
// (sharing their SMs: ~4.5 KB of shared memory, 256 threads), lets its
// successor launch at once, and waits for the score only before it
// completes: its completion then implies the score's, so the top-k and the
// attention keep single programmatic dependencies.
#include "common.cuh"
#include "act_quant_dev.cuh"
#include "compressor_dev.cuh"
#include "indexer_row.cuh"
#include "window_rows.cuh"

namespace dsa {

struct PrologueArgs {
  CmpStep icmp, cmp;            // indexer compressor, attention compressor
  const __nv_bfloat16* iq;      // newest score: q [B, 64, 128], w [B, 64], score [B, ld_score]
  const float* iw;
  const int32_t* t_active;
  float* score;
  int64_t ld_score;
  int T;
  const __nv_bfloat16* kv;      // window write: kv [B, D] into cmp.cache's ring slot pos % win
  float* kv_scales;
  int D, rope_dim, win;
  int32_t* idx;                 // window indices: idx[b, 0:win]
  int64_t ld_idx;
  int beside;                   // wait for the previous kernel only before completing
};

__global__ void __launch_bounds__(kCmpThreads) layer_prologue_kernel(const __grid_constant__ PrologueArgs a) {
  __shared__ float s_row[kCmpMaxD];
  __shared__ float s_red[32];
  __shared__ float s_dot[kRowHeads];
  if (!a.beside) pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  if (blockIdx.y == 0) {
    compressor_step_row(a.icmp, b, s_row, s_red);
    __syncthreads();  // the compressed row it may have written is read below
    score_newest_row(a.iq, a.icmp.cache, a.icmp.cache_bstride, a.iw, a.t_active, a.score, a.ld_score, a.T, b,
                     s_dot);
  } else {
    kv_window_write_row(a.kv, a.cmp.cache, a.kv_scales, a.cmp.pos, a.D, a.rope_dim, a.cmp.cache_bstride, a.win,
                        448.f, float(1.0 / 448.0), 1e-4f, b);
    window_indices_row(a.cmp.pos, a.idx, a.ld_idx, a.win, b);
    compressor_step_row(a.cmp, b, s_row, s_red);
  }
  // this kernel completes only after its predecessor has: a successor that
  // waits for it also sees everything the predecessor wrote
  if (a.beside) pdl_wait();
}

static int check_cmp(const dsa_compressor_args* c, const char* what) {
  DSA_CHECK_ARG(c && c->kv_row && c->score_row && c->ape && c->kv_state && c->score_state && c->gamma && c->kv_cache,
                "layer_prologue: %s: null pointer", what);
  DSA_CHECK_ARG(c->d > 0 && c->d <= kCmpMaxD && c->d % 2 == 0, "layer_prologue: %s: d=%d must be even and <= %d", what,
                c->d, kCmpMaxD);
  DSA_CHECK_ARG(c->rope_dim >= 0 && c->rope_dim <= c->d && c->rope_dim % 2 == 0, "layer_prologue: %s: bad rope_dim",
                what);
  DSA_CHECK_ARG(c->ratio > 0, "layer_prologue: %s: ratio must be positive", what);
  DSA_CHECK_ARG(c->ld_row >= (c->overlap ? 2 : 1) * c->d, "layer_prologue: %s: ld_row too small", what);
  DSA_CHECK_ARG(c->cache_rows > 0 && c->cache_bstride >= c->cache_rows * c->d, "layer_prologue: %s: bad cache shape",
                what);
  DSA_CHECK_ARG(!c->rotate || (c->d & (c->d - 1)) == 0, "layer_prologue: %s: Hadamard needs power-of-two d", what);
  return DSA_OK;
}

static CmpStep to_step(const dsa_compressor_args* c, const float* cos_tab, const float* sin_tab, int n_pos,
                       const int32_t* pos, float eps) {
  return CmpStep{static_cast<const __nv_bfloat16*>(c->kv_row), static_cast<const __nv_bfloat16*>(c->score_row),
                 c->ld_row, c->ape, c->kv_state, c->score_state, c->gamma, cos_tab, sin_tab, n_pos,
                 static_cast<__nv_bfloat16*>(c->kv_cache), c->cache_bstride, c->cache_rows, c->slot_offset, pos,
                 nullptr, c->d, c->rope_dim, c->ratio, c->overlap ? 1 : 0, c->rotate ? 1 : 0, 1,
                 float(1.0 / sqrt(double(c->d))), eps};
}

}  // namespace dsa

using namespace dsa;

extern "C" int dsa_layer_prologue(const dsa_compressor_args* icmp, const dsa_compressor_args* cmp,
                                  const float* cos_tab, const float* sin_tab, int n_pos, float eps,
                                  const int32_t* pos, const int32_t* t_active, const void* iq, const float* iw,
                                  float* score, int64_t ld_score, int T, const void* kv, float* kv_scales, int D,
                                  int rope_dim, int win, int32_t* idx, int64_t ld_idx, int B, unsigned flags,
                                  dsa_stream_t stream) {
  clear_error();
  int rc = check_cmp(icmp, "indexer compressor");
  if (rc) return rc;
  rc = check_cmp(cmp, "attention compressor");
  if (rc) return rc;
  DSA_CHECK_ARG(cos_tab && sin_tab && n_pos > 0 && pos && t_active && iq && iw && score && kv && idx,
                "layer_prologue: null pointer");
  DSA_CHECK_ARG((flags & ~unsigned(DSA_BESIDE_PREVIOUS)) == 0, "layer_prologue: unknown flags 0x%x", flags);
  DSA_CHECK_ARG(B >= 0 && T > 0 && ld_score >= T, "layer_prologue: bad B/T/ld_score");
  // the newest score reads the indexer compressor's cache: 64 heads x 128 dims
  DSA_CHECK_ARG(icmp->d == kRowDim && icmp->cache_rows >= T, "layer_prologue: the indexer cache must be [B, >=T, 128]");
  DSA_CHECK_ARG(aligned(iq, 8) && aligned(icmp->kv_cache, 8) && icmp->cache_bstride % 4 == 0,
                "layer_prologue: q, the indexer cache and its row stride must be 8-byte aligned");
  DSA_CHECK_ARG(D == cmp->d && rope_dim >= 0 && rope_dim < D && (D - rope_dim) % 64 == 0,
                "layer_prologue: the window row must be the attention compressor's d with 64-multiple nope dims");
  DSA_CHECK_ARG(win > 0 && cmp->cache_bstride >= int64_t(win) * D && ld_idx >= win,
                "layer_prologue: bad window / cache stride / ld_idx");
  DSA_CHECK_ARG(aligned(kv, 4) && aligned(cmp->kv_cache, 4) && D % 2 == 0 && cmp->cache_bstride % 2 == 0,
                "layer_prologue: kv and the attention cache must be 4-byte aligned");
  if (B == 0) return DSA_OK;
  PrologueArgs a{};
  a.icmp = to_step(icmp, cos_tab, sin_tab, n_pos, pos, eps);
  a.cmp = to_step(cmp, cos_tab, sin_tab, n_pos, pos, eps);
  a.iq = static_cast<const __nv_bfloat16*>(iq);
  a.iw = iw;
  a.t_active = t_active;
  a.score = score;
  a.ld_score = ld_score;
  a.T = T;
  a.kv = static_cast<const __nv_bfloat16*>(kv);
  a.kv_scales = kv_scales;
  a.D = D;
  a.rope_dim = rope_dim;
  a.win = win;
  a.idx = idx;
  a.ld_idx = ld_idx;
  a.beside = (flags & DSA_BESIDE_PREVIOUS) ? 1 : 0;
  launch_pdl(layer_prologue_kernel, dim3(B, 2), dim3(kCmpThreads), 0, reinterpret_cast<cudaStream_t>(stream), a);
  DSA_CHECK_LAUNCH("layer_prologue");
  return DSA_OK;
}
