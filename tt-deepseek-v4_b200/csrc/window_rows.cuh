// The window ring slots of one sequence's query (window_indices_kernel in
// topk.cu and the decode layer's prologue kernel in prologue.cu): entry i of
// idx[b] is the ring slot of the i-th oldest of the last min(pos + 1, win)
// tokens, -1 for slots not yet written (inference.py:479-506, picked at
// 6020-6026).
#pragma once

#include "common.cuh"

namespace dsa {

__device__ __forceinline__ void window_indices_row(const int32_t* __restrict__ pos, int32_t* __restrict__ idx,
                                                   int64_t ld, int win, int b) {
  const int p = pos[b];
  for (int i = threadIdx.x; i < win; i += blockDim.x) {
    int v;
    if (p < win) v = (i <= p) ? i : -1;
    else v = (p % win + 1 + i) % win;
    idx[int64_t(b) * ld + i] = v;
  }
}

}  // namespace dsa
