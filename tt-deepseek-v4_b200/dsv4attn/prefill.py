"""Multi-token (prefill-chunk) sparse attention for one layer.

S new tokens at positions base .. base+S-1 of one sequence attend, each,
to its own indexer top-k of the compressed entries it may see and to its
causal window of the last W raw tokens (the multi-token QK^T / PV case of
the path).  Per chunk:

  positions   t_active[s] = (p + 1) // ratio and the window rows   (1 launch)
  indexer     dense [S*64 x 128] x [128 x T] contraction on the tensor
              cores, relu * w reduced over heads in the epilogue, causal
              rows skipped (t >= t_active[s])                      (1 launch)
  top-k       per token, k of T (two levels when T > 16384)        (2 launches)
  attention   S query rows x (W + k) gathered rows, sink softmax   (1-2 launches)

Buffers are owned by the object and sized at construction, so ``run`` can
be captured in a CUDA graph.  The decode path (layer.py) is the S = 1 case
with a ring window; the reference runs prefill as a loop of decode steps
(inference.py:5757-5766), so this is the chunked form of that loop, with
every token's selection made against the cache as it stands when the
chunk starts (all compressed entries written before the chunk).
"""

from __future__ import annotations

import torch

from . import ops
from .tables import PathArgs

BF16 = torch.bfloat16
F32 = torch.float32
I32 = torch.int32


class PrefillChunk:
    """Scratch and launch sequence of one prefill chunk of S tokens over a
    compressed cache of up to T_cap entries."""

    def __init__(self, args: PathArgs, S: int, T_cap: int, device, k: int | None = None):
        self.args = args
        self.S = S
        self.T_cap = T_cap
        self.W = args.window_size
        self.k = args.index_topk if k is None else k
        if self.k > T_cap:
            raise ValueError(f"index_topk {self.k} > compressed capacity {T_cap}")
        dev = self.device = torch.device(device)
        self.score = torch.zeros(S, T_cap, dtype=F32, device=dev)
        self.t_active = torch.zeros(S, dtype=I32, device=dev)
        self.idx = torch.full((S, self.W + self.k), -1, dtype=I32, device=dev)
        self.status = torch.zeros(1, dtype=I32, device=dev)
        L = ops.lib()
        self.ws = ops.Workspace(dev, max(int(L.dsa_indexer_topk_workspace_size(S, T_cap, self.k)),
                                         int(L.dsa_sparse_attn_workspace_size(1, S, args.n_heads, args.head_dim,
                                                                              self.W + self.k))))

    def run(self, q: torch.Tensor, kv: torch.Tensor, n_raw: int, iq: torch.Tensor, ikeys: torch.Tensor,
            iw: torch.Tensor, sink: torch.Tensor, base: int, n_hist: int, T: int, out: torch.Tensor | None = None,
            scale: float | None = None) -> torch.Tensor:
        """q [S, H, D] bf16; kv [n_raw + >=T, D] bf16 - the raw rows (n_hist
        tokens before the chunk, then the chunk) followed by the compressed
        entries; iq [S, Hi, Di] bf16; ikeys [>=T, Di] bf16; iw [S, Hi] fp32
        (scale folded); sink [H] fp32.  Returns o [S, H, D] bf16."""
        a, S, W = self.args, self.S, self.W
        if q.shape[0] != S or iq.shape[0] != S or iw.shape[0] != S:
            raise ValueError(f"chunk built for S={S} tokens")
        if T > self.T_cap or self.k > T:
            raise ValueError(f"T={T} outside (k={self.k}, T_cap={self.T_cap}]")
        if n_raw != n_hist + S or kv.shape[0] < n_raw + T:
            raise ValueError("kv must hold n_hist + S raw rows followed by the compressed entries")
        ops.prefill_positions(S, base, T, W, n_hist, a.compress_ratio, self.t_active, self.idx)
        ops.indexer_score(iq, ikeys, iw, T, out=self.score, t_valid=self.t_active)
        ops.indexer_topk(self.score, self.t_active, self.k, n_raw, T=T, mask_mode=1, out=self.idx[:, W:],
                         ws=self.ws)
        if out is None:
            out = torch.empty_like(q)
        sc = a.softmax_scale if scale is None else scale
        ops.sparse_attn(q.view(1, S, a.n_heads, a.head_dim), kv.unsqueeze(0), self.idx.view(1, S, W + self.k),
                        sink, sc, out=out.view(1, S, a.n_heads, a.head_dim), ws=self.ws, status=self.status)
        return out

    def flops(self, T: int) -> dict:
        """Algorithmic FLOPs of one chunk (dense indexer, attention)."""
        a = self.args
        return {"indexer": 2 * self.S * a.index_n_heads * a.index_head_dim * T,
                "attention": 4 * self.S * a.n_heads * a.head_dim * (self.W + self.k)}
