"""Host-side constant tables: rotary angles (YaRN) and the model constants the
path uses.  Built once in fp32 on the host and uploaded; the kernels read
rows by position on the device."""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class PathArgs:
    """Shapes and constants of the decode sparse-attention path (the subset of
    ModelArgs, inference.py:335-376, that the path reads)."""
    n_heads: int = 64
    head_dim: int = 512
    rope_head_dim: int = 64
    window_size: int = 128
    compress_ratio: int = 4
    index_n_heads: int = 64
    index_head_dim: int = 128
    index_topk: int = 512
    norm_eps: float = 1e-6
    act_quant_block: int = 64
    compress_rope_theta: float = 160000.0
    rope_theta: float = 10000.0
    original_seq_len: int = 65536
    rope_factor: float = 16.0
    beta_fast: int = 32
    beta_slow: int = 1

    @property
    def softmax_scale(self) -> float:
        return self.head_dim ** -0.5

    @property
    def index_weight_scale(self) -> float:
        """softmax_scale * H^-1/2 folded into weights_proj (inference.py:5175-5185)."""
        return self.index_head_dim ** -0.5 * self.index_n_heads ** -0.5


def rope_angles(dim: int, seqlen: int, original_seq_len: int, base: float, factor: float,
                beta_fast: int, beta_slow: int) -> torch.Tensor:
    """[seqlen, dim/2] fp32 rotary angles; with ``original_seq_len > 0`` the
    YaRN blend of interpolated and extrapolated frequencies over the
    correction band [beta_fast, beta_slow] rotations (the published YaRN
    rule that precompute_freqs_cis, inference.py:453-476, applies)."""
    base_f = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    if original_seq_len > 0:
        def band_edge(n_rot: float) -> float:
            return dim * math.log(original_seq_len / (n_rot * 2 * math.pi)) / (2 * math.log(base))
        lo = max(math.floor(band_edge(beta_fast)), 0)
        hi = min(math.ceil(band_edge(beta_slow)), dim - 1)
        span = (hi - lo) if hi != lo else 0.001
        keep = 1 - ((torch.arange(dim // 2, dtype=torch.float32) - lo) / span).clamp(0, 1)
        base_f = base_f / factor * (1 - keep) + base_f * keep
    pos = torch.arange(seqlen, dtype=torch.float32)
    return torch.outer(pos, base_f)


def rope_cos_sin(args: PathArgs, seqlen: int, compressed: bool = True, device=None):
    """(cos, sin) [seqlen, rope/2] fp32 on ``device`` for a compressed
    (theta 160000 + YaRN) or dense (theta 10000) attention layer."""
    if compressed:
        ang = rope_angles(args.rope_head_dim, seqlen, args.original_seq_len, args.compress_rope_theta,
                          args.rope_factor, args.beta_fast, args.beta_slow)
    else:
        ang = rope_angles(args.rope_head_dim, seqlen, 0, args.rope_theta, args.rope_factor,
                          args.beta_fast, args.beta_slow)
    c, s = torch.cos(ang), torch.sin(ang)
    if device is not None:
        c, s = c.to(device), s.to(device)
    return c.contiguous(), s.contiguous()


INDEXER_TOPK_BUCKETS = (128, 256, 384, 512, 640, 768, 896, 1024)


def pick_indexer_topk_bucket(t_active: int) -> int:
    """Scoring extent for ``t_active`` compressed entries: the reference's
    128-step buckets up to 1024 (inference.py:509-520), and beyond them the
    next multiple of 128 (the reference caps at 1024 because it never ran
    longer contexts; the kernels here have no such cap)."""
    for bk in INDEXER_TOPK_BUCKETS:
        if t_active <= bk:
            return bk
    return -(-t_active // 128) * 128
