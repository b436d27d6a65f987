"""CPU restatement (torch fp32) of the per-layer decode sparse-attention path.

TEST INFRASTRUCTURE ONLY - see ``oracle/__init__.py``.  Citations are
``file:line`` into the reference project zoecarver/tt-deepseek-v4.

Order of one decode step at position ``pos`` (inference.py:5888-6127):

1. ``attn.kv``       kv row -> act_quant_block on the 448 nope dims -> window
                     ring write at ``pos % W``                  (5997-6006, 6072-6079)
2. ``attn.topk``     window indices (6020-6026); indexer compressor state write
                     + emit (5247); indexer score (5260-5275); top-k (5823-5851)
3. ``attn.compress`` attention compressor state write + emit, compressed row
                     written at ``W + pos // r``                (6080-6083, 4938-5097)
4. ``attn.sparse``   gather + sink softmax attention           (6085-6093, 4459-4501)
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch

__all__ = [
    "FP8_MAX", "ACT_QUANT_EPS", "TOPK_MASK_AMP", "TOPK_VALID_MIN",
    "act_quant_fp32", "act_quant_block", "kv_quant_row", "window_indices", "window_table",
    "yarn_freqs", "rope_tables", "rotary_interleaved", "rmsnorm",
    "compressor_init_state", "compressor_state_write", "compressor_emit",
    "compressor_step", "shift_matrix_apply", "indexer_score", "indexer_topk",
    "sparse_attn", "sparse_attn_partial", "lse_combine", "topk_merge",
    "hadamard_rotate", "LayerState", "decode_layer_step", "linear_bf16",
    "head_norm_rope", "kv_norm_rope_quant", "BlockWeights", "attention_decode_block", "prefill_chunk",
]

FP8_MAX = 448.0
ACT_QUANT_EPS = 1e-4
TOPK_MASK_AMP = 1e4      # inference.py:5556-5560 (-1e4 additive mask constant)
TOPK_VALID_MIN = -1000.0  # inference.py:5845 (valid = val >= -1000)


# --------------------------------------------------------------------------
# attn.kv : act_quant_block
# --------------------------------------------------------------------------

def act_quant_fp32(x: torch.Tensor, block: int = 64, fp8_max: float = FP8_MAX,
                   eps: float = ACT_QUANT_EPS, e4m3: bool = True):
    """The act_quant round trip in fp32, before the final bf16 rounding.

    Follows the ttnn chain ``_device_act_quant_block`` (inference.py:4578-4607)
    op for op: ``amax = maximum(max(|z|), eps)``, ``s = multiply(amax,
    1 / fp8_max)`` (a multiply by the fp32 constant 1/448, inference.py:4602,
    not a division by 448), ``y = clamp(divide(z, s), -fp8_max, fp8_max)``
    (an IEEE division), ``out = multiply(y, s)``.  With ``e4m3=True`` the
    e4m3 cast of the CPU ``act_quant`` (inference.py:4582-4583,
    device-compressor-indexer/README.md:76-82) is applied to ``y``; with
    ``e4m3=False`` this is exactly the reference chain.
    Returns ``(out fp32, s fp32 [..., N/block, 1], y or its e4m3 codes)``."""
    n = x.shape[-1]
    if n % block:
        raise ValueError(f"last dim {n} must be divisible by block_size {block}")
    xf = x.float()
    z = xf.reshape(*xf.shape[:-1], n // block, block)
    amax = torch.maximum(z.abs().amax(dim=-1, keepdim=True), torch.tensor(eps, dtype=torch.float32))
    s = amax * (1.0 / fp8_max)
    y = torch.clamp(z / s, -fp8_max, fp8_max)
    if e4m3:
        q = y.to(torch.float8_e4m3fn)
        return q.float() * s, s, q
    return y * s, s, y


def act_quant_block(x: torch.Tensor, block: int = 64, fp8_max: float = FP8_MAX,
                    eps: float = ACT_QUANT_EPS):
    """Block-wise max-abs FP8-e4m3 round trip along the last dim: the
    reference chain ``_device_act_quant_block`` (inference.py:4578-4607, see
    ``act_quant_fp32``) with the CPU path's e4m3 cast, rounded to bf16.

    Returns ``(xhat bf16, scales fp32 [..., N/block], codes float8_e4m3fn)``.
    """
    out, s, q = act_quant_fp32(x, block, fp8_max, eps, e4m3=True)
    xhat = out.to(torch.bfloat16).reshape(x.shape)
    return xhat, s.squeeze(-1), q.reshape(x.shape)


def kv_quant_row(kv: torch.Tensor, rope_dim: int = 64, block: int = 64):
    """The attn.kv output row: act_quant on the nope dims, rope dims pass
    through (inference.py:5997-6006; Lk-D1 test_lk_d1.py:540-594).
    kv: [..., D] bf16 (already kv_norm'ed and rotated).  Returns
    (row bf16 [..., D], scales [..., nope/block], codes [..., nope])."""
    d = kv.shape[-1]
    nope = d - rope_dim
    xhat, s, q = act_quant_block(kv[..., :nope], block)
    row = torch.cat([xhat, kv[..., nope:].to(torch.bfloat16)], dim=-1)
    return row, s, q


# --------------------------------------------------------------------------
# attn.topk : window indices
# --------------------------------------------------------------------------

def window_indices(pos: int, win: int) -> torch.Tensor:
    """Ring-slot indices of the attended raw-token window at position ``pos``
    (inference.py:479-506 table, row pick 5491-5522 / 6020-6026):
    ``[0..pos, -1, ...]`` while ``pos < win``, else the rotation that lists
    the oldest resident slot first: ``[(pos%win)+1 .. win-1, 0 .. pos%win]``."""
    out = torch.full((win,), -1, dtype=torch.int32)
    if pos < win:
        out[: pos + 1] = torch.arange(pos + 1, dtype=torch.int32)
    else:
        r = pos % win
        out = torch.cat([torch.arange(r + 1, win, dtype=torch.int32),
                         torch.arange(0, r + 1, dtype=torch.int32)])
    return out


def window_table(win: int) -> torch.Tensor:
    """[2*win, win] table in the reference's row layout (rows [0,win): pos<win,
    rows [win,2win): pos%win) - used only to pin ``window_indices``."""
    rows = [window_indices(p, win) for p in range(win)]
    rows += [window_indices(win + s, win) for s in range(win)]
    return torch.stack(rows)


# --------------------------------------------------------------------------
# rotary / norm helpers
# --------------------------------------------------------------------------

def yarn_freqs(dim: int, seqlen: int, original_seq_len: int, base: float,
               factor: float, beta_fast: int, beta_slow: int) -> torch.Tensor:
    """Rotary angles [seqlen, dim/2] fp32 with YaRN frequency correction.
    Restates ``precompute_freqs_cis`` (inference.py:453-476), which returns
    ``polar(1, angles)``."""
    inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    if original_seq_len > 0:
        def corr_dim(rot):
            return dim * math.log(original_seq_len / (rot * 2 * math.pi)) / (2 * math.log(base))
        lo = max(math.floor(corr_dim(beta_fast)), 0)
        hi = min(math.ceil(corr_dim(beta_slow)), dim - 1)
        if lo == hi:
            hi += 0.001
        ramp = ((torch.arange(dim // 2, dtype=torch.float32) - lo) / (hi - lo)).clamp(0, 1)
        keep = 1 - ramp
        inv = inv / factor * (1 - keep) + inv * keep
    return torch.outer(torch.arange(seqlen, dtype=torch.float32), inv)


def rope_tables(dim: int, seqlen: int, compressed: bool):
    """cos/sin [seqlen, dim/2] fp32 for an attention layer.  Compressed layers
    use original_seq_len 65536 and theta 160000, others theta 10000 with no
    YaRN correction (inference.py:609-621, ModelArgs 363-372)."""
    if compressed:
        ang = yarn_freqs(dim, seqlen, 65536, 160000.0, 16.0, 32, 1)
    else:
        ang = yarn_freqs(dim, seqlen, 0, 10000.0, 16.0, 32, 1)
    return torch.cos(ang), torch.sin(ang)


def rotary_interleaved(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                       inverse: bool = False) -> torch.Tensor:
    """Interleaved-pair rotary on the last dim (pairs ``x[2k], x[2k+1]`` as a
    complex number times ``cos_k + i sin_k``), fp32.  Same convention as the
    reference's swap-matrix form (inference.py:4504-4553)."""
    xf = x.float()
    a, b = xf[..., 0::2], xf[..., 1::2]
    sn = -sin if inverse else sin
    out = torch.empty_like(xf)
    out[..., 0::2] = a * cos - b * sn
    out[..., 1::2] = a * sn + b * cos
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm in fp32 (inference.py:438-450), returned in fp32."""
    xf = x.float()
    var = xf.square().mean(-1, keepdim=True)
    return weight.float() * (xf * torch.rsqrt(var + eps))


def hadamard_rotate(x: torch.Tensor) -> torch.Tensor:
    """Orthonormal Walsh-Hadamard transform on the last dim (Sylvester order,
    scaled by d^-1/2; inference.py:4610-4631)."""
    d = x.shape[-1]
    y = x.float().clone()
    h = 1
    while h < d:
        y = y.reshape(*y.shape[:-1], d // (2 * h), 2, h)
        a, b = y[..., 0, :], y[..., 1, :]
        y = torch.stack([a + b, a - b], dim=-2).reshape(*x.shape[:-1], d)
        h *= 2
    return y * (d ** -0.5)


# --------------------------------------------------------------------------
# attn.compress : compressor state write / emit / slot shift
# --------------------------------------------------------------------------

def compressor_init_state(B: int, d: int, ratio: int, overlap: bool):
    """kv_state zeros and score_state -inf, [B, coff*r, coff*d] fp32
    (inference.py:538-551)."""
    coff = 2 if overlap else 1
    kv = torch.zeros(B, coff * ratio, coff * d, dtype=torch.float32)
    sc = torch.full((B, coff * ratio, coff * d), float("-inf"), dtype=torch.float32)
    return kv, sc


def compressor_state_write(kv_state, score_state, kv_row, score_row, ape, pos,
                           ratio: int, overlap: bool):
    """Per-step state write (inference.py:4954-4991; CPU formulas
    compressor_overlap.py:35-38, compressor_no_overlap.py:9-13):
    ``score += ape[pos % r]``; row written at slot ``r + pos % r`` (overlap)
    or ``pos % r``.  kv_row/score_row: [B, coff*d]; ``pos`` int or [B]."""
    B = kv_state.shape[0]
    pos_t = torch.as_tensor(pos).expand(B) if torch.as_tensor(pos).dim() == 0 else torch.as_tensor(pos)
    for b in range(B):
        p = int(pos_t[b])
        slot = (ratio + p % ratio) if overlap else (p % ratio)
        kv_state[b, slot] = kv_row[b].float()
        score_state[b, slot] = score_row[b].float() + ape[p % ratio].float()


def shift_matrix_apply(state: torch.Tensor, ratio: int) -> torch.Tensor:
    """Slot shift after an emit: rows [0,r) <- rows [r,2r), others unchanged
    (``out = P @ buf``, inference.py:3011-3098, P 3189-3202)."""
    out = state.clone()
    out[:, :ratio] = state[:, ratio:2 * ratio]
    return out


def compressor_emit(kv_state, score_state, gamma, cos_row, sin_row, ratio: int,
                    overlap: bool, rope_dim: int = 64, eps: float = 1e-6,
                    rotate: bool = False):
    """Emit one compressed row per batch element (inference.py:4997-5097):
    overlap view ``cat(state[:, :r, :d], state[:, r:, d:])`` (cssn masks
    3367-3380, compressor_overlap.py:44-47), fp32 softmax over the slot axis,
    weighted sum, RMSNorm(gamma, eps) (cssn 3205-3364), interleaved rotary on
    the last ``rope_dim`` dims with ``freqs_cis[pos+1-r]``, optional Hadamard
    (compressor_overlap_rotate.py:16-23).  fp32 throughout, one bf16
    rounding at the end.  Does NOT shift the state (see compressor_step).
    cos_row/sin_row: [B, rope_dim/2] or [rope_dim/2]."""
    if overlap:
        d = kv_state.shape[-1] // 2
        kv_v = torch.cat([kv_state[:, :ratio, :d], kv_state[:, ratio:2 * ratio, d:]], dim=1)
        sc_v = torch.cat([score_state[:, :ratio, :d], score_state[:, ratio:2 * ratio, d:]], dim=1)
    else:
        kv_v, sc_v = kv_state, score_state
    p = torch.softmax(sc_v.float(), dim=1)
    kv = (kv_v.float() * p).sum(dim=1)
    kv = rmsnorm(kv, gamma, eps)
    nope = kv.shape[-1] - rope_dim
    kv = torch.cat([kv[..., :nope], rotary_interleaved(kv[..., nope:], cos_row, sin_row)], dim=-1)
    if rotate:
        kv = hadamard_rotate(kv)
    return kv.to(torch.bfloat16)


def compressor_step(kv_state, score_state, kv_row, score_row, ape, gamma, cos, sin,
                    pos: int, ratio: int, overlap: bool, kv_cache=None,
                    slot_offset: int = 0, rope_dim: int = 64, eps: float = 1e-6,
                    rotate: bool = False):
    """One DeviceCompressor.forward_device decode step (inference.py:4938-4995):
    state write, then on ``(pos+1) % r == 0`` emit, cache write at
    ``slot_offset + pos // r`` and (overlap) slot shift.  Returns the emitted
    rows [B, d] bf16 or None; updates the state tensors in place."""
    compressor_state_write(kv_state, score_state, kv_row, score_row, ape, pos, ratio, overlap)
    if (pos + 1) % ratio != 0:
        return None
    row = pos + 1 - ratio
    out = compressor_emit(kv_state, score_state, gamma, cos[row], sin[row], ratio,
                          overlap, rope_dim, eps, rotate)
    if kv_cache is not None:
        kv_cache[:, slot_offset + pos // ratio] = out
    if overlap:
        kv_state.copy_(shift_matrix_apply(kv_state, ratio))
        score_state.copy_(shift_matrix_apply(score_state, ratio))
    return out


# --------------------------------------------------------------------------
# attn.topk : indexer score + top-k
# --------------------------------------------------------------------------

def indexer_score(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``s[b,t] = sum_h w[b,h] * relu(q[b,h,:] . k[b,t,:])`` in fp32
    (inference.py:5260-5275; CPU formula indexer.py:10-23).
    q [B,H,Di], k [B,T,Di], w [B,H] (already scaled) -> [B,T] fp32."""
    sc = torch.einsum("bhd,btd->bht", q.float(), k.float())
    return (sc.relu() * w.float().unsqueeze(-1)).sum(dim=1)


def indexer_topk(score: torch.Tensor, t_active, k: int, win: int,
                 sorted_out: bool = True) -> torch.Tensor:
    """Bucketed pad+mask top-k (inference.py:5823-5851; ttnn reference chain
    test_lk_d_topk.py:121-138): ``masked = score - 1e4 * (t >= T_active)``;
    ``topk(masked, k)`` largest first; ``idx + win`` where ``val >= -1000``
    else ``-1``.  score [B, T_pad] fp32; t_active int or [B]; k <= T_pad."""
    B, T = score.shape
    ta = torch.as_tensor(t_active).reshape(-1).expand(B) if torch.as_tensor(t_active).dim() == 0 \
        else torch.as_tensor(t_active)
    ramp = torch.arange(T).unsqueeze(0)
    masked = score.float() - TOPK_MASK_AMP * (ramp >= ta.unsqueeze(1)).float()
    vals, idx = torch.topk(masked, k, dim=-1, largest=True, sorted=True)
    out = torch.where(vals >= TOPK_VALID_MIN, idx.to(torch.int32) + win,
                      torch.full_like(idx, -1, dtype=torch.int32))
    return out.to(torch.int32)


def topk_merge(cand_score: torch.Tensor, cand_idx: torch.Tensor, k: int):
    """Global top-k from per-shard candidate lists (sequence split; the plan in
    briefs/future_max_utilization.md:177-204).  cand_*: [G*k'] -> top k by
    score (ties: lower global index first)."""
    order = sorted(range(cand_score.numel()),
                   key=lambda i: (-float(cand_score[i]), int(cand_idx[i])))
    sel = order[:k]
    return cand_score[sel], cand_idx[sel]


# --------------------------------------------------------------------------
# attn.sparse : gather + sink softmax attention
# --------------------------------------------------------------------------

def sparse_attn_partial(q: torch.Tensor, kv: torch.Tensor, idx: torch.Tensor,
                        scale: float):
    """Un-normalised partial attention over the rows ``idx`` (-1 = masked):
    returns (m [.., H], l [.., H], o [.., H, D]) with ``o = sum e^{z-m} v`` and
    ``l = sum e^{z-m}`` (no sink) - the split-K building block (a12).
    q [M,H,D] bf16, kv [M,N,D] (per query row), idx [M,K]."""
    qf = q.float()
    safe = idx.clamp_min(0).long()
    g = torch.gather(kv.float(), 1, safe.unsqueeze(-1).expand(-1, -1, kv.shape[-1]))
    z = torch.einsum("mhd,mkd->mhk", qf, g) * scale
    z = z.masked_fill((idx < 0).unsqueeze(1), float("-inf"))
    m = z.amax(dim=-1)
    msafe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    p = torch.exp(z - msafe.unsqueeze(-1))
    l = p.sum(-1)
    o = torch.einsum("mhk,mkd->mhd", p, g)
    return m, l, o


def lse_combine(parts, sink: torch.Tensor) -> torch.Tensor:
    """Merge partials ``(m_s, l_s, o_s)`` with the sink counted once:
    ``M = max(max_s m_s, sink)``, ``L = sum l_s e^{m_s-M} + e^{sink-M}``,
    ``o = sum o_s e^{m_s-M} / L``.  Returns fp32 o."""
    sinkf = sink.float()
    M = sinkf.expand_as(parts[0][0]).clone()
    for m, _, _ in parts:
        M = torch.maximum(M, m)
    L = torch.exp(sinkf - M)
    O = torch.zeros_like(parts[0][2])
    for m, l, o in parts:
        f = torch.where(torch.isinf(m), torch.zeros_like(m), torch.exp(m - M))
        L = L + l * f
        O = O + o * f.unsqueeze(-1)
    return O / L.unsqueeze(-1)


def sparse_attn(q: torch.Tensor, kv: torch.Tensor, idx: torch.Tensor,
                sink: torch.Tensor, scale: float) -> torch.Tensor:
    """``DeviceSparseAttn.forward_device`` (inference.py:4459-4501, mask
    4444-4457): gather ``kv[safe]``, ``z = q.kv^T * scale + (idx<0 ? -inf : 0)``,
    ``m = max(max z, sink)``, ``p = e^{z-m} / (sum e^{z-m} + e^{sink-m})``,
    ``o = p . kv`` (K = V = the 512-d latent, MQA).
    q [B,S,H,D] or [M,H,D]; kv [B,N,D] (query row m reads kv[m // S]);
    idx [B,S,K] or [M,K]; sink [H] -> o like q, bf16."""
    shp = q.shape
    if q.dim() == 4:
        B, S = shp[0], shp[1]
        q3 = q.reshape(B * S, shp[2], shp[3])
        idx2 = idx.reshape(B * S, idx.shape[-1])
        kv3 = kv.repeat_interleave(S, dim=0) if S > 1 else kv
    else:
        q3, idx2, kv3 = q, idx, kv
    m, l, o = sparse_attn_partial(q3, kv3, idx2, scale)
    out = lse_combine([(m, l, o)], sink.float().unsqueeze(0))
    return out.to(torch.bfloat16).reshape(shp)


# --------------------------------------------------------------------------
# one full layer decode step
# --------------------------------------------------------------------------

@dataclass
class LayerState:
    """Per-layer persistent decode state for B sequences (the buffers that
    DeviceAttention/_alloc_decode_tensors own, inference.py:5460-5580 and
    DeviceCompressor 4757-4813)."""
    kv_cache: torch.Tensor            # [B, W + T_max, D] bf16
    idx_kv_cache: torch.Tensor        # [B, T_max, Di] bf16 (indexer keys)
    cmp_kv: torch.Tensor              # attention compressor state
    cmp_sc: torch.Tensor
    icmp_kv: torch.Tensor             # indexer compressor state
    icmp_sc: torch.Tensor
    ape: torch.Tensor                 # [r, 2D] fp32
    gamma: torch.Tensor               # [D]
    iape: torch.Tensor                # [r, 2Di]
    igamma: torch.Tensor              # [Di]
    sink: torch.Tensor                # [H] fp32
    cos: torch.Tensor                 # [max_seq, rope/2]
    sin: torch.Tensor
    win: int = 128
    ratio: int = 4
    index_topk: int = 512
    scale: float = 512 ** -0.5
    extra: dict = field(default_factory=dict)


def decode_layer_step(st: LayerState, pos: int, q, kv_row, cmp_kv_row, cmp_sc_row,
                      iq, icmp_kv_row, icmp_sc_row, iw):
    """One decode step of the path for B sequences at the same ``pos``
    (inference.py:5888-6093 ordering; SURVEY call-stack 3.2):
    kv quant -> window write; indexer compressor step; indexer score + top-k;
    attention compressor step; sparse attention.  Returns (o, topk_idxs)."""
    W, r = st.win, st.ratio
    row, _, _ = kv_quant_row(kv_row)
    st.kv_cache[:, pos % W] = row
    win_idx = window_indices(pos, W)
    B = q.shape[0]
    t_active = (pos + 1) // r
    compressor_step(st.icmp_kv, st.icmp_sc, icmp_kv_row, icmp_sc_row, st.iape, st.igamma,
                    st.cos, st.sin, pos, r, True, kv_cache=st.idx_kv_cache, slot_offset=0)
    idx = win_idx.unsqueeze(0).expand(B, W)
    st.extra["score"] = None
    if t_active > 0:
        T_pad = t_active
        score = indexer_score(iq, st.idx_kv_cache[:, :T_pad], iw)
        st.extra["score"] = score          # for near-tie checks of a selection
        k = min(st.index_topk, T_pad)
        cidx = indexer_topk(score, t_active, k, W)
        idx = torch.cat([idx, cidx], dim=-1)
    compressor_step(st.cmp_kv, st.cmp_sc, cmp_kv_row, cmp_sc_row, st.ape, st.gamma,
                    st.cos, st.sin, pos, r, True, kv_cache=st.kv_cache, slot_offset=W)
    o = sparse_attn(q, st.kv_cache, idx, st.sink, st.scale)
    return o, idx


# --------------------------------------------------------------------------
# around the path: q path, Lk-D1 kv path, output side, the whole block
# --------------------------------------------------------------------------

def linear_bf16(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """bf16 projection with fp32 accumulation, rounded to bf16 (the device
    matmuls of inference.py:5934-5960; the CPU Linear is F.linear, 390-396)."""
    return (x.to(torch.bfloat16).float() @ w.to(torch.bfloat16).float().t()).to(torch.bfloat16)


def head_norm_rope(x: torch.Tensor, n_heads: int, head_dim: int, cos_row=None, sin_row=None,
                   rope_dim: int = 0, gamma=None, weight: float = 1.0, norm: bool = True,
                   eps: float = 1e-6, inverse: bool = False) -> torch.Tensor:
    """Per-head RMSNorm (result rounded to bf16 as RMSNorm returns the input
    dtype, inference.py:436-450) with weight ``gamma`` or the scalar
    ``weight`` (q_rsqrt_ones = softmax_scale, 5348-5350, 5982-5983), then
    interleaved rotary of the last ``rope_dim`` dims (5990; inverse for the
    output side, 6102).  x [B, n_heads*head_dim] -> bf16 same shape.
    cos_row/sin_row: [B, rope_dim/2]."""
    B = x.shape[0]
    xs = x.float().reshape(B, n_heads, head_dim)
    if norm:
        w = gamma.float() if gamma is not None else torch.full((head_dim,), float(weight))
        xs = rmsnorm(xs, w, eps).to(torch.bfloat16).float()
    if rope_dim:
        c = cos_row.float().reshape(B, 1, -1)
        s = sin_row.float().reshape(B, 1, -1)
        xs = torch.cat([xs[..., :head_dim - rope_dim],
                        rotary_interleaved(xs[..., head_dim - rope_dim:], c, s, inverse)], dim=-1)
    return xs.to(torch.bfloat16).reshape(x.shape)


def kv_norm_rope_quant(kv: torch.Tensor, gamma: torch.Tensor, cos_row, sin_row,
                       eps: float = 1e-6, rope_dim: int = 64):
    """The Lk-D1 zone (inference.py:5997-6006, test_lk_d1.py:498-594):
    kv_norm -> bf16 -> rotary on the rope dims -> act_quant on the nope dims.
    Returns (row bf16 [B, D], scales, codes)."""
    D = kv.shape[-1]
    y = head_norm_rope(kv, 1, D, cos_row, sin_row, rope_dim, gamma=gamma, eps=eps)
    return kv_quant_row(y, rope_dim)


@dataclass
class BlockWeights:
    """Weights of one compressed attention block (the CPU Attention,
    inference.py:576-623; Compressor 523-552; Indexer 554-574)."""
    wq_a: torch.Tensor          # [q_lora, dim]
    q_norm: torch.Tensor        # [q_lora]
    wq_b: torch.Tensor          # [H*D, q_lora]
    wkv: torch.Tensor           # [D, dim]
    kv_norm: torch.Tensor       # [D]
    wo_a: torch.Tensor          # [G*R, H*D/G]
    wo_b: torch.Tensor          # [dim, G*R]
    c_wkv: torch.Tensor         # [2D, dim]  attention compressor
    c_wgate: torch.Tensor       # [2D, dim]
    i_wq_b: torch.Tensor        # [Hi*Di, q_lora]
    i_wproj: torch.Tensor       # [Hi, dim]
    i_wkv: torch.Tensor         # [2Di, dim] indexer compressor
    i_wgate: torch.Tensor       # [2Di, dim]
    n_groups: int = 8
    eps: float = 1e-6


def attention_decode_block(bw: BlockWeights, st: LayerState, x: torch.Tensor, pos: int,
                           n_heads: int = 64, head_dim: int = 512, rope_dim: int = 64,
                           index_n_heads: int = 64, index_head_dim: int = 128) -> torch.Tensor:
    """DeviceAttention.forward_device for one token per sequence
    (inference.py:5888-6127): q path (wq_a, q_norm, wq_b, per-head rms with
    weight softmax_scale, rotary), kv path (wkv, Lk-D1, window write), the
    indexer (wq_b + rotary on q, its compressor, weights_proj scaled by
    softmax_scale * Hi^-1/2, 5175-5185), top-k, the attention compressor,
    sparse attention with q pre-scaled, inverse rotary, grouped wo_a, wo_b.
    x [B, 1, dim] -> [B, 1, dim] bf16; st.scale must be 1.0 (q carries it)."""
    B = x.shape[0]
    x2 = x.reshape(B, -1)
    H, D, Hi, Di = n_heads, head_dim, index_n_heads, index_head_dim
    cr, sr = st.cos[pos].expand(B, -1), st.sin[pos].expand(B, -1)
    q_lora = linear_bf16(x2, bw.wq_a)
    qr = head_norm_rope(q_lora, 1, q_lora.shape[-1], gamma=bw.q_norm, eps=bw.eps)
    q = linear_bf16(qr, bw.wq_b)
    q = head_norm_rope(q, H, D, cr, sr, rope_dim, weight=D ** -0.5, eps=bw.eps).view(B, H, D)
    kv = head_norm_rope(linear_bf16(x2, bw.wkv), 1, D, cr, sr, rope_dim, gamma=bw.kv_norm, eps=bw.eps)
    iq = linear_bf16(qr, bw.i_wq_b)
    iq = head_norm_rope(iq, Hi, Di, cr, sr, rope_dim, norm=False).view(B, Hi, Di)
    iw = linear_bf16(x2, (bw.i_wproj.float() * (Di ** -0.5 * Hi ** -0.5)).to(torch.bfloat16)).float()
    o, idx = decode_layer_step(st, pos, q, kv, linear_bf16(x2, bw.c_wkv), linear_bf16(x2, bw.c_wgate),
                               iq, linear_bf16(x2, bw.i_wkv), linear_bf16(x2, bw.i_wgate), iw)
    o = head_norm_rope(o.reshape(B, H * D), H, D, cr, sr, rope_dim, norm=False, inverse=True)
    G = bw.n_groups
    R = bw.wo_a.shape[0] // G
    og = o.view(B, G, H * D // G).float()
    wa = bw.wo_a.to(torch.bfloat16).float().view(G, R, H * D // G)
    a = torch.einsum("bgi,gri->bgr", og, wa).to(torch.bfloat16).reshape(B, G * R)
    return linear_bf16(a, bw.wo_b).view(B, 1, -1)


# --------------------------------------------------------------------------
# multi-token (prefill chunk)
# --------------------------------------------------------------------------

def prefill_chunk(q, kv, n_raw: int, iq, ikeys, iw, sink, base: int, n_hist: int, T: int,
                  k: int, W: int = 128, ratio: int = 4, scale: float = 512 ** -0.5, rows=None):
    """S tokens at positions base..base+S-1, each attending its own top-k of
    the compressed entries it may see (t < (p + 1) // ratio, the T_active
    rule of inference.py:6028 per token) plus its causal window of W raw
    tokens; indexer score and top-k as in the decode step (indexer.py:10-23,
    inference.py:5823-5851), sink attention as inference.py:4459-4501.
    kv: [n_raw + T', D] raw rows (n_hist before the chunk, then the chunk)
    followed by the compressed entries.  ``rows``: chunk offsets of the
    given tokens (default 0..S-1) when checking a sample of a chunk.
    Returns (o [S, H, D] bf16, idx)."""
    S = q.shape[0]
    rows = list(range(S)) if rows is None else list(rows)
    sc = torch.einsum("shd,td->sht", iq.float(), ikeys[:T].float())
    score = (sc.relu() * iw.float().unsqueeze(-1)).sum(dim=1)
    ta = torch.tensor([min(T, (base + s + 1) // ratio) for s in rows])
    cidx = indexer_topk(score, ta, k, n_raw)
    win = torch.tensor([[s + i + n_hist - (W - 1) for i in range(W)] for s in rows], dtype=torch.int32)
    win = torch.where(win >= 0, win, torch.full_like(win, -1))
    idx = torch.cat([win, cidx], dim=1)
    kv3 = kv.unsqueeze(0).expand(S, -1, -1)
    o = sparse_attn(q, kv3, idx, sink, scale)
    return o, idx
