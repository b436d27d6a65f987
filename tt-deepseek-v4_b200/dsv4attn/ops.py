"""Functional torch-tensor wrappers over the C ABI.

Every function takes CUDA tensors, validates dtype / device / layout, calls
the native entry point on ``torch.cuda.current_stream()`` and returns the
output tensor(s).  Outputs may be passed in (``out=``) so a caller can keep
all buffers persistent (CUDA-graph capture); nothing here synchronises.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import DSA_KEYS_READY, check, lib

BF16 = torch.bfloat16
I32 = torch.int32
F32 = torch.float32


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _need(t: torch.Tensor, name: str, dtype=None, cuda=True):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if cuda and not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU fallback)")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")


def _contig(t: torch.Tensor, name: str):
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _ptr(t):
    return None if t is None else t.data_ptr()


class Workspace:
    """Grow-only per-device scratch buffer owned by the caller (allocate it
    before CUDA-graph capture; the native calls never allocate)."""

    def __init__(self, device, nbytes: int = 0):
        self.device = torch.device(device)
        self.buf = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=self.device)

    def get(self, nbytes: int) -> torch.Tensor:
        if nbytes > self.buf.numel():
            self.buf = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        return self.buf

    @property
    def nbytes(self) -> int:
        return self.buf.numel()


_default_ws: dict = {}

# bits of the device status words the kernels set (the ``status`` tensors)
STATUS_BAD_INDEX = 1   # an attention index fell outside the cache (clamped)
STATUS_TIMEOUT = 2     # a bounded device wait ran out (lost arrival, missing peer)


def set_wait_limit(cycles: int) -> int:
    """Set the spin budget (SM clock cycles) of every bounded device wait
    of the library (``dsa_set_wait_limit``; <= 0 restores ~1 s); returns
    the previous budget.  Kernels already captured in a graph keep theirs."""
    L = lib()
    prev = int(L.dsa_get_wait_limit())
    check(L.dsa_set_wait_limit(int(cycles)), "set_wait_limit")
    return prev


def raise_for_status(status: torch.Tensor, what: str) -> None:
    """Read a device status word (synchronises) and map it to the
    reference's error types: TimeoutError when a bounded wait ran out,
    RuntimeError for any other device error."""
    v = int(status.reshape(-1)[0].item())
    if v & STATUS_TIMEOUT:
        raise TimeoutError(f"{what}: a bounded device wait ran out (status {v}); "
                           "a peer or an arrival never came")
    if v:
        raise RuntimeError(f"{what}: device status {v} (bit 1: an index fell outside the cache)")


def _ws(device, nbytes: int, ws: Workspace | None) -> Workspace:
    if ws is None:
        key = torch.device(device)
        ws = _default_ws.get(key)
        if ws is None:
            ws = _default_ws[key] = Workspace(key)
    ws.get(nbytes)
    return ws


# ------------------------------------------------------- projections

class LinearWeight:
    """A projection weight W [G*N, K] stored once in the tile layout the
    kernel streams (dsa_linear_pack): ``packed`` is a uint8 device tensor,
    ``N`` rows per group, ``K`` inputs per group, ``G`` groups."""

    __slots__ = ("packed", "N", "K", "G")

    def __init__(self, packed: torch.Tensor, N: int, K: int, G: int):
        self.packed, self.N, self.K, self.G = packed, N, K, G

    @property
    def device(self):
        return self.packed.device

    @property
    def shape(self):
        return (self.G * self.N, self.K)


def pack_linear_weight(w: torch.Tensor, groups: int = 1) -> LinearWeight:
    """W [G*N, K] bf16 (CUDA, contiguous, K a multiple of 64) -> LinearWeight."""
    _need(w, "w", BF16)
    _contig(w, "w")
    if w.dim() != 2 or w.shape[0] % groups:
        raise ValueError(f"w {tuple(w.shape)} does not form {groups} groups")
    N, K = w.shape[0] // groups, w.shape[1]
    nbytes = lib().dsa_linear_packed_bytes(N, K, groups)
    if nbytes == 0:
        raise ValueError(f"w [{w.shape[0]}, {K}]: K must be a multiple of 64")
    packed = torch.empty(nbytes, dtype=torch.uint8, device=w.device)
    check(lib().dsa_linear_pack(w.data_ptr(), N, K, groups, packed.data_ptr(), nbytes, _stream(w)), "linear_pack")
    return LinearWeight(packed, N, K, groups)


def linear(x: torch.Tensor, w, out: torch.Tensor | None = None, groups: int = 1,
           out_f32: bool = False, rope: tuple | None = None, status: torch.Tensor | None = None) -> torch.Tensor:
    """``y[b, g*N + n] = bf16(x[b, g*K:(g+1)*K] . W[g*N + n])`` on the tensor
    cores (dsa_linear): x [B, G*K] bf16 (row stride a multiple of 8), ``w`` a
    LinearWeight (its groups win over ``groups``) or W [G*N, K] bf16, which is
    packed for this call, K a multiple of 64 -> y [B, G*N] bf16, or fp32 of
    the bf16 value with ``out_f32``.  ``rope=(cos, sin, pos, head_dim,
    rope_dim[, col0])``: interleaved rotary on the last rope_dim columns of
    every head_dim block of columns [col0, N) (default 0), at per-row
    positions ``pos`` [B] int32."""
    _need(x, "x", BF16)
    if not isinstance(w, LinearWeight):
        w = pack_linear_weight(w, groups)
    _need(w.packed, "w")
    groups, N, K = w.G, w.N, w.K
    GN = groups * N
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be [B, G*K] with contiguous rows")
    B = x.shape[0]
    if x.shape[1] != groups * K:
        raise ValueError(f"x [{B}, {x.shape[1]}] does not match {groups} groups of K={K}")
    if out is None:
        out = torch.empty(B, GN, dtype=F32 if out_f32 else BF16, device=x.device)
    _need(out, "out", F32 if out_f32 else BF16)
    if out.dim() != 2 or out.stride(1) != 1 or out.shape[0] < B or out.shape[1] < GN:
        raise ValueError("out must be [B, G*N] with contiguous rows")
    cos = sin = pos = None
    n_pos = head_dim = rope_dim = col0 = 0
    if rope is not None:
        cos, sin, pos, head_dim, rope_dim = rope[:5]
        col0 = rope[5] if len(rope) > 5 else 0
        _need(cos, "cos", F32)
        _need(sin, "sin", F32)
        _need(pos, "pos", I32)
        _contig(pos, "pos")
        if pos.numel() < B or cos.shape != sin.shape or cos.dim() != 2 or cos.shape[1] * 2 != rope_dim:
            raise ValueError("rope: pos needs one entry per row and cos/sin [n_pos, rope_dim/2]")
        _contig(cos, "cos")
        _contig(sin, "sin")
        n_pos = cos.shape[0]
    check(lib().dsa_linear(x.data_ptr(), x.stride(0), w.packed.data_ptr(), out.data_ptr(), out.stride(0), B, N, K,
                           groups, int(out_f32), _ptr(cos), _ptr(sin), n_pos, _ptr(pos), head_dim, rope_dim, col0,
                           _ptr(status), _stream(x)), "linear")
    return out


# ------------------------------------------------------------------ attn.kv

def act_quant_block(x: torch.Tensor, block: int = 64, fp8_max: float = 448.0, eps: float = 1e-4,
                    out: torch.Tensor | None = None, scales: torch.Tensor | None = None,
                    codes: torch.Tensor | None = None):
    """Block-wise e4m3 round trip along the last dim (inference.py:3383-3499,
    4578-4607).  Returns ``(out, scales, codes)``; scales/codes are filled only
    when passed in or requested with ``scales=True`` / ``codes=True``."""
    _need(x, "x", BF16)
    if x.stride(-1) != 1:
        raise ValueError("x must have a unit stride in the last dim")
    N = x.shape[-1]
    if N % block:
        raise ValueError(f"last dim {N} must be divisible by block_size {block}")
    x2 = x.reshape(-1, N)
    M = x2.shape[0]
    if out is None:
        out = torch.empty_like(x)
    out2 = out.view(-1, N)
    if scales is True:
        scales = torch.empty(*x.shape[:-1], N // block, dtype=F32, device=x.device)
    if codes is True:
        codes = torch.empty(*x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    check(lib().dsa_act_quant_block(x2.data_ptr(), out2.data_ptr(), _ptr(scales), _ptr(codes), M, N,
                                    x2.stride(0), out2.stride(0), block, fp8_max, eps, _stream(x)),
          "act_quant_block")
    return out, scales, codes


def kv_window_write(kv: torch.Tensor, kv_cache: torch.Tensor, pos: torch.Tensor, win: int,
                    rope_dim: int = 64, scales: torch.Tensor | None = None) -> None:
    """act_quant on the nope dims of ``kv [B, D]`` and ring write into
    ``kv_cache[b, pos[b] % win]`` (inference.py:5997-6006, 6072-6079)."""
    _need(kv, "kv", BF16)
    _need(kv_cache, "kv_cache", BF16)
    _need(pos, "pos", I32)
    _contig(kv, "kv")
    B, D = kv.shape
    if kv_cache.dim() != 3 or kv_cache.shape[0] < B or kv_cache.shape[2] != D or kv_cache.stride(1) != D:
        raise ValueError("kv_cache must be [B, rows, D] with contiguous rows")
    check(lib().dsa_kv_window_write(kv.data_ptr(), kv_cache.data_ptr(), _ptr(scales), pos.data_ptr(), B, D,
                                    rope_dim, kv_cache.stride(0), win, 64, _stream(kv)), "kv_window_write")


def kv_norm_rope_window_write(kv: torch.Tensor, gamma: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                              pos: torch.Tensor, kv_cache: torch.Tensor, win: int, eps: float = 1e-6,
                              rope_dim: int = 64, kv_out: torch.Tensor | None = None,
                              scales: torch.Tensor | None = None, status: torch.Tensor | None = None) -> None:
    """kv_norm -> rotary -> act_quant(nope) -> ring write at ``pos % win``
    in one launch (Lk-D1 + attn.kv_update, inference.py:5997-6006,
    6072-6079).  kv [B, D] bf16 (wkv output); gamma [D] fp32; cos/sin
    [n_pos, rope/2] fp32; kv_cache [B, rows, D] bf16."""
    _need(kv, "kv", BF16)
    _need(gamma, "gamma", F32)
    _need(cos, "cos", F32)
    _need(sin, "sin", F32)
    _need(pos, "pos", I32)
    _need(kv_cache, "kv_cache", BF16)
    for t, n in ((gamma, "gamma"), (cos, "cos"), (sin, "sin"), (pos, "pos")):
        _contig(t, n)
    if kv.dim() != 2 or kv.stride(-1) != 1:
        raise ValueError("kv must be [B, D] with a unit stride in the last dim")
    B, D = kv.shape
    if gamma.numel() != D:
        raise ValueError(f"gamma has {gamma.numel()} elements, expected {D}")
    if kv_cache.dim() != 3 or kv_cache.shape[0] < B or kv_cache.shape[2] != D or kv_cache.stride(1) != D:
        raise ValueError("kv_cache must be [B, rows, D] with contiguous rows")
    if cos.shape != sin.shape or cos.shape[-1] * 2 != rope_dim:
        raise ValueError(f"cos/sin must be [n_pos, {rope_dim // 2}]")
    ld_out = 0
    if kv_out is not None:
        _need(kv_out, "kv_out", BF16)
        ld_out = kv_out.stride(0)
    check(lib().dsa_kv_norm_rope_window_write(kv.data_ptr(), kv.stride(0), gamma.data_ptr(), eps, cos.data_ptr(),
                                              sin.data_ptr(), cos.shape[0], pos.data_ptr(), kv_cache.data_ptr(),
                                              kv_cache.stride(0), win, _ptr(kv_out), ld_out, _ptr(scales), B, D,
                                              rope_dim, _ptr(status), _stream(kv)), "kv_norm_rope_window_write")


def head_norm_rope(x: torch.Tensor, n_heads: int, head_dim: int, cos=None, sin=None, pos=None, rope_dim: int = 0,
                   gamma: torch.Tensor | None = None, weight: float = 1.0, norm: bool = True, eps: float = 1e-6,
                   inverse: bool = False, out: torch.Tensor | None = None,
                   status: torch.Tensor | None = None) -> torch.Tensor:
    """Per-head RMSNorm (gamma [head_dim] or scalar ``weight``) and/or
    interleaved rotary of the last ``rope_dim`` dims at ``pos[b]`` for x
    [B, ..., n_heads*head_dim] bf16 (inference.py:5982-5991, 6032-6034,
    6100-6102).  ``out`` may be ``x`` (in place)."""
    _need(x, "x", BF16)
    if x.stride(-1) != 1:
        raise ValueError("x must have a unit stride in the last dim")
    B = x.numel() // (n_heads * head_dim)
    x2 = x.reshape(B, n_heads * head_dim)
    if out is None:
        out = torch.empty_like(x)
    o2 = out.view(B, n_heads * head_dim) if out.is_contiguous() else out.reshape(B, n_heads * head_dim)
    if o2.data_ptr() != out.data_ptr():
        raise ValueError("out must be viewable as [B, n_heads*head_dim]")
    if gamma is not None:
        _need(gamma, "gamma", F32)
        _contig(gamma, "gamma")
        if gamma.numel() != head_dim:
            raise ValueError(f"gamma has {gamma.numel()} elements, expected {head_dim}")
    n_pos = 0
    if rope_dim:
        for t, n in ((cos, "cos"), (sin, "sin")):
            _need(t, n, F32)
            _contig(t, n)
        _need(pos, "pos", I32)
        if cos.shape[-1] * 2 != rope_dim:
            raise ValueError(f"cos/sin must be [n_pos, {rope_dim // 2}]")
        n_pos = cos.shape[0]
    check(lib().dsa_head_norm_rope(x2.data_ptr(), x2.stride(0), o2.data_ptr(), o2.stride(0), B, n_heads, head_dim,
                                   rope_dim, _ptr(gamma), float(weight), int(norm), eps, _ptr(cos), _ptr(sin),
                                   n_pos, _ptr(pos), int(inverse), _ptr(status), _stream(x)), "head_norm_rope")
    return out


def fold_index_mask(idx: torch.Tensor, valid: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """-1 where the additive bf16 mask is negative, else idx (inverse of
    inference.py:4444-4457)."""
    _need(idx, "idx", I32)
    _need(valid, "valid", BF16)
    _contig(idx, "idx")
    _contig(valid, "valid")
    if valid.numel() != idx.numel():
        raise ValueError(f"valid has {valid.numel()} elements, idx {idx.numel()}")
    if out is None:
        out = torch.empty_like(idx)
    check(lib().dsa_fold_index_mask(idx.data_ptr(), valid.data_ptr(), idx.numel(), out.data_ptr(), _stream(idx)),
          "fold_index_mask")
    return out


# ------------------------------------------------------------ attn.compress

def compressor_step(kv_row, score_row, ape, kv_state, score_state, gamma, cos, sin, kv_cache, slot_offset: int,
                    pos, ratio: int, overlap: bool, rotate: bool = False, eps: float = 1e-6,
                    rope_dim: int = 64, emitted=None, write_state: bool = True) -> None:
    """One compressor decode step (state write + on-device emit decision,
    inference.py:4938-5097).  kv_row/score_row [B, coff*d] bf16; state fp32
    [B, coff*r, coff*d]; gamma [d] fp32; cos/sin [n_pos, rope/2] fp32;
    kv_cache [B, rows, d] bf16."""
    for t, n in ((kv_state, "kv_state"), (score_state, "score_state"), (gamma, "gamma"), (cos, "cos"),
                 (sin, "sin")):
        _need(t, n, F32)
        _contig(t, n)
    _need(kv_cache, "kv_cache", BF16)
    _need(pos, "pos", I32)
    B = kv_state.shape[0]
    d = gamma.shape[0]
    coff = 2 if overlap else 1
    if tuple(kv_state.shape) != (B, coff * ratio, coff * d) or kv_state.shape != score_state.shape:
        raise ValueError(f"state must be [B, {coff * ratio}, {coff * d}], got {tuple(kv_state.shape)}")
    if kv_cache.dim() != 3 or kv_cache.shape[2] != d or kv_cache.stride(1) != d:
        raise ValueError("kv_cache must be [B, rows, d] with contiguous rows")
    ld_row = 0
    if write_state:
        _need(kv_row, "kv_row", BF16)
        _need(score_row, "score_row", BF16)
        _need(ape, "ape", F32)
        _contig(ape, "ape")
        if kv_row.shape[-1] != coff * d or kv_row.stride(-1) != 1 or score_row.stride() != kv_row.stride():
            raise ValueError("kv_row/score_row must be [B, coff*d] with matching strides")
        ld_row = kv_row.stride(0)
    check(lib().dsa_compressor_step(_ptr(kv_row) if write_state else None, _ptr(score_row) if write_state else None,
                                    ld_row, _ptr(ape) if write_state else None, kv_state.data_ptr(),
                                    score_state.data_ptr(), gamma.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                    cos.shape[0], kv_cache.data_ptr(), kv_cache.stride(0), kv_cache.shape[1],
                                    slot_offset, pos.data_ptr(), _ptr(emitted), B, d, rope_dim, ratio,
                                    int(overlap), int(rotate), int(write_state), eps, _stream(kv_state)),
          "compressor_step")


def _cmp_args(kv_row, score_row, ape, kv_state, score_state, gamma, kv_cache, slot_offset: int, ratio: int,
              overlap: bool, rotate: bool, rope_dim: int) -> "_lib.CompressorArgs":
    for t, n in ((kv_state, "kv_state"), (score_state, "score_state"), (gamma, "gamma"), (ape, "ape")):
        _need(t, n, F32)
        _contig(t, n)
    _need(kv_row, "kv_row", BF16)
    _need(score_row, "score_row", BF16)
    _need(kv_cache, "kv_cache", BF16)
    B = kv_state.shape[0]
    d = gamma.shape[0]
    coff = 2 if overlap else 1
    if tuple(kv_state.shape) != (B, coff * ratio, coff * d) or kv_state.shape != score_state.shape:
        raise ValueError(f"state must be [B, {coff * ratio}, {coff * d}], got {tuple(kv_state.shape)}")
    if kv_cache.dim() != 3 or kv_cache.shape[2] != d or kv_cache.stride(1) != d:
        raise ValueError("kv_cache must be [B, rows, d] with contiguous rows")
    if kv_row.shape[-1] != coff * d or kv_row.stride(-1) != 1 or score_row.stride() != kv_row.stride():
        raise ValueError("kv_row/score_row must be [B, coff*d] with matching strides")
    return _lib.CompressorArgs(kv_row.data_ptr(), score_row.data_ptr(), kv_row.stride(0), ape.data_ptr(),
                               kv_state.data_ptr(), score_state.data_ptr(), gamma.data_ptr(), kv_cache.data_ptr(),
                               kv_cache.stride(0), kv_cache.shape[1], slot_offset, d, rope_dim, ratio, int(overlap),
                               int(rotate))


def layer_prologue(icmp: tuple, cmp: tuple, cos, sin, pos, t_active, iq, iw, score, T: int, kv, idx, win: int,
                   ratio: int, eps: float = 1e-6, rope_dim: int = 64, overlap: bool = True, rotate: bool = False,
                   kv_scales=None, beside_previous: bool = False) -> None:
    """A decode layer's small stages as one launch (dsa_layer_prologue):
    ``compressor_step(*icmp, slot_offset=0)`` then ``indexer_score_newest``
    on its cache, and ``kv_window_write(kv, cache)``, ``window_indices(pos,
    win, out=idx[:, :win])``, ``compressor_step(*cmp, slot_offset=win)`` on
    the attention cache.  icmp / cmp = (kv_row, score_row, ape, kv_state,
    score_state, gamma, kv_cache).  ``beside_previous``: run beside the
    previous kernel on the stream (DSA_BESIDE_PREVIOUS; see the header for
    the caller's guarantee)."""
    ia = _cmp_args(*icmp, 0, ratio, overlap, rotate, rope_dim)
    ca = _cmp_args(*cmp, win, ratio, overlap, rotate, rope_dim)
    for t, n in ((cos, "cos"), (sin, "sin")):
        _need(t, n, F32)
        _contig(t, n)
    _need(pos, "pos", I32)
    _need(t_active, "t_active", I32)
    _need(iq, "iq", BF16)
    _need(iw, "iw", F32)
    _need(score, "score", F32)
    _need(kv, "kv", BF16)
    _need(idx, "idx", I32)
    _contig(iq, "iq")
    _contig(iw, "iw")
    _contig(kv, "kv")
    B, D = kv.shape
    if iq.shape[1:] != (64, 128) or score.stride(1) != 1 or idx.stride(1) != 1:
        raise ValueError("layer_prologue: iq [B,64,128], score and idx rows contiguous")
    check(lib().dsa_layer_prologue(ctypes.byref(ia), ctypes.byref(ca), cos.data_ptr(), sin.data_ptr(), cos.shape[0],
                                   eps, pos.data_ptr(), t_active.data_ptr(), iq.data_ptr(), iw.data_ptr(),
                                   score.data_ptr(), score.stride(0), T, kv.data_ptr(), _ptr(kv_scales), D, rope_dim,
                                   win, idx.data_ptr(), idx.stride(0), B,
                                   _lib.DSA_BESIDE_PREVIOUS if beside_previous else 0, _stream(kv)),
          "layer_prologue")


# ---------------------------------------------------------------- attn.topk

def window_indices(pos: torch.Tensor, win: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Window ring indices per sequence (inference.py:479-506, 6020-6026)."""
    _need(pos, "pos", I32)
    B = pos.shape[0]
    if out is None:
        out = torch.empty(B, win, dtype=I32, device=pos.device)
    check(lib().dsa_window_indices(pos.data_ptr(), out.data_ptr(), out.stride(0), B, win, _stream(pos)),
          "window_indices")
    return out


def indexer_score(q: torch.Tensor, k_cache: torch.Tensor, w: torch.Tensor, T: int,
                  out: torch.Tensor | None = None, t_valid: torch.Tensor | None = None,
                  keys_ready: bool = False, counters: torch.Tensor | None = None) -> torch.Tensor:
    """``s[b,t] = sum_h w[b,h] relu(q[b,h].k[b,t])`` for t < T
    (inference.py:5260-5275).  q [B,64,128] bf16, k_cache [B, >=T, 128] bf16
    (or [>=T, 128]: one cache shared by all B rows, the queries of a prefill
    chunk), w [B,64] fp32 -> [B, T] fp32.  ``keys_ready``: k_cache and
    t_valid were complete before the previous kernel on the stream started
    (DSA_KEYS_READY: the kernel requests its first key tiles before waiting
    for that kernel).  ``counters`` (int32 [2], zero; left zero): split the
    work dynamically (dsa_indexer_score_dyn; one pair per stream that can
    run it concurrently)."""
    _need(q, "q", BF16)
    _need(k_cache, "k_cache", BF16)
    _need(w, "w", F32)
    _contig(q, "q")
    _contig(w, "w")
    B, H, Di = q.shape
    if k_cache.dim() == 2:
        if k_cache.shape[0] < T or k_cache.shape[1] != Di or k_cache.stride(0) != Di:
            raise ValueError("a shared k_cache must be [>=T, Di] with contiguous rows")
        k_bstride = 0
    else:
        if k_cache.shape[0] < B or k_cache.shape[1] < T or k_cache.shape[2] != Di or k_cache.stride(1) != Di:
            raise ValueError("k_cache must be [B, >=T, Di] with contiguous rows")
        k_bstride = k_cache.stride(0)
    if out is None:
        out = torch.empty(B, T, dtype=F32, device=q.device)
    if counters is not None:
        _need(counters, "counters", I32)
        if counters.numel() < 2:
            raise ValueError("counters must hold 2 int32")
        check(lib().dsa_indexer_score_dyn(q.data_ptr(), k_cache.data_ptr(), w.data_ptr(), out.data_ptr(),
                                          _ptr(t_valid), B, H, Di, T, k_bstride, out.stride(0),
                                          DSA_KEYS_READY if keys_ready else 0, counters.data_ptr(), _stream(q)),
              "indexer_score")
        return out
    check(lib().dsa_indexer_score_ex(q.data_ptr(), k_cache.data_ptr(), w.data_ptr(), out.data_ptr(),
                                     _ptr(t_valid), B, H, Di, T, k_bstride, out.stride(0),
                                     DSA_KEYS_READY if keys_ready else 0, _stream(q)), "indexer_score")
    return out


def indexer_score_newest(q: torch.Tensor, k_cache: torch.Tensor, w: torch.Tensor, t_active: torch.Tensor, T: int,
                         out: torch.Tensor) -> torch.Tensor:
    """The score of each sequence's newest live row, t = min(t_active, T) - 1,
    written into ``out[b, t]`` (inference.py:5260-5275 for one row; the value
    the top-k's ``refresh`` recomputes).  q [B,64,128] bf16, k_cache
    [B, >=T, 128] bf16 rows contiguous, w [B,64] fp32, out [B, >=T] fp32."""
    _need(q, "q", BF16)
    _need(k_cache, "k_cache", BF16)
    _need(w, "w", F32)
    _need(t_active, "t_active", I32)
    _need(out, "out", F32)
    _contig(q, "q")
    _contig(w, "w")
    B = q.shape[0]
    if q.shape[1:] != (64, 128) or k_cache.dim() != 3 or k_cache.shape[0] < B or k_cache.shape[1] < T \
            or k_cache.shape[2] != 128 or k_cache.stride(1) != 128 or out.shape[0] < B or out.stride(1) != 1:
        raise ValueError("indexer_score_newest: q [B,64,128], k_cache [B,>=T,128] rows contiguous, out [B,>=T]")
    check(lib().dsa_indexer_score_newest(q.data_ptr(), k_cache.data_ptr(), k_cache.stride(0), w.data_ptr(),
                                         t_active.data_ptr(), out.data_ptr(), out.stride(0), B, T, _stream(q)),
          "indexer_score_newest")
    return out


def indexer_topk(score: torch.Tensor, t_active: torch.Tensor, k: int, win: int, T: int | None = None,
                 sort_desc: bool = False, mask_mode: int = 0, out: torch.Tensor | None = None,
                 out_score: torch.Tensor | None = None, ws: Workspace | None = None,
                 refresh: tuple | None = None) -> torch.Tensor:
    """Masked top-k (inference.py:5823-5851) -> int32 [B, k] (idx + win, -1
    for invalid).  ``refresh=(q [B,64,128] bf16, k_cache [B,T',128] bf16,
    w [B,64] f32)``: the score of each row's newest live entry (t_active - 1)
    is recomputed from the indexer inputs instead of read from ``score``, so
    the score matrix may be computed before that key row is written."""
    _need(score, "score", F32)
    _need(t_active, "t_active", I32)
    B = score.shape[0]
    T = score.shape[1] if T is None else T
    if out is None:
        out = torch.empty(B, k, dtype=I32, device=score.device)
    L = lib()
    need = L.dsa_indexer_topk_workspace_size(B, T, k)
    if refresh is not None:
        q, kc, w = refresh
        _need(q, "q", BF16)
        _need(kc, "k_cache", BF16)
        _need(w, "w", F32)
        if q.shape[-2:] != (64, 128) or kc.shape[-1] != 128 or kc.stride(1) != 128 or not q.is_contiguous() \
                or not w.is_contiguous():
            raise ValueError("indexer_topk refresh: q [B,64,128], k_cache [B,T,128] rows contiguous, w [B,64]")
        wsb = _ws(score.device, need, ws) if need else None
        rc = L.dsa_indexer_topk_newest(score.data_ptr(), score.stride(0), t_active.data_ptr(), out.data_ptr(),
                                       _ptr(out_score), out.stride(0), B, T, k, win, int(sort_desc), mask_mode,
                                       q.data_ptr(), kc.data_ptr(), kc.stride(0), w.data_ptr(),
                                       wsb.buf.data_ptr() if wsb else None, wsb.nbytes if wsb else 0, _stream(score))
        check(rc, "indexer_topk_newest")
        return out
    if need:
        w = _ws(score.device, need, ws)
        rc = L.dsa_indexer_topk_ws(score.data_ptr(), score.stride(0), t_active.data_ptr(), out.data_ptr(),
                                   _ptr(out_score), out.stride(0), B, T, k, win, int(sort_desc), mask_mode,
                                   w.buf.data_ptr(), w.nbytes, _stream(score))
    else:
        rc = L.dsa_indexer_topk(score.data_ptr(), score.stride(0), t_active.data_ptr(), out.data_ptr(),
                                _ptr(out_score), out.stride(0), B, T, k, win, int(sort_desc), mask_mode,
                                _stream(score))
    check(rc, "indexer_topk")
    return out


class WideTopkWorkspace:
    """Zero-initialised, grow-only workspace of dsa_topk_wide (the kernel
    leaves it zeroed after every call)."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.buf = torch.zeros(64, dtype=torch.uint8, device=self.device)

    def get(self, B: int, T: int) -> torch.Tensor:
        need = int(lib().dsa_topk_wide_workspace_size(B, T))
        if need > self.buf.numel():
            self.buf = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self.buf


def topk_wide(score: torch.Tensor, k: int, win: int, t_active: torch.Tensor | None = None, T: int | None = None,
              ids: torch.Tensor | None = None, mask_mode: int = 1, out: torch.Tensor | None = None,
              out_score: torch.Tensor | None = None, ws: WideTopkWorkspace | None = None,
              status: torch.Tensor | None = None, seg_len: int = 0, seg_stride: int = 0,
              B: int | None = None, ld_score: int | None = None) -> torch.Tensor:
    """Multi-CTA top-k of a few long rows (see dsa_topk_wide); output in
    ascending position order.  With ``seg_len`` the T elements of a row are
    read as T / seg_len pieces ``seg_stride`` elements apart (the rank-major
    result of an all-gather); B / ld_score then describe the rows."""
    _need(score, "score", F32)
    B = score.shape[0] if B is None else B
    T = score.shape[1] if T is None else T
    if score.stride(-1) != 1:
        raise ValueError("score must have a unit stride in the last dim")
    ld_ids = 0
    if ids is not None:
        _need(ids, "ids", I32)
        if ids.stride(-1) != 1:
            raise ValueError("ids must have a unit stride in the last dim")
        ld_ids = ids.stride(0)
    if t_active is not None:
        _need(t_active, "t_active", I32)
    if out is None:
        out = torch.empty(B, k, dtype=I32, device=score.device)
    if out_score is not None and out_score.stride(0) != out.stride(0):
        raise ValueError("out and out_score must share the row stride")
    if ws is None:
        ws = _wide_ws.setdefault(score.device, WideTopkWorkspace(score.device))
    buf = ws.get(B, T)
    lds = score.stride(0) if ld_score is None else ld_score
    if ids is not None and ld_score is not None:
        ld_ids = ld_score
    check(lib().dsa_topk_wide(score.data_ptr(), lds, _ptr(ids), ld_ids, _ptr(t_active), out.data_ptr(),
                              _ptr(out_score), out.stride(0), B, T, k, win, mask_mode, seg_len, seg_stride,
                              buf.data_ptr(), buf.numel(), _ptr(status), _stream(score)), "topk_wide")
    return out


_wide_ws: dict = {}


def topk_merge(cand_score: torch.Tensor, cand_idx: torch.Tensor, k: int, win: int,
               out: torch.Tensor | None = None, out_score: torch.Tensor | None = None) -> torch.Tensor:
    """Global top-k from concatenated per-shard candidate lists."""
    _need(cand_score, "cand_score", F32)
    _need(cand_idx, "cand_idx", I32)
    _contig(cand_score, "cand_score")
    _contig(cand_idx, "cand_idx")
    B, n = cand_score.shape
    if out is None:
        out = torch.empty(B, k, dtype=I32, device=cand_score.device)
    check(lib().dsa_topk_merge(cand_score.data_ptr(), cand_idx.data_ptr(), n, out.data_ptr(), _ptr(out_score),
                               out.stride(0), B, k, win, _stream(cand_score)), "topk_merge")
    return out


def prefill_positions(S: int, base: int, T: int, W: int, n_hist: int, ratio: int, t_active: torch.Tensor,
                      idx: torch.Tensor) -> None:
    """Per-token t_active and causal-window columns idx[:, :W] of a prefill
    chunk (see dsa_prefill_positions)."""
    _need(t_active, "t_active", I32)
    _need(idx, "idx", I32)
    if idx.stride(-1) != 1 or idx.shape[0] < S:
        raise ValueError("idx must be [>=S, >=W] with a unit last stride")
    check(lib().dsa_prefill_positions(S, base, ratio, T, W, n_hist, t_active.data_ptr(), idx.data_ptr(),
                                      idx.stride(0), _stream(idx)), "prefill_positions")


def shard_active(t_active: torch.Tensor, lo: int, n_local: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """This shard's share of T_active: clamp(t_active - lo, 0, n_local)."""
    _need(t_active, "t_active", I32)
    if out is None:
        out = torch.empty_like(t_active)
    check(lib().dsa_shard_active(t_active.data_ptr(), out.data_ptr(), t_active.numel(), lo, n_local,
                                 _stream(t_active)), "shard_active")
    return out


def shard_local_indices(sel: torch.Tensor, lo: int, hi: int, W: int, win_idx: torch.Tensor | None = None,
                        local_base: int = 0, win_base: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """[B, W + k] local attention rows of a shard from the merged global
    selection ``sel`` [B, k] (see dsa_shard_local_indices)."""
    _need(sel, "sel", I32)
    B, k = sel.shape
    if sel.stride(-1) != 1:
        raise ValueError("sel must have a unit stride in the last dim")
    ld_win = 0
    if win_idx is not None:
        _need(win_idx, "win_idx", I32)
        if win_idx.shape[-1] != W or win_idx.stride(-1) != 1:
            raise ValueError(f"win_idx must be [B, {W}] with a unit last stride")
        ld_win = win_idx.stride(0)
    if out is None:
        out = torch.empty(B, W + k, dtype=I32, device=sel.device)
    check(lib().dsa_shard_local_indices(sel.data_ptr(), sel.stride(0), k, _ptr(win_idx), ld_win, W, lo, hi,
                                        local_base, win_base, out.data_ptr(), out.stride(0), B, _stream(sel)),
          "shard_local_indices")
    return out


def advance_positions(pos: torch.Tensor, t_active: torch.Tensor | None, ratio: int, step: int = 1) -> None:
    _need(pos, "pos", I32)
    check(lib().dsa_advance_positions(pos.data_ptr(), _ptr(t_active), pos.shape[0], ratio, step, _stream(pos)),
          "advance_positions")


# -------------------------------------------------------------- attn.sparse

def _attn_shapes(q, kv, idx):
    _need(q, "q", BF16)
    _need(kv, "kv", BF16)
    _need(idx, "idx", I32)
    _contig(q, "q")
    H, D = q.shape[-2], q.shape[-1]
    if q.dim() == 4:
        B, S = q.shape[0], q.shape[1]
    elif q.dim() == 3:
        B, S = q.shape[0], 1
    else:
        raise ValueError("q must be [B, S, H, D] or [B, H, D]")
    if kv.dim() == 2:
        kv = kv.unsqueeze(0)
    if kv.shape[0] not in (1, B) or kv.shape[2] != D or kv.stride(1) != D:
        raise ValueError("kv must be [N, D] or [B, N, D] with contiguous rows")
    kv_bstride = 0 if kv.shape[0] == 1 else kv.stride(0)
    if kv_bstride == 0:
        kv_bstride = kv.shape[1] * D  # checked >= rows * D; batch 0 for all rows
    K = idx.shape[-1]
    idx2 = idx.reshape(B * S, K)
    if idx2.stride(-1) != 1:
        raise ValueError("idx must have a unit stride in the last dim")
    return B, S, H, D, K, kv, kv_bstride, idx2


LEAD_READY = 1


def sparse_attn(q, kv, idx, sink, scale: float, out=None, lse=None, ws: Workspace | None = None,
                status=None, lead_cols: int = 0, lead_ready: bool = False) -> torch.Tensor:
    """Sink-softmax sparse attention (inference.py:4459-4501).  q [B,S,H,D] or
    [B,H,D] bf16; kv [B,N,D] or [N,D] bf16; idx [B,S,K] / [B,K] int32 with -1
    = masked; sink [H] fp32.  ``lead_cols``/``lead_ready``: the first
    lead_cols index columns (the window slots), q and the kv rows they name
    are not written by the previous kernel on the stream and were complete
    before this launch (dsa_sparse_attn_ex with DSA_LEAD_READY): they are
    requested before the kernel waits for that one."""
    B, S, H, D, K, kv3, kv_bstride, idx2 = _attn_shapes(q, kv, idx)
    if kv3.shape[0] == 1 and B > 1:
        raise ValueError("a shared [N, D] kv needs B == 1; pass [B, N, D]")
    _need(sink, "sink", F32)
    if out is None:
        out = torch.empty_like(q)
    L = lib()
    need = L.dsa_sparse_attn_workspace_size(B, S, H, D, K)
    w = _ws(q.device, need, ws) if need else None
    if lead_ready and lead_cols > 0:
        check(L.dsa_sparse_attn_ex(q.data_ptr(), kv3.data_ptr(), kv_bstride, kv3.shape[1], idx2.data_ptr(),
                                   idx2.stride(0), sink.data_ptr(), out.data_ptr(), _ptr(lse), B, S, H, D, K, scale,
                                   w.buf.data_ptr() if w else None, w.nbytes if w else 0, lead_cols, LEAD_READY,
                                   _ptr(status), _stream(q)), "sparse_attn")
        return out
    check(L.dsa_sparse_attn(q.data_ptr(), kv3.data_ptr(), kv_bstride, kv3.shape[1], idx2.data_ptr(),
                            idx2.stride(0), sink.data_ptr(), out.data_ptr(), _ptr(lse), B, S, H, D, K, scale,
                            w.buf.data_ptr() if w else None, w.nbytes if w else 0, _ptr(status), _stream(q)),
          "sparse_attn")
    return out


def sparse_attn_partial(q, kv, idx, scale: float, part_ml=None, part_o=None, ws: Workspace | None = None,
                        status=None):
    """Un-normalised partial (m, l, o) over the rows of ``idx`` (no sink)."""
    B, S, H, D, K, kv3, kv_bstride, idx2 = _attn_shapes(q, kv, idx)
    M = B * S
    if part_ml is None:
        part_ml = torch.empty(M, H, 2, dtype=F32, device=q.device)
    if part_o is None:
        part_o = torch.empty(M, H, D, dtype=F32, device=q.device)
    L = lib()
    need = L.dsa_sparse_attn_workspace_size(B, S, H, D, K)
    w = _ws(q.device, need, ws) if need else None
    check(L.dsa_sparse_attn_partial(q.data_ptr(), kv3.data_ptr(), kv_bstride, kv3.shape[1], idx2.data_ptr(),
                                    idx2.stride(0), part_ml.data_ptr(), part_o.data_ptr(), B, S, H, D, K, scale,
                                    w.buf.data_ptr() if w else None, w.nbytes if w else 0, _ptr(status),
                                    _stream(q)), "sparse_attn_partial")
    return part_ml, part_o


def lse_combine_strided(part_ml: torch.Tensor, ml_pstride: int, part_o: torch.Tensor, o_pstride: int, P: int,
                        M: int, H: int, D: int, sink: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """lse_combine over P partials ``ml_pstride`` / ``o_pstride`` floats apart
    (rank-major all-gather output); out bf16 [M, H, D]."""
    _need(part_ml, "part_ml", F32)
    _need(part_o, "part_o", F32)
    _need(sink, "sink", F32)
    _need(out, "out", BF16)
    check(lib().dsa_lse_combine_strided(part_ml.data_ptr(), ml_pstride, part_o.data_ptr(), o_pstride,
                                        sink.data_ptr(), out.data_ptr(), P, M, H, D, _stream(part_o)),
          "lse_combine_strided")
    return out


def lse_combine(part_ml, part_o, sink, out=None) -> torch.Tensor:
    """Merge P partials [P, M, H, 2] / [P, M, H, D] with the sink once -> bf16 [M, H, D]."""
    _need(part_ml, "part_ml", F32)
    _need(part_o, "part_o", F32)
    _need(sink, "sink", F32)
    _contig(part_ml, "part_ml")
    _contig(part_o, "part_o")
    Pn, M, H, D = part_o.shape
    if out is None:
        out = torch.empty(M, H, D, dtype=BF16, device=part_o.device)
    check(lib().dsa_lse_combine(part_ml.data_ptr(), part_o.data_ptr(), sink.data_ptr(), out.data_ptr(), Pn, M, H, D,
                                _stream(part_o)), "lse_combine")
    return out
