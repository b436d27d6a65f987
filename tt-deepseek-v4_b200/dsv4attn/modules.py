"""Drop-ins for the reference's device attention modules, same call signatures.

Each class keeps the constructor, method names, argument meaning and error
behaviour of its counterpart in zoecarver/tt-deepseek-v4 ``inference.py``
so a caller switches by changing the import:

=====================  ==============================  =====================
reference              here                            native entry points
=====================  ==============================  =====================
DeviceSparseAttn       DeviceSparseAttn   (4336-4501)  dsa_sparse_attn,
                                                       dsa_fold_index_mask
DeviceCompressor       DeviceCompressor   (4634-5097)  dsa_compressor_step
DeviceIndexer          DeviceIndexer      (5100-5275)  dsa_head_norm_rope,
                                                       dsa_indexer_score
DeviceAttention        DeviceAttention    (5278-6127)  all of the above plus
                                                       dsa_kv_norm_rope_window_write,
                                                       dsa_window_indices,
                                                       dsa_indexer_topk
=====================  ==============================  =====================

``mesh`` (a ttnn mesh in the reference) is a torch device here - a
``torch.device``, a device string / index, or any object with a ``.device``
attribute.  Device tensors (``*_tt`` in the reference) are CUDA torch
tensors.  The per-step integers are staged by ``pre_stage_decode`` into
device buffers; the ``forward_device`` bodies allocate nothing and make no
host transfer except the outputs they return, so they can be captured in a
CUDA graph (the reference's trace capture, inference.py:7498-7543).

The weight projections around the path (wq_a, wq_b, wkv, the compressor's
wkv/wgate, weights_proj, wo_a, wo_b) are plain GEMMs and run through
``DeviceLinear`` (the library's weight-streaming tcgen05 kernel,
``dsa_linear``); everything between them is the native library too.  Errors follow the reference: ``ValueError`` for shapes,
``RuntimeError`` for unallocated state (inference.py:4394-4397, 4949-4952).
"""

from __future__ import annotations

import torch

from . import ops
from .tables import pick_indexer_topk_bucket

BF16 = torch.bfloat16
F32 = torch.float32
I32 = torch.int32

FP8_WEIGHT_BLOCK = 128  # block_size of the reference's fp8 weights (inference.py:178)


def _device_of(mesh) -> torch.device:
    dev = getattr(mesh, "device", mesh)
    dev = torch.device(dev) if not isinstance(dev, torch.device) else dev
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise ValueError(f"device modules need a CUDA device, got {dev} (there is no CPU fallback)")
    return dev


def weight_bf16(w) -> torch.Tensor:
    """bf16 copy of a Linear weight [out, in]: a tensor, or a module with
    ``.weight`` (fp8 e4m3 weights carry a per-128x128-block ``scale``,
    inference.py:399-433, and are expanded block by block)."""
    t = getattr(w, "weight", w)
    if not isinstance(t, torch.Tensor):
        raise ValueError("weight must be a tensor or have a .weight tensor")
    t = t.detach()
    if t.dtype == torch.float8_e4m3fn:
        scale = getattr(t, "scale", None)
        if scale is None:
            scale = getattr(w, "scale", None)
        if scale is None:
            raise ValueError("fp8 weight without a block scale")
        n, k = t.shape
        s = scale.detach().float()
        s = s.repeat_interleave(FP8_WEIGHT_BLOCK, 0).repeat_interleave(FP8_WEIGHT_BLOCK, 1)[:n, :k]
        return (t.float() * s).to(BF16)
    if t.dtype in (torch.float32, torch.bfloat16, torch.float16):
        return t.to(BF16)
    raise ValueError(f"unsupported weight dtype {t.dtype} for the attention projections")


def _gamma_of(norm, fallback=None) -> torch.Tensor:
    for name in ("_cpu_gamma", "gamma", "weight"):
        g = getattr(norm, name, None) if norm is not None else None
        if isinstance(g, torch.Tensor):
            return g.detach().float().reshape(-1)
    if fallback is not None:
        return _gamma_of(fallback)
    raise ValueError("norm module has no gamma / weight")


def _eps_of(norm, default: float) -> float:
    e = getattr(norm, "eps", None) if norm is not None else None
    return float(e) if e is not None else float(default)


def _freqs_tables(freqs_cis: torch.Tensor, device):
    """(cos, sin) fp32 [seq, rope/2] from the reference's complex freqs_cis
    (inference.py:452-476)."""
    if torch.is_complex(freqs_cis):
        c, s = freqs_cis.real, freqs_cis.imag
    else:
        c, s = torch.cos(freqs_cis), torch.sin(freqs_cis)
    return c.float().contiguous().to(device), s.float().contiguous().to(device)


class DeviceLinear:
    """``y = x @ W^T`` on the device: the weight-streaming tcgen05 kernel of
    ``dsa_linear`` (bf16 result; ``out_dtype=F32`` gives the fp32 value of
    it).  Replaces the reference's DeviceColLinear matmuls
    (inference.py:4954-4966, 5934-5960, 6126).

    ``fused(device, [w_a, w_b])`` concatenates weights along the output dim
    and records ``_fused_*_out`` widths like the reference's fused
    DeviceColLinear (inference.py:4954-4966, 5941-5953)."""

    def __init__(self, device, weight, scale: float = 1.0, out_dtype=BF16):
        self.device = _device_of(device)
        w = weight_bf16(weight)
        if scale != 1.0:
            w = (w.float() * scale).to(BF16)
        self.out_dim, self.in_dim = w.shape
        # stored once in the tile layout the projection kernel streams
        self.weight = ops.pack_linear_weight(w.to(self.device).contiguous())
        self.out_dtype = out_dtype

    @classmethod
    def fused(cls, device, weights, names=("kv", "gate")):
        ws = [weight_bf16(w) for w in weights]
        lin = cls(device, torch.cat(ws, 0))
        for n, w in zip(names, ws):
            setattr(lin, f"_fused_{n}_out", w.shape[0])
        return lin

    def forward_device(self, x: torch.Tensor, rope: tuple | None = None, status=None) -> torch.Tensor:
        """``rope=(cos, sin, pos, head_dim, rope_dim)`` rotates the last
        rope_dim columns of every head_dim block of the result (the
        reference's Lk-D-idx-q fusion of wq_b and the q rotary)."""
        if x.shape[-1] != self.in_dim:
            raise ValueError(f"input dim {x.shape[-1]} != weight in_dim {self.in_dim}")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_dim).to(BF16).contiguous()
        y = ops.linear(x2, self.weight, out_f32=self.out_dtype != BF16, rope=rope, status=status)
        return y.reshape(*lead, self.out_dim)

    __call__ = forward_device


# --------------------------------------------------------------------------
# attn.sparse
# --------------------------------------------------------------------------

class DeviceSparseAttn(torch.nn.Module):
    """Sink-concat softmax sparse attention (inference.py:4336-4501).

    ``forward(q, kv, topk_idxs)`` is the host-facing drop-in for
    ``sparse_attn(q, kv, attn_sink, topk_idxs, softmax_scale)``: any device,
    result on q's device and dtype.  Unlike the reference it accepts B > 1
    (kv then [B, N, D]).  ``forward_device`` takes q with the softmax scale
    already folded in (the reference pre-bakes it through q_rsqrt_ones,
    inference.py:4476-4477, 5348-5350)."""

    def __init__(self, mesh, attn_sink: torch.Tensor, softmax_scale: float):
        super().__init__()
        self.device = _device_of(mesh)
        self.softmax_scale = float(softmax_scale)
        self.n_heads_full = int(attn_sink.shape[0])
        self.n_heads = self.n_heads_full
        self.sink = attn_sink.detach().float().reshape(-1).contiguous().to(self.device)
        self._alloc_decode_tensors()

    def _alloc_decode_tensors(self):
        """Split-K workspace and the bounded-wait status word.  The workspace
        grows on first use of a larger shape; call forward_device once at
        the largest shape before capturing a graph."""
        self.ws = ops.Workspace(self.device)
        self.status = torch.zeros(1, dtype=I32, device=self.device)

    def forward(self, q: torch.Tensor, kv: torch.Tensor, topk_idxs: torch.Tensor) -> torch.Tensor:
        B, S, H, D = q.shape
        if H != self.n_heads:
            raise ValueError(f"q heads {H} != attn_sink heads {self.n_heads}")
        if topk_idxs.dim() != 3 or tuple(topk_idxs.shape[:2]) != (B, S):
            raise ValueError(f"topk_idxs must be [B, S, K] = [{B}, {S}, K], got {tuple(topk_idxs.shape)}")
        dev = self.device
        q_d = q.to(dev, BF16).contiguous()
        kv_d = kv.to(dev, BF16)
        if kv_d.dim() == 3 and kv_d.shape[0] == 1 and B == 1:
            kv_d = kv_d[0]
        kv_d = kv_d.contiguous()
        idx = topk_idxs.to(dev, I32).contiguous()
        out = ops.sparse_attn(q_d, kv_d, idx, self.sink, self.softmax_scale, ws=self.ws, status=self.status)
        return out.to(q.device, q.dtype)

    def _idxs_int_tile_to_idxs_and_mask(self, idxs_int_tt: torch.Tensor, B: int, S: int, K: int):
        """(indices [B, S*K] int32, mask) for forward_device.  The kernel
        skips -1 sentinels itself, so the indices keep them and the mask is
        None: no [B, S, 1, K] additive tensor is materialised
        (inference.py:4444-4457 builds one)."""
        if idxs_int_tt.numel() != B * S * K:
            raise ValueError(f"index tensor has {idxs_int_tt.numel()} elements, expected {B}*{S}*{K}")
        if idxs_int_tt.dtype != I32:
            raise ValueError("indices must be int32")
        return idxs_int_tt.reshape(B, S * K), None

    def forward_device(self, q_tt, kv_tt, idxs_tt, valid_tt, S: int, K: int, out=None):
        """q_tt [B, S, H, D] bf16 (pre-scaled); kv_tt [N, D] (B == 1) or
        [B, N, D]; idxs_tt [B, S*K] int32; valid_tt None (sentinels in the
        indices) or the reference's additive bf16 {0, -inf} mask [B, S, 1, K]
        over clamped indices.  Returns o [B, S, H, D] bf16."""
        B, Sq, H, D = q_tt.shape
        if Sq != S:
            raise ValueError(f"q has S={Sq}, argument S={S}")
        if H != self.n_heads:
            raise ValueError(f"q heads {H} != attn_sink heads {self.n_heads}")
        if idxs_tt.numel() != B * S * K:
            raise ValueError(f"indices have {idxs_tt.numel()} elements, expected {B}*{S}*{K}")
        idx = idxs_tt.reshape(B, S, K)
        if valid_tt is not None:
            idx = ops.fold_index_mask(idx.contiguous(), valid_tt.reshape(B, S, K).contiguous())
        if kv_tt.dim() == 2 and B != 1:
            raise ValueError("a flat [N, D] kv needs B == 1; pass [B, N, D]")
        return ops.sparse_attn(q_tt, kv_tt, idx, self.sink, 1.0, out=out, ws=self.ws, status=self.status)


# --------------------------------------------------------------------------
# attn.compress
# --------------------------------------------------------------------------

class DeviceCompressor(torch.nn.Module):
    """Decode-only compressor (inference.py:4634-5097): state write, emit on
    ``(pos + 1) % ratio == 0`` (softmax over slots, weighted sum, RMSNorm,
    rotary, cache write) and the overlap slot shift, all in one launch.

    ``comp`` is the CPU Compressor (inference.py:523-552): head_dim,
    rope_head_dim, compress_ratio, overlap, rotate, ape, kv_state,
    score_state, kv_cache, freqs_cis, norm.  The state stays fp32 (the CPU
    layout); the reference's device copy is bf16.  As on the reference's
    device path the Walsh-Hadamard rotation of the indexer compressor is
    skipped: it cancels against the q-side rotation in the score
    (inference.py:5066-5070, 5239-5241); ``apply_hadamard=True`` keeps it."""

    def __init__(self, mesh, comp, wkv_dev, wgate_dev, norm_dev, slot_offset: int = 0, kv_cache_tt=None,
                 apply_hadamard: bool = False):
        super().__init__()
        self.device = _device_of(mesh)
        self.comp = comp
        self.wkv = wkv_dev
        self.wgate = wgate_dev
        self.norm_dev = norm_dev
        self.head_dim = int(comp.head_dim)
        self.rope_head_dim = int(comp.rope_head_dim)
        self.compress_ratio = int(comp.compress_ratio)
        self.overlap = bool(comp.overlap)
        self.rotate = bool(comp.rotate) and apply_hadamard
        self.coff = 2 if self.overlap else 1
        self.cdim = self.coff * self.head_dim
        self.row_count = 2 * self.compress_ratio if self.overlap else self.compress_ratio
        self.slot_offset = int(slot_offset)
        norm = getattr(comp, "norm", None)
        self.gamma = _gamma_of(norm_dev, norm).to(self.device).contiguous()
        self.eps = _eps_of(norm_dev, _eps_of(norm, 1e-6))
        self.ape = comp.ape.detach().float().contiguous().to(self.device)
        self.cos, self.sin = _freqs_tables(comp.freqs_cis, self.device)
        self.kv_state = None
        self.score_state = None
        self.kv_cache_tt = kv_cache_tt
        self._owns_kv_cache = kv_cache_tt is None
        self._start_pos = None

    def bind_kv_cache_tt(self, kv_cache_tt, slot_offset: int):
        """Write compressed rows into an existing cache (the attention's
        joint window+compressed buffer) at slot_offset + pos // ratio
        (inference.py:4748-4755)."""
        self.kv_cache_tt = kv_cache_tt
        self.slot_offset = int(slot_offset)
        self._owns_kv_cache = False

    def _alloc_decode_tensors(self, B: int = 1):
        """Device state from the CPU module's current state
        (inference.py:4757-4906); idempotent."""
        dev = self.device
        comp = self.comp
        self.kv_state = comp.kv_state[:B].detach().float().contiguous().to(dev)
        self.score_state = comp.score_state[:B].detach().float().contiguous().to(dev)
        if self._owns_kv_cache:
            kc = getattr(comp, "kv_cache", None)
            if kc is None:
                raise RuntimeError("DeviceCompressor owns its kv_cache but comp.kv_cache is None; "
                                   "set it or call bind_kv_cache_tt first")
            self.kv_cache_tt = kc[:B].detach().to(BF16).contiguous().to(dev)
        self._pos_tt = torch.zeros(B, dtype=I32, device=dev)
        self._emitted = torch.zeros(B, dtype=I32, device=dev)
        self.B = B

    def pre_stage_decode(self, start_pos: int, B: int = 1):
        """Stage this step's position on the device (inference.py:4907-4936)."""
        if self.kv_state is None or self.kv_state.shape[0] != B:
            self._alloc_decode_tensors(B)
        self._start_pos = int(start_pos)
        if getattr(self, "_slots_shared", False):
            return
        self._pos_tt.fill_(int(start_pos))

    def _pos_for(self, start_pos_tt, B):
        if (isinstance(start_pos_tt, torch.Tensor) and start_pos_tt.is_cuda and start_pos_tt.dtype == I32
                and start_pos_tt.numel() == B and start_pos_tt.is_contiguous()):
            return start_pos_tt.reshape(B)
        return self._pos_tt

    def _emitted_row(self, B: int, start_pos: int):
        if (start_pos + 1) % self.compress_ratio != 0:
            return None
        row = self.slot_offset + start_pos // self.compress_ratio
        return self.kv_cache_tt[:B, row].unsqueeze(1)

    def forward_device(self, x_tt, B: int, start_pos: int, start_pos_tt):
        """State write (+ emit on emit positions).  Returns the emitted row
        [B, 1, d] (a view of the cache) or None (inference.py:4938-4995)."""
        if start_pos_tt is None:
            raise ValueError("DeviceCompressor.forward_device requires start_pos_tt "
                             "(no host->device upload inside the trace body).")
        if self.kv_state is None:
            raise RuntimeError("DeviceCompressor decode buffers not allocated; "
                               "call pre_stage_decode at least once before forward_device.")
        if self.wkv is self.wgate:
            fused = self.wkv.forward_device(x_tt).reshape(B, -1)
            kv_out, gate_out = self.wkv._fused_kv_out, self.wkv._fused_gate_out
            kv = fused[:, :kv_out]
            score = fused[:, kv_out:kv_out + gate_out]
        else:
            kv = self.wkv.forward_device(x_tt).reshape(B, -1)
            score = self.wgate.forward_device(x_tt).reshape(B, -1)
        return self.step_rows(kv, score, B, start_pos, start_pos_tt)

    def step_rows(self, kv_row, score_row, B: int, start_pos: int, start_pos_tt=None):
        """forward_device after the wkv / wgate projections: kv_row and
        score_row [B, coff*d] (bf16)."""
        if self.kv_state is None:
            raise RuntimeError("DeviceCompressor decode buffers not allocated; "
                               "call pre_stage_decode at least once before forward_device.")
        kv_row = kv_row.to(BF16)
        score_row = score_row.to(BF16)
        if kv_row.stride() != score_row.stride():
            kv_row, score_row = kv_row.contiguous(), score_row.contiguous()
        ops.compressor_step(kv_row, score_row, self.ape, self.kv_state, self.score_state, self.gamma, self.cos,
                            self.sin, self.kv_cache_tt, self.slot_offset, self._pos_for(start_pos_tt, B),
                            self.compress_ratio, self.overlap, rotate=self.rotate, eps=self.eps,
                            rope_dim=self.rope_head_dim, emitted=self._emitted)
        return self._emitted_row(B, start_pos)

    def _emit_body(self, B: int, d: int, rd: int, start_pos_tt):
        """Emit only (no state write), at the staged position: cssn + rotary
        + cache write + slot shift (inference.py:4997-5097)."""
        if self.kv_state is None:
            raise RuntimeError("DeviceCompressor decode buffers not allocated; "
                               "call pre_stage_decode at least once before forward_device.")
        if d != self.head_dim or rd != self.rope_head_dim:
            raise ValueError(f"no compressor emit built for d={d}, rd={rd} on this module "
                             f"(head_dim {self.head_dim}, rope {self.rope_head_dim})")
        ops.compressor_step(None, None, None, self.kv_state, self.score_state, self.gamma, self.cos, self.sin,
                            self.kv_cache_tt, self.slot_offset, self._pos_for(start_pos_tt, B),
                            self.compress_ratio, self.overlap, rotate=self.rotate, eps=self.eps, rope_dim=rd,
                            emitted=self._emitted, write_state=False)
        sp = self._start_pos
        if sp is None:
            return None
        row = self.slot_offset + sp // self.compress_ratio
        return self.kv_cache_tt[:B, row].unsqueeze(1)


# --------------------------------------------------------------------------
# attn.topk: indexer
# --------------------------------------------------------------------------

class DeviceIndexer(torch.nn.Module):
    """Indexer scoring (inference.py:5100-5275): q = rotary(qr @ wq_b^T),
    the inner compressor step, w = x @ weights_proj^T * softmax_scale *
    n_heads^-1/2 (folded into the weight, inference.py:5175-5185), and
    ``score[b, t] = sum_h w[b, h] relu(q[b, h] . k[b, t])``.

    ``indexer`` is the CPU Indexer (inference.py:554-574): head_dim,
    rope_head_dim, n_heads, compress_ratio, softmax_scale, index_topk,
    freqs_cis, wq_b, weights_proj.  ``wq_b_dev`` / ``weights_proj_dev`` may
    be None (built from the CPU module) or DeviceLinear-like objects; a
    weights_proj_dev passed in must already carry the scale fold."""

    def __init__(self, mesh, indexer, dc: DeviceCompressor, wq_b_dev=None, weights_proj_dev=None):
        super().__init__()
        self.device = _device_of(mesh)
        self.indexer = indexer
        self.dc = dc
        self.head_dim = int(indexer.head_dim)
        self.rope_head_dim = int(indexer.rope_head_dim)
        self.n_heads = int(indexer.n_heads)
        self.n_local_heads = self.n_heads
        self.compress_ratio = int(indexer.compress_ratio)
        self.softmax_scale = float(indexer.softmax_scale)
        self.index_topk = int(indexer.index_topk)
        if wq_b_dev is None:
            wq_b_dev = DeviceLinear(self.device, indexer.wq_b)
        if weights_proj_dev is None:
            scale = self.softmax_scale * self.n_heads ** -0.5
            weights_proj_dev = DeviceLinear(self.device, indexer.weights_proj, scale=scale, out_dtype=F32)
        self.wq_b = wq_b_dev
        self.weights_proj = weights_proj_dev
        self.q_lora_rank = getattr(wq_b_dev, "in_dim", None)
        self.dim = getattr(weights_proj_dev, "in_dim", None)
        self.cos, self.sin = _freqs_tables(indexer.freqs_cis, self.device)
        self._alloc_decode_tensors()

    def _alloc_decode_tensors(self):
        self._score = None
        self.status = torch.zeros(1, dtype=I32, device=self.device)

    def _score_buf(self, B: int, T: int) -> torch.Tensor:
        if self._score is None or self._score.shape[0] < B or self._score.shape[1] != T:
            self._score = torch.zeros(B, T, dtype=F32, device=self.device)
        return self._score[:B]

    def forward_device_score(self, x_tt, qr_tt, B: int, start_pos: int, start_pos_tt, t_valid=None):
        """Returns score [B, 1, T] fp32 over every row of the indexer cache
        (inference.py:5226-5275).  ``t_valid`` ([B] int32 device, optional)
        skips rows at or past it - they are masked by the top-k anyway."""
        if start_pos_tt is None:
            raise ValueError("DeviceIndexer.forward_device_score requires start_pos_tt "
                             "(no host->device upload inside the trace body).")
        H, Di, rd = self.n_heads, self.head_dim, self.rope_head_dim
        pos = self.dc._pos_for(start_pos_tt, B)
        # wq_b with the q rotary in its epilogue (the Lk-D-idx-q fusion)
        q = self.wq_b.forward_device(qr_tt.reshape(B, -1), rope=(self.cos, self.sin, pos, Di, rd),
                                     status=self.status).reshape(B, H * Di)
        self.dc.forward_device(x_tt, B, start_pos, start_pos_tt)
        w = self.weights_proj.forward_device(x_tt).reshape(B, H).float().contiguous()
        return self.score_rows(q, w, B, t_valid)

    def score_rows(self, q_roped, w, B: int, t_valid=None):
        """The score stage after the projections and the compressor step:
        q_roped [B, H*Di] bf16 (wq_b output with the q rotary), w [B, H] fp32
        (weights_proj with its scale).  Returns score [B, 1, T]."""
        H, Di = self.n_heads, self.head_dim
        cache = self.dc.kv_cache_tt
        T = cache.shape[1]
        score = self._score_buf(B, T)
        ops.indexer_score(q_roped.reshape(B, H, Di).contiguous(), cache, w.reshape(B, H).float().contiguous(), T,
                          out=score, t_valid=t_valid)
        return score.view(B, 1, T)


# --------------------------------------------------------------------------
# the attention block
# --------------------------------------------------------------------------

class DeviceAttention(torch.nn.Module):
    """Decode attention block on the device (inference.py:5278-6127):
    q path, Lk-D1 kv path with the window write, window + indexer top-k
    indices, the attention compressor and sparse attention, then the output
    side (inverse rotary, grouped wo_a, wo_b).

    ``attn`` is the CPU Attention (inference.py:576-623).  Its compressor
    and indexer get device twins here unless ``attn._device_compressor`` /
    ``attn._device_indexer`` are already bound (the reference binds them in
    offload_compressor_indexer).  ``q_norm_dev`` / ``kv_norm_dev`` may be
    None (gammas then come from attn.q_norm / attn.kv_norm)."""

    def __init__(self, mesh, attn, sparse_attn_dev: DeviceSparseAttn | None = None, q_norm_dev=None,
                 kv_norm_dev=None, wo_a_cpu_weight: torch.Tensor | None = None, max_seq_len: int | None = None):
        super().__init__()
        dev = self.device = _device_of(mesh)
        self.attn = attn
        self.dim = int(attn.dim)
        self.n_heads = int(attn.n_local_heads)
        self.n_local_heads = self.n_heads
        self.head_dim = int(attn.head_dim)
        self.rope_head_dim = int(attn.rope_head_dim)
        self.q_lora_rank = int(attn.q_lora_rank)
        self.n_groups = int(attn.n_local_groups)
        self.o_lora_rank = int(attn.o_lora_rank)
        self.softmax_scale = float(attn.softmax_scale)
        self.eps = float(attn.eps)
        self.window_size = int(attn.window_size)
        self.compress_ratio = int(attn.compress_ratio or 0)
        self.cos, self.sin = _freqs_tables(attn.freqs_cis, dev)
        self.max_seq_len = int(max_seq_len or self.cos.shape[0])
        if sparse_attn_dev is None:
            sparse_attn_dev = DeviceSparseAttn(dev, attn.attn_sink, self.softmax_scale)
        self.sparse_attn_dev = sparse_attn_dev
        self.q_norm_gamma = _gamma_of(q_norm_dev, getattr(attn, "q_norm", None)).to(dev).contiguous()
        self.kv_norm_gamma = _gamma_of(kv_norm_dev, getattr(attn, "kv_norm", None)).to(dev).contiguous()
        self.wq_a = DeviceLinear(dev, attn.wq_a)
        self.wq_b = DeviceLinear(dev, attn.wq_b)
        self.wkv = DeviceLinear(dev, attn.wkv)
        self.wo_b = DeviceLinear(dev, attn.wo_b)
        wo_a = weight_bf16(wo_a_cpu_weight if wo_a_cpu_weight is not None else attn.wo_a)
        out_total, in_per_group = wo_a.shape
        if out_total != self.n_groups * self.o_lora_rank:
            raise ValueError(f"wo_a shape {tuple(wo_a.shape)} != expected "
                             f"({self.n_groups * self.o_lora_rank}, in_per_group)")
        if in_per_group * self.n_groups != self.n_heads * self.head_dim:
            raise ValueError(f"wo_a in_per_group {in_per_group} * groups {self.n_groups} != "
                             f"heads*head_dim {self.n_heads * self.head_dim}")
        self.wo_a_in_per_group = in_per_group
        # [G, in, R] so that o [G, B, in] @ w -> [G, B, R]
        # [G*R, in_per_group], tiled for the projection kernel: group g reads
        # columns [g in_per_group, (g+1) in_per_group) of o
        self.wo_a_w = ops.pack_linear_weight(wo_a.contiguous().to(dev), groups=self.n_groups)
        kv_shape = tuple(attn.kv_cache.shape)
        if len(kv_shape) != 3:
            raise ValueError(f"expected attn.kv_cache to be 3D [B, kv_cache_size, D], got {kv_shape}")
        if kv_shape[2] != self.head_dim:
            raise ValueError(f"attn.kv_cache last dim {kv_shape[2]} != head_dim {self.head_dim}")
        self.kv_cache_size = kv_shape[1]
        made_comp = made_ind = False
        if self.compress_ratio:
            if getattr(attn, "_device_compressor", None) is None:
                comp = attn.compressor
                attn._device_compressor = DeviceCompressor(
                    dev, comp, DeviceLinear(dev, comp.wkv), DeviceLinear(dev, comp.wgate), None)
                made_comp = True
            ind = getattr(attn, "indexer", None)
            if ind is not None and getattr(attn, "_device_indexer", None) is None:
                ic = ind.compressor
                idc = DeviceCompressor(dev, ic, DeviceLinear(dev, ic.wkv), DeviceLinear(dev, ic.wgate), None)
                attn._device_indexer = DeviceIndexer(dev, ind, idc)
                made_ind = True
        # The projections that read the same input run as one launch each
        # when this block built its compressor and indexer twins from the CPU
        # modules (their weights are then known): x -> wq_a | wkv | compressor
        # wkv | wgate | indexer compressor wkv | wgate | weights_proj (scaled
        # as DeviceIndexer scales it), and q_lora -> wq_b | indexer wq_b with
        # the indexer's q rotary on its columns.  Same values as the separate
        # projections (each output column is the same dot product).
        self._merged = None
        if made_comp and made_ind:
            self._merged = self._merge_projections(dev, attn, attn.compressor, attn.indexer)
        di = self.device_indexer
        # the indexer's compressor writes into the indexer's own key cache
        # (inference.py:5113-5122) unless it was given one
        self._bind_indexer_cache = (di is not None and di.dc._owns_kv_cache
                                    and getattr(di.dc.comp, "kv_cache", None) is None)
        self.kv_cache_tt = None
        self._indexer_score_in_tt = None
        self._alloc_decode_tensors()

    def _merge_projections(self, dev, attn, comp, ind):
        ic = ind.compressor
        wscale = float(ind.softmax_scale) * int(ind.n_heads) ** -0.5
        wproj = (weight_bf16(ind.weights_proj).float() * wscale).to(BF16)
        xs = [weight_bf16(attn.wq_a), weight_bf16(attn.wkv), weight_bf16(comp.wkv), weight_bf16(comp.wgate),
              weight_bf16(ic.wkv), weight_bf16(ic.wgate), wproj]
        qs = [weight_bf16(attn.wq_b), weight_bf16(ind.wq_b)]
        if len({w.shape[1] for w in xs}) != 1 or len({w.shape[1] for w in qs}) != 1:
            return None
        cuts = [0]
        for w in xs:
            cuts.append(cuts[-1] + w.shape[0])
        return {"x": ops.pack_linear_weight(torch.cat(xs, 0).to(dev).contiguous()), "x_cuts": cuts,
                "q": ops.pack_linear_weight(torch.cat(qs, 0).to(dev).contiguous()), "q_cut": qs[0].shape[0]}

    @property
    def device_compressor(self):
        return getattr(self.attn, "_device_compressor", None)

    @property
    def device_indexer(self):
        return getattr(self.attn, "_device_indexer", None)

    def _alloc_decode_tensors(self, B: int = 1):
        """Joint window+compressed cache [B, W + T, D] and the staged
        per-step device scalars (inference.py:5460-5580)."""
        dev = self.device
        self.kv_cache_tt = self.attn.kv_cache[:B].detach().to(BF16).contiguous().to(dev)
        self._pos_tt = torch.zeros(B, dtype=I32, device=dev)
        self._t_active_tt = torch.zeros(B, dtype=I32, device=dev)
        self.status = torch.zeros(1, dtype=I32, device=dev)
        dc = self.device_compressor
        if dc is not None:
            dc.bind_kv_cache_tt(self.kv_cache_tt, self.window_size)
            dc._alloc_decode_tensors(B)
        di = self.device_indexer
        if di is not None:
            if self._bind_indexer_cache:
                di.dc.bind_kv_cache_tt(self.attn.indexer.kv_cache[:B].detach().to(BF16).contiguous().to(dev), 0)
            di.dc._alloc_decode_tensors(B)
        self.B = B

    def pre_stage_decode(self, start_pos: int, B: int = 1, S: int = 1):
        """Stage this step's integers on the device for this layer and its
        compressor / indexer (inference.py:5853-5885)."""
        if S != 1:
            raise RuntimeError(f"DeviceAttention decodes one token per step; got S={S}")
        if self.B != B:
            self._alloc_decode_tensors(B)
        self._start_pos = int(start_pos)
        self._pos_tt.fill_(int(start_pos))
        if self.compress_ratio:
            self._t_active_tt.fill_((int(start_pos) + 1) // self.compress_ratio)
        dc = self.device_compressor
        if dc is not None:
            dc.pre_stage_decode(start_pos, B=B)
        di = self.device_indexer
        if di is not None:
            di.dc.pre_stage_decode(start_pos, B=B)

    def _indexer_topk_body(self, bucket: int, k_fixed: int, win: int, B: int, S: int, mask_mode: int = 0):
        """Top-k over the first ``bucket`` staged scores with the additive
        -1e4 mask at t >= T_active; returns int32 [B, S, k_fixed] holding
        idx + win, -1 where the masked score is below -1000, in descending
        score order (inference.py:5823-5851).  ``mask_mode=1`` treats
        t >= T_active as -inf without reading those scores (same result
        unless a score exceeds 9000); forward_device uses it because its
        score stage skips those rows."""
        if self._indexer_score_in_tt is None:
            raise RuntimeError("indexer scores not staged; run the indexer score stage first")
        if S != 1:
            raise ValueError(f"decode top-k is per token; got S={S}")
        score = self._indexer_score_in_tt.reshape(B, -1)
        if bucket > score.shape[1] or k_fixed > bucket:
            raise ValueError(f"bucket {bucket} / k {k_fixed} exceed the {score.shape[1]} staged scores")
        out = ops.indexer_topk(score, self._t_active_tt, k_fixed, win, T=bucket, sort_desc=True,
                               mask_mode=mask_mode)
        return out.view(B, S, k_fixed)

    def forward(self, x: torch.Tensor, start_pos: int) -> torch.Tensor:
        """Single-token host forward: upload, forward_device, download."""
        bsz, seqlen, _ = x.shape
        if seqlen != 1:
            raise RuntimeError(f"DeviceAttention expects seqlen=1; got seqlen={seqlen}. "
                               "Prefill must loop one token at a time.")
        self.pre_stage_decode(start_pos, B=bsz, S=1)
        out = self.forward_device(x.to(self.device, BF16), start_pos, self._pos_tt)
        return out.to(x.device, x.dtype)

    def forward_device(self, x_tt, start_pos: int, start_pos_tt, wq_a_out_tt=None):
        """x_tt [B, 1, dim] bf16 -> out [B, 1, dim] bf16 (inference.py:5888-6127)."""
        if start_pos_tt is None:
            raise ValueError("DeviceAttention.forward_device requires start_pos_tt "
                             "(no host->device upload inside the trace body).")
        B = int(x_tt.shape[0])
        H, D, rd, W = self.n_heads, self.head_dim, self.rope_head_dim, self.window_size
        dc, di = self.device_compressor, self.device_indexer
        if self.compress_ratio and dc is None:
            raise RuntimeError("DeviceAttention.forward_device requires attn._device_compressor "
                               "when compress_ratio is set.")
        pos = self._pos_tt if not (isinstance(start_pos_tt, torch.Tensor) and start_pos_tt.numel() == B
                                   and start_pos_tt.dtype == I32 and start_pos_tt.is_cuda) else start_pos_tt
        x2 = x_tt.reshape(B, self.dim)
        mg = self._merged if wq_a_out_tt is None and di is not None and dc is not None else None
        if mg is not None:
            # the projections of x in one launch; slices are strided views
            xp = ops.linear(x2.to(BF16).contiguous(), mg["x"])
            c = mg["x_cuts"]
            q_lora, kv = xp[:, c[0]:c[1]], xp[:, c[1]:c[2]]
            c_rows = (xp[:, c[2]:c[3]], xp[:, c[3]:c[4]])
            i_rows = (xp[:, c[4]:c[5]], xp[:, c[5]:c[6]])
            iw = xp[:, c[6]:c[7]]
            qr = ops.head_norm_rope(q_lora, 1, self.q_lora_rank, gamma=self.q_norm_gamma, eps=self.eps)
            # wq_b and the indexer's wq_b in one launch, the indexer q rotary on its columns
            ipos = di.dc._pos_for(pos, B)
            qp = ops.linear(qr, mg["q"], rope=(di.cos, di.sin, ipos, di.head_dim, di.rope_head_dim, mg["q_cut"]),
                            status=di.status)
            q = ops.head_norm_rope(qp[:, :mg["q_cut"]], H, D, self.cos, self.sin, pos, rope_dim=rd,
                                   weight=self.softmax_scale, eps=self.eps, status=self.status)
            iq = qp[:, mg["q_cut"]:]
        else:
            # q path: wq_a -> q_norm -> wq_b -> per-head rms (weight = softmax_scale) -> rotary
            q_lora = wq_a_out_tt.reshape(B, self.q_lora_rank) if wq_a_out_tt is not None else self.wq_a(x2)
            qr = ops.head_norm_rope(q_lora, 1, self.q_lora_rank, gamma=self.q_norm_gamma, eps=self.eps)
            q = self.wq_b(qr)
            ops.head_norm_rope(q, H, D, self.cos, self.sin, pos, rope_dim=rd, weight=self.softmax_scale,
                               eps=self.eps, out=q, status=self.status)
        # kv path + window write (Lk-D1 + attn.kv_update)
        if mg is None:
            kv = self.wkv(x2)
        ops.kv_norm_rope_window_write(kv, self.kv_norm_gamma, self.cos, self.sin, pos, self.kv_cache_tt, W,
                                      eps=self.eps, rope_dim=rd, status=self.status)
        # indices: window ring, then the indexer's top-k
        win_idx = ops.window_indices(pos, W)
        parts = [win_idx]
        T_active = (start_pos + 1) // self.compress_ratio if self.compress_ratio else 0
        if self.compress_ratio and T_active > 0:
            if di is not None:
                if mg is not None:
                    di.dc.step_rows(i_rows[0], i_rows[1], B, start_pos, pos)
                    score = di.score_rows(iq, iw, B, t_valid=self._t_active_tt)
                else:
                    score = di.forward_device_score(x2, qr, B, start_pos, pos, t_valid=self._t_active_tt)
                self._indexer_score_in_tt = score
                bucket = min(pick_indexer_topk_bucket(T_active), score.shape[-1])
                k_fixed = min(di.index_topk, bucket)
                parts.append(self._indexer_topk_body(bucket, k_fixed, W, B, 1, mask_mode=1).view(B, k_fixed))
            else:
                ramp = torch.arange(W, W + T_active, dtype=I32, device=self.device)
                parts.append(ramp.unsqueeze(0).expand(B, T_active))
        idx = torch.cat(parts, dim=-1).contiguous() if len(parts) > 1 else win_idx
        if self.compress_ratio:
            if mg is not None:
                dc.step_rows(c_rows[0], c_rows[1], B, start_pos, pos)
            else:
                dc.forward_device(x2, B, start_pos, pos)
        K = idx.shape[-1]
        idxs_tt, valid_tt = self.sparse_attn_dev._idxs_int_tile_to_idxs_and_mask(idx, B, 1, K)
        o = self.sparse_attn_dev.forward_device(q.view(B, 1, H, D), self.kv_cache_tt, idxs_tt, valid_tt, 1, K)
        # output side: inverse rotary, grouped wo_a, wo_b
        ops.head_norm_rope(o, H, D, self.cos, self.sin, pos, rope_dim=rd, norm=False, inverse=True, out=o,
                           status=self.status)
        # head-grouped wo_a: group g of o (its heads' dims) against its R rows
        a = ops.linear(o.reshape(B, H * D), self.wo_a_w)
        return self.wo_b(a).view(B, 1, self.dim)
