"""The per-layer decode sparse-attention path, device-resident and graph-capturable.

``DecodeLayer`` owns one attention layer's persistent decode state for B
sequences (the buffers DeviceAttention / DeviceCompressor / DeviceIndexer
allocate in the reference, inference.py:4757-4813, 5460-5580):

* ``kv_cache``  [B, W + T_max, D] bf16 - raw-token window ring (rows 0..W-1)
  followed by the compressed rows (W + pos // r), inference.py:611-614;
* ``idx_cache`` [B, T_max, Di] bf16 - the indexer's compressed keys;
* compressor states (fp32, the CPU layout of inference.py:538-551) for the
  attention compressor (d = D) and the indexer compressor (d = Di);
* the per-step scratch it needs: indexer scores [B, T_max] fp32, the joint
  index list [B, W + k] int32 (window ring slots, then compressed rows) and
  the split-K workspace of the attention kernel.

``DecodePath`` runs one decode step over a stack of layers in the
reference's order (inference.py:5888-6093):

    attn.topk        indexer_score        relu-weighted multi-head scores
    (prologue)       layer_prologue       the indexer compressor (emit on
                                          device) and the newest row's score;
                                          attn.kv act_quant(nope) + ring
                                          write; the window's ring slots;
                                          attn.compress (emit on device)
    attn.topk        indexer_topk         k best compressed rows (+W, -1)
    attn.sparse      sparse_attn          gather + sink softmax attention

and then advances the device-resident positions, so a captured CUDA graph
of the whole step can be replayed without any host work (the reference
needs two traces and host staging per step, inference.py:7498-7543).  The
four kernels of a layer form one chain of programmatic dependent launches
on one stream.  The score covers the compressed rows before the newest;
the prologue (dsa_layer_prologue), which writes at most the newest row and
that row's score, runs beside it and completes after it; the top-k then
finds every live score in place -- the same selection as scoring after the
compressor, with the compressors and the small stages off the critical
path.  (Side streams joined before the top-k and the attention turned
those programmatic launches into full dependencies, ~4 us each.)
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from .tables import PathArgs, rope_cos_sin

BF16 = torch.bfloat16
F32 = torch.float32
I32 = torch.int32


@dataclass
class LayerInputs:
    """Per-step inputs of one layer (the projections that produce them are
    outside the path): q [B,H,D] (already softmax-scaled or not, see
    DecodePath.scale), kv [B,D] (kv_norm'ed + rotated latent row),
    cmp_kv/cmp_score [B,2D] (attention compressor wkv/wgate rows),
    iq [B,Hi,Di] (indexer q after rotary), icmp_kv/icmp_score [B,2Di],
    iw [B,Hi] fp32 (weights_proj output, already scaled)."""
    q: torch.Tensor
    kv: torch.Tensor
    cmp_kv: torch.Tensor
    cmp_score: torch.Tensor
    iq: torch.Tensor
    icmp_kv: torch.Tensor
    icmp_score: torch.Tensor
    iw: torch.Tensor

    @staticmethod
    def empty(args: PathArgs, B: int, device, pin: bool = False) -> "LayerInputs":
        kw = dict(device=device)
        if pin:
            kw = dict(pin_memory=True)
        D, Di = args.head_dim, args.index_head_dim
        return LayerInputs(
            q=torch.empty(B, args.n_heads, D, dtype=BF16, **kw),
            kv=torch.empty(B, D, dtype=BF16, **kw),
            cmp_kv=torch.empty(B, 2 * D, dtype=BF16, **kw),
            cmp_score=torch.empty(B, 2 * D, dtype=BF16, **kw),
            iq=torch.empty(B, args.index_n_heads, Di, dtype=BF16, **kw),
            icmp_kv=torch.empty(B, 2 * Di, dtype=BF16, **kw),
            icmp_score=torch.empty(B, 2 * Di, dtype=BF16, **kw),
            iw=torch.empty(B, args.index_n_heads, dtype=F32, **kw))

    @staticmethod
    def shapes(args: PathArgs, B: int):
        """(shape, dtype) of each input tensor, in field order."""
        D, Di, H, Hi = args.head_dim, args.index_head_dim, args.n_heads, args.index_n_heads
        return [((B, H, D), BF16), ((B, D), BF16), ((B, 2 * D), BF16), ((B, 2 * D), BF16),
                ((B, Hi, Di), BF16), ((B, 2 * Di), BF16), ((B, 2 * Di), BF16), ((B, Hi), F32)]

    @staticmethod
    def packed(args: PathArgs, B: int, n_layers: int, device=None, pin: bool = False):
        """Inputs of n_layers layers as views of ONE flat byte buffer (so a
        host->device refresh of a whole step is a single copy).  Returns
        (flat uint8 tensor, [LayerInputs] views)."""
        sh = LayerInputs.shapes(args, B)
        sizes = []
        for shape, dt in sh:
            n = 1
            for x in shape:
                n *= x
            sizes.append(-(-n * torch.tensor([], dtype=dt).element_size() // 256) * 256)
        per_layer = sum(sizes)
        kw = dict(pin_memory=True) if pin else dict(device=device)
        flat = torch.empty(n_layers * per_layer, dtype=torch.uint8, **kw)
        layers = []
        for li in range(n_layers):
            off = li * per_layer
            ts = []
            for (shape, dt), nb in zip(sh, sizes):
                esz = torch.tensor([], dtype=dt).element_size()
                n = 1
                for x in shape:
                    n *= x
                ts.append(flat[off:off + n * esz].view(dt).view(shape))
                off += nb
            layers.append(LayerInputs(*ts))
        return flat, layers

    def tensors(self):
        return [self.q, self.kv, self.cmp_kv, self.cmp_score, self.iq, self.icmp_kv, self.icmp_score, self.iw]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors())

    def copy_(self, other: "LayerInputs", non_blocking: bool = True) -> None:
        for a, b in zip(self.tensors(), other.tensors()):
            a.copy_(b, non_blocking=non_blocking)


class DecodeLayer:
    """Persistent device state of one compressed (ratio 4) attention layer."""

    def __init__(self, args: PathArgs, B: int, max_seq_len: int, device, index_topk: int | None = None):
        self.args = args
        self.B = B
        self.device = torch.device(device)
        self.win = args.window_size
        self.ratio = args.compress_ratio
        self.k = index_topk if index_topk is not None else args.index_topk
        self.T_max = max_seq_len // self.ratio
        if self.k > self.T_max:
            raise ValueError(f"index_topk {self.k} > compressed capacity {self.T_max}")
        D, Di, r = args.head_dim, args.index_head_dim, self.ratio
        dev = self.device
        self.kv_cache = torch.zeros(B, self.win + self.T_max, D, dtype=BF16, device=dev)
        self.idx_cache = torch.zeros(B, self.T_max, Di, dtype=BF16, device=dev)
        self.cmp_kv = torch.zeros(B, 2 * r, 2 * D, dtype=F32, device=dev)
        self.cmp_sc = torch.full((B, 2 * r, 2 * D), float("-inf"), dtype=F32, device=dev)
        self.icmp_kv = torch.zeros(B, 2 * r, 2 * Di, dtype=F32, device=dev)
        self.icmp_sc = torch.full((B, 2 * r, 2 * Di), float("-inf"), dtype=F32, device=dev)
        # parameters (random-init by the caller or loaded)
        self.ape = torch.zeros(r, 2 * D, dtype=F32, device=dev)
        self.gamma = torch.ones(D, dtype=F32, device=dev)
        self.iape = torch.zeros(r, 2 * Di, dtype=F32, device=dev)
        self.igamma = torch.ones(Di, dtype=F32, device=dev)
        self.sink = torch.zeros(args.n_heads, dtype=F32, device=dev)
        # per-step scratch
        self.score = torch.zeros(B, self.T_max, dtype=F32, device=dev)
        self.idx = torch.full((B, self.win + self.k), -1, dtype=I32, device=dev)
        self.ws = ops.Workspace(dev, max(
            int(ops.lib().dsa_sparse_attn_workspace_size(B, 1, args.n_heads, D, self.win + self.k)),
            int(ops.lib().dsa_indexer_topk_workspace_size(B, self.T_max, self.k))))

    def nbytes(self) -> int:
        ts = [self.kv_cache, self.idx_cache, self.cmp_kv, self.cmp_sc, self.icmp_kv, self.icmp_sc, self.score,
              self.idx]
        return sum(t.numel() * t.element_size() for t in ts) + self.ws.nbytes


class DecodePath:
    """Runs the four-stage decode path over a stack of layers for B sequences
    at device-resident positions ``pos`` (all layers share them)."""

    def __init__(self, layers: list[DecodeLayer], max_seq_len: int, scale: float | None = None):
        if not layers:
            raise ValueError("need at least one layer")
        self.layers = layers
        a = layers[0].args
        self.args = a
        self.B = layers[0].B
        self.device = layers[0].device
        self.scale = a.softmax_scale if scale is None else scale
        self.cos, self.sin = rope_cos_sin(a, max_seq_len, compressed=True, device=self.device)
        self.pos = torch.zeros(self.B, dtype=I32, device=self.device)
        self.t_active = torch.zeros(self.B, dtype=I32, device=self.device)
        # t_active - 1: the indexer scores the rows before the newest, which
        # the indexer compressor may write in the same step (the prologue
        # scores that one row after its compressor)
        self.t_prev = torch.zeros(self.B, dtype=I32, device=self.device)
        self.status = torch.zeros(1, dtype=I32, device=self.device)
        # the indexer score's dynamic work split (claimed items, CTAs done):
        # zero, and left zero by every call; the layers run one at a time
        self.score_counters = torch.zeros(2, dtype=I32, device=self.device)
        self.graph = None

    def set_positions(self, pos) -> None:
        """Stage the current decode position(s) (pre_stage_decode,
        inference.py:5853); ``pos`` int or [B]."""
        p = torch.as_tensor(pos, dtype=I32).reshape(-1).expand(self.B).contiguous()
        self.pos.copy_(p.to(self.device, non_blocking=False))
        self.t_active.copy_(((p + 1) // self.args.compress_ratio).to(self.device))
        ops.shard_active(self.t_active, 1, 1 << 30, out=self.t_prev)

    def layer_step(self, L: DecodeLayer, x: LayerInputs, out: torch.Tensor) -> None:
        a = self.args
        W, r = L.win, L.ratio
        # One stream, every hand-over a programmatic dependent launch:
        #   indexer score -> prologue -> top-k -> attention.
        # attn.topk's score covers the compressed rows before the newest
        # (t_prev = t_active - 1).  keys_ready: the rows it scores were
        # written by earlier steps and t_prev before the first layer, so from
        # the second layer on its first key tiles are requested before the
        # previous layer's last kernel ends (the first layer may directly
        # follow the kernel that writes t_prev).
        # The work split is dynamic: CTAs placed late, on SMs the previous
        # layer's attention still held, take fewer items.
        ops.indexer_score(x.iq, L.idx_cache, x.iw, L.T_max, out=L.score, t_valid=self.t_prev,
                          keys_ready=L is not self.layers[0], counters=self.score_counters)
        # The prologue: the indexer compressor (it may write row t_active - 1
        # of the indexer cache) and that row's score, the window-ring KV
        # write (attn.kv), the window indices and attn.compress.  None of it
        # touches what the score reads or writes, so it runs beside the
        # score and waits for it only before completing: the top-k, which
        # waits for the prologue, sees every live score in place.
        ops.layer_prologue((x.icmp_kv, x.icmp_score, L.iape, L.icmp_kv, L.icmp_sc, L.igamma, L.idx_cache),
                           (x.cmp_kv, x.cmp_score, L.ape, L.cmp_kv, L.cmp_sc, L.gamma, L.kv_cache),
                           self.cos, self.sin, self.pos, self.t_active, x.iq, x.iw, L.score, L.T_max, x.kv, L.idx,
                           W, r, eps=a.norm_eps, rope_dim=a.rope_head_dim, beside_previous=True)
        # the top-k writes idx[:, W:], disjoint from the window columns
        ops.indexer_topk(L.score, self.t_active, L.k, W, T=L.T_max, mask_mode=1, out=L.idx[:, W:], ws=L.ws)
        # the window columns of idx, q and the window rows were complete when
        # the attention was launched (the top-k lets it launch only after its
        # own wait, i.e. after the prologue completed): each key split
        # requests its window tile before waiting for the top-k
        ops.sparse_attn(x.q, L.kv_cache, L.idx, L.sink, self.scale, out=out, ws=L.ws, status=self.status,
                        lead_cols=W, lead_ready=True)

    def step(self, inputs: list[LayerInputs], outs: list[torch.Tensor], advance: bool = True) -> None:
        for L, x, o in zip(self.layers, inputs, outs):
            self.layer_step(L, x, o)
        if advance:
            ops.advance_positions(self.pos, self.t_active, self.args.compress_ratio, 1)
            ops.shard_active(self.t_active, 1, 1 << 30, out=self.t_prev)

    def capture(self, inputs: list[LayerInputs], outs: list[torch.Tensor], warmup: int = 1):
        """Capture ``step`` (with the position advance) in a CUDA graph.  The
        warm-up runs advance the positions; callers re-stage positions after
        capturing.  Returns the graph; ``replay()`` runs one step."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.step(inputs, outs)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step(inputs, outs)
        self.graph = g
        return g

    def replay(self) -> None:
        self.graph.replay()

    kernels_per_layer = 4  # launches per layer without a split-K combine launch

    def launches_per_step(self) -> int:
        L0 = self.layers[0]
        H, D = self.args.n_heads, self.args.head_dim
        ws = int(ops.lib().dsa_sparse_attn_workspace_size(self.B, 1, H, D, L0.win + L0.k))
        nsplit = ws // (self.B * H * (2 * 4 + D * 2)) if ws else 1
        # a row's two key splits combine inside the attention; more need the
        # combine launch
        extra = 1 if nsplit > 2 else 0
        topk2 = 1 if ops.lib().dsa_indexer_topk_workspace_size(self.B, L0.T_max, L0.k) else 0
        n = len(self.layers) * (self.kernels_per_layer + extra + topk2)
        return n + 2  # + the position advance and t_prev
